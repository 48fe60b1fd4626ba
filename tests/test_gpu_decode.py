"""CUDA parity of the device decode step.

Glue kernels: each against a plain torch fp32 restatement of the reference op
(tolerance 1e-4 * max|ref| per output, fp32 accumulation-order differences
only). Engine: greedy tokens identical to those quartz itself produced on the
same seeded synthetic checkpoints (tests/golden/golden_model.npz), eager and
CUDA-graph replay, prompt prefill and prefilled-cache starts.
"""

import json
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

HERE = Path(__file__).resolve().parent
TOL = 1e-4


@pytest.fixture(scope="module", autouse=True)
def _clean_status():
    from quartz_b200 import device
    if torch.cuda.is_available():
        device.status(clear=True)
    yield
    if torch.cuda.is_available():
        device.check_status()


def _close(got, ref, what=""):
    got = got.detach().double().cpu()
    ref = ref.detach().double().cpu()
    inf = float(ref.abs().max()) if ref.numel() else 0.0
    err = float((got - ref).abs().max()) if ref.numel() else 0.0
    assert np.isfinite(err) and err <= TOL * max(inf, 1e-30), f"{what}: err {err:.3e}, |ref| {inf:.3e}"


# ------------------------------------------------------------ torch references
def _rms_ref(x, w, eps):
    x = x.double()
    return (x / torch.sqrt((x * x).mean(-1, keepdim=True) + eps) * w.double()).float()


def _rope_ref(x, pos, inv_freq):
    # half-split rotation at positions pos (quartz/rope.py:36-78); x [..., seq, D]
    # the angle is an fp32 product, as in the reference; cos/sin in fp64
    d = x.shape[-1] // 2
    ang = (pos.float()[:, None] * inv_freq.float()[None, :]).double()
    c, s = torch.cos(ang), torch.sin(ang)
    x1, x2 = x[..., :d].double(), x[..., d:].double()
    return torch.cat([x1 * c - x2 * s, x2 * c + x1 * s], -1).float()


def _sdpa_ref(q, k, v, scale, n_rep, mask=None):
    # q [nq, Lq, D], k/v [nkv, Lk, D] (quartz/attention.py:29-43)
    k = k.double().repeat_interleave(n_rep, 0)
    v = v.double().repeat_interleave(n_rep, 0)
    s = q.double() @ k.transpose(-1, -2) * scale
    if mask is not None:
        s = s + mask
    return (torch.softmax(s, -1) @ v).float()


# ------------------------------------------------------------------ glue ops
@pytest.mark.parametrize("rows,n", [(1, 1024), (3, 2048), (7, 64), (1, 1), (2, 4097)])
def test_rmsnorm(cuda_dev, rows, n):
    from quartz_b200 import device as qd
    g = torch.Generator().manual_seed(rows * 131 + n)
    x = torch.randn(rows, n, generator=g).to(cuda_dev)
    w = (1 + 0.1 * torch.randn(n, generator=g)).to(cuda_dev)
    _close(qd.rmsnorm(x, w, 1e-6), _rms_ref(x, w, 1e-6), f"rmsnorm {rows}x{n}")


@pytest.mark.parametrize("V,H,ng", [(1000, 64, 1), (151936, 1024, 1), (257, 96, 3)])
def test_embed_gather(cuda_dev, V, H, ng):
    from quartz_b200 import device as qd
    g = torch.Generator().manual_seed(V)
    q = torch.randint(-127, 128, (V, H), generator=g, dtype=torch.int8).to(cuda_dev)
    s = (torch.rand(V, ng, generator=g) * 0.01 + 1e-4).to(cuda_dev)
    ids = torch.tensor([0, V - 1, 5, V // 2, 5], dtype=torch.int64, device=cuda_dev)
    out = qd.embed_gather(q, s, ids)
    ref = (q.float().view(V, ng, H // ng) * s[:, :, None]).view(V, H)[ids]
    assert torch.equal(out, ref)


@pytest.mark.parametrize("qk_norm", [True, False])
@pytest.mark.parametrize("nq,nkv,hd,M,pos0", [(16, 8, 128, 1, 512), (4, 2, 16, 5, 0),
                                              (32, 8, 64, 7, 1000), (8, 8, 256, 2, 3)])
def test_qk_rope(cuda_dev, qk_norm, nq, nkv, hd, M, pos0):
    from quartz_b200 import device as qd
    from quartz_b200.model import ModelSpec, rope_inv_freq, LLAMA3_SCALING
    g = torch.Generator().manual_seed(nq * hd + M)
    max_ctx = pos0 + M + 3
    spec = ModelSpec(arch="LlamaForCausalLM", hidden=64, layers=1, n_heads=nq, n_kv=nkv,
                     head_dim=hd, inter=64, vocab=8, rope_theta=5e5, tie=True,
                     rope_scaling=None if qk_norm else LLAMA3_SCALING)
    inv = torch.from_numpy(rope_inv_freq(spec)).to(cuda_dev)
    qkv = torch.randn(M, (nq + 2 * nkv) * hd, generator=g).to(cuda_dev)
    qn = (1 + 0.1 * torch.randn(hd, generator=g)).to(cuda_dev) if qk_norm else None
    kn = (1 + 0.1 * torch.randn(hd, generator=g)).to(cuda_dev) if qk_norm else None
    kc = torch.zeros(nkv, max_ctx, hd, device=cuda_dev)
    vc = torch.zeros(nkv, max_ctx, hd, device=cuda_dev)
    q = qd.qk_rope(qkv, inv, kc, vc, nq, pos0=pos0, q_norm=qn, k_norm=kn)
    parts = qkv.view(M, nq + 2 * nkv, hd)
    qh, kh, vh = parts[:, :nq], parts[:, nq:nq + nkv], parts[:, nq + nkv:]
    if qk_norm:
        qh, kh = _rms_ref(qh, qn, 1e-6), _rms_ref(kh, kn, 1e-6)
    pos = torch.arange(pos0, pos0 + M, device=cuda_dev, dtype=torch.float32)
    qr = _rope_ref(qh.transpose(0, 1), pos, inv).transpose(0, 1).reshape(M, nq * hd)
    kr = _rope_ref(kh.transpose(0, 1), pos, inv)               # [nkv, M, hd]
    _close(q, qr, "q")
    _close(kc[:, pos0:pos0 + M], kr, "k cache")
    assert torch.equal(vc[:, pos0:pos0 + M], vh.transpose(0, 1))
    assert float(kc[:, :pos0].abs().sum()) == 0.0 and float(kc[:, pos0 + M:].abs().sum()) == 0.0


@pytest.mark.parametrize("nq,nkv,hd,T,max_ctx", [(16, 8, 128, 513, 1024), (4, 2, 16, 1, 40),
                                                 (32, 8, 64, 64, 64), (8, 1, 128, 65, 200),
                                                 (8, 8, 256, 300, 301), (16, 4, 256, 700, 4096),
                                                 (64, 8, 128, 5000, 8192), (6, 2, 96, 100, 128),
                                                 (16, 2, 256, 33, 64)])
def test_attention_decode(cuda_dev, nq, nkv, hd, T, max_ctx):
    from quartz_b200 import device as qd
    g = torch.Generator().manual_seed(T * 7 + hd)
    q = torch.randn(nq * hd, generator=g).to(cuda_dev)
    kc = torch.randn(nkv, max_ctx, hd, generator=g).to(cuda_dev)
    vc = torch.randn(nkv, max_ctx, hd, generator=g).to(cuda_dev)
    ref = _sdpa_ref(q.view(nq, 1, hd), kc[:, :T], vc[:, :T], hd ** -0.5, nq // nkv).view(-1)
    _close(qd.attention_decode(q, kc, vc, T=T), ref, "attention T")
    # device-held length (graph form): T = *T_dev + 1
    T_dev = torch.tensor([T - 1], dtype=torch.int64, device=cuda_dev)
    _close(qd.attention_decode(q, kc, vc, T_dev=T_dev, t_offset=1), ref, "attention T_dev")


@pytest.mark.parametrize("qk_norm", [True, False])
@pytest.mark.parametrize("nq,nkv,hd,pos,max_ctx", [(16, 8, 128, 512, 640), (32, 8, 64, 0, 16),
                                                   (16, 4, 256, 1000, 1001), (4, 2, 16, 39, 52),
                                                   (12, 2, 96, 70, 80)])
def test_attention_decode_qkv(cuda_dev, qk_norm, nq, nkv, hd, pos, max_ctx):
    """norm + RoPE + append + attention in one launch, against the separate ops'
    references; positions other than pos untouched."""
    from quartz_b200 import device as qd
    from quartz_b200.model import ModelSpec, rope_inv_freq
    g = torch.Generator().manual_seed(pos * 3 + hd)
    spec = ModelSpec(arch="Qwen3ForCausalLM", hidden=64, layers=1, n_heads=nq, n_kv=nkv,
                     head_dim=hd, inter=64, vocab=8, rope_theta=1e6, tie=True)
    inv = torch.from_numpy(rope_inv_freq(spec)).to(cuda_dev)
    qkv = torch.randn((nq + 2 * nkv) * hd, generator=g).to(cuda_dev)
    qn = (1 + 0.1 * torch.randn(hd, generator=g)).to(cuda_dev) if qk_norm else None
    kn = (1 + 0.1 * torch.randn(hd, generator=g)).to(cuda_dev) if qk_norm else None
    kc = torch.randn(nkv, max_ctx, hd, generator=g).to(cuda_dev)
    vc = torch.randn(nkv, max_ctx, hd, generator=g).to(cuda_dev)
    kc0, vc0 = kc.clone(), vc.clone()
    pos_dev = torch.tensor([pos], dtype=torch.int64, device=cuda_dev)
    out = qd.attention_decode_qkv(qkv, inv, kc, vc, nq, pos_dev=pos_dev, q_norm=qn, k_norm=kn)
    parts = qkv.view(nq + 2 * nkv, hd)
    qh, kh, vh = parts[:nq], parts[nq:nq + nkv], parts[nq + nkv:]
    if qk_norm:
        qh, kh = _rms_ref(qh, qn, 1e-6), _rms_ref(kh, kn, 1e-6)
    p = torch.tensor([float(pos)], device=cuda_dev)
    qr = _rope_ref(qh[:, None], p, inv)[:, 0]
    kr = _rope_ref(kh[:, None], p, inv)[:, 0]
    _close(kc[:, pos], kr, "appended k")
    assert torch.equal(vc[:, pos], vh)
    keep = [t for t in range(max_ctx) if t != pos]
    assert torch.equal(kc[:, keep], kc0[:, keep]) and torch.equal(vc[:, keep], vc0[:, keep])
    kref, vref = kc0.clone(), vc0.clone()
    kref[:, pos], vref[:, pos] = kr, vh
    ref = _sdpa_ref(qr[:, None], kref[:, :pos + 1], vref[:, :pos + 1], hd ** -0.5, nq // nkv)
    _close(out, ref.view(-1), "attention")
    # twice in a row: the workspace's tickets were left ready
    out2 = qd.attention_decode_qkv(qkv, inv, kc, vc, nq, pos_dev=pos_dev, q_norm=qn, k_norm=kn)
    _close(out2, ref.view(-1), "attention, second call")


@pytest.mark.parametrize("nq,nkv,hd,M,pos0", [(4, 2, 16, 5, 0), (32, 8, 64, 130, 0),
                                              (16, 8, 128, 9, 40), (8, 8, 256, 3, 7),
                                              (16, 2, 128, 100, 300), (8, 8, 64, 33, 0),
                                              (32, 8, 64, 512, 0), (8, 1, 128, 70, 5)])
def test_attention_prefill(cuda_dev, nq, nkv, hd, M, pos0):
    from quartz_b200 import device as qd
    g = torch.Generator().manual_seed(M * 11 + hd)
    max_ctx = pos0 + M + 5
    q = torch.randn(M, nq * hd, generator=g).to(cuda_dev)
    kc = torch.randn(nkv, max_ctx, hd, generator=g).to(cuda_dev)
    vc = torch.randn(nkv, max_ctx, hd, generator=g).to(cuda_dev)
    T = pos0 + M
    qp = torch.arange(pos0, T, device=cuda_dev)[:, None]
    kp = torch.arange(T, device=cuda_dev)[None, :]
    mask = torch.where(kp <= qp, 0.0, float("-inf")).double()
    ref = _sdpa_ref(q.view(M, nq, hd).transpose(0, 1), kc[:, :T], vc[:, :T], hd ** -0.5,
                    nq // nkv, mask)
    _close(qd.attention_prefill(q, kc, vc, pos0), ref.transpose(0, 1).reshape(M, nq * hd),
           "prefill attention")


def test_argmax(cuda_dev):
    from quartz_b200 import device as qd
    g = torch.Generator().manual_seed(5)
    V = 151936
    x = torch.randn(3, V, generator=g)
    x[1] = -x[1].abs() - 1.0               # all negative
    x[2, 77] = x[2, 99] = x[2].max() + 1   # tie: the lower index wins (np.argmax)
    x[0, V - 1] = 50.0
    got = qd.argmax(x.to(cuda_dev)).cpu()
    assert got.tolist() == [V - 1, int(np.argmax(x[1].numpy())), 77]
    pos = torch.tensor([10], dtype=torch.int64, device=cuda_dev)
    qd.argmax(x[:1].to(cuda_dev), pos_dev=pos, pos_step=3)
    assert int(pos.item()) == 13


# ------------------------------------------------------------------ the model
def _cases():
    return {c["id"]: c for c in json.loads((HERE / "golden" / "cases_model.json").read_text())["cases"]}


def _golden(cid, key):
    with np.load(HERE / "golden" / "golden_model.npz") as z:
        return z[f"{cid}__{key}"]


def _engine(case, extra_ctx=0, persistent=False, fold_norms=True):
    from quartz_b200.decode import DecodeEngine
    from quartz_b200.model import ModelSpec, cached_int8_weights, norm_weights
    spec = ModelSpec.from_hf(case["cfg"], case["arch"])
    start = case.get("kv_len") or len(case["prompt"])
    eng = DecodeEngine(spec, cached_int8_weights(spec), norm_weights(spec),
                       max_ctx=start + case["steps"] + extra_ctx,
                       max_prefill=max(2, len(case.get("prompt", [])) or 2),
                       persistent=persistent, fold_norms=fold_norms)
    return spec, eng


def _run(case, eng, graph, unroll=8):
    from quartz_b200.model import seeded_kv
    if case["start"] == "kv":
        eng.load_kv(seeded_kv(eng.spec, case["kv_len"]))
        return eng.generate(case["first"], case["steps"], graph=graph, unroll=unroll)
    t0 = eng.prefill(case["prompt"])
    return [t0] + eng.generate(t0, case["steps"] - 1, graph=graph, unroll=unroll)


@pytest.mark.parametrize("cid", ["qwen3_tiny_prompt", "llama_tiny_prompt", "qwen3_tiny_kv",
                                 "qwen3_small_kv", "llama_small_prompt"])
@pytest.mark.parametrize("persistent", [True, False])
def test_engine_small(cuda_dev, cid, persistent):
    """Greedy tokens of small models, eager and graph replay; every eager step's
    top-8 logits against the reference's (1e-4 of the largest)."""
    from quartz_b200.model import seeded_kv
    case = _cases()[cid]
    gold = _golden(cid, "tokens").tolist()
    top_ids = _golden(cid, "top_ids")
    top_vals = _golden(cid, "top_vals")
    _, eng = _engine(case, persistent=persistent)
    if persistent and case["cfg"]["head_dim"] in (64, 128):
        assert eng.persistent, "the one-launch decode kernel should take these shapes"
    if case["start"] == "kv":
        eng.load_kv(seeded_kv(eng.spec, case["kv_len"]))
        tok = case["first"]
        toks = []
    else:
        tok = eng.prefill(case["prompt"])
        toks = [tok]
        _close(eng.logits.cpu()[torch.from_numpy(top_ids[0])], torch.from_numpy(top_vals[0]),
               f"{cid} prefill logits")
    while len(toks) < case["steps"]:
        tok = eng.decode(tok)
        step = len(toks)
        _close(eng.logits.cpu()[torch.from_numpy(top_ids[step])],
               torch.from_numpy(top_vals[step]), f"{cid} step {step} logits")
        toks.append(tok)
    assert toks == gold, "eager"
    eng.reset(0)
    assert _run(case, eng, graph=True, unroll=5) == gold, "graph"


@pytest.mark.parametrize("persistent,fold_norms", [(True, True), (False, True), (False, False)])
def test_engine_qwen3_0p6b_kv512(cuda_dev, persistent, fold_norms):
    """The all-int8 Qwen3-0.6B decode workload: 512 prefilled positions, 128
    greedy tokens through the graph replay; the first step's top-8 logits too.
    Per-op engine with the RMSNorms folded into the GEMVs and as launches of
    their own."""
    case = _cases()["qwen3_0p6b_kv512"]
    gold = _golden(case["id"], "tokens").tolist()
    spec, eng = _engine(case, persistent=persistent, fold_norms=fold_norms)
    assert eng.persistent == persistent
    from quartz_b200.model import seeded_kv
    eng.load_kv(seeded_kv(spec, case["kv_len"]))
    first = eng.generate(case["first"], 1, graph=False)
    top_ids = torch.from_numpy(_golden(case["id"], "top_ids")[0])
    top_vals = torch.from_numpy(_golden(case["id"], "top_vals")[0])
    _close(eng.logits.cpu()[top_ids], top_vals, "step-0 top-8 logits")
    eng.reset(case["kv_len"])
    toks = eng.generate(case["first"], case["steps"], graph=True, unroll=16)
    assert first == gold[:1]
    assert toks == gold


@pytest.mark.parametrize("persistent", [True, False])
def test_engine_llama_1b_prompt512(cuda_dev, persistent):
    """Llama-3.2-1B shapes: a 512-token prefill (tensor-core int8 GEMM, causal
    attention, llama3 RoPE) then greedy decode."""
    case = _cases()["llama_1b_prompt512"]
    gold = _golden(case["id"], "tokens").tolist()
    _, eng = _engine(case, persistent=persistent)
    assert eng.persistent == persistent
    assert _run(case, eng, graph=True, unroll=16) == gold


@pytest.mark.parametrize("N,K,ng,w_off", [(4096, 1024, 1, 0), (3072, 2048, 1, 0),
                                          (1024, 3072, 1, 0), (500, 100, 1, 0),
                                          (2048, 1024, 8, 0), (8192, 1024, 1, 0),
                                          (6000, 1024, 4, 0), (8192, 1024, 1, 1)])
def test_gemv_with_folded_rmsnorm(cuda_dev, N, K, ng, w_off):
    """The GEMV of RMSNorm(x) * w with the norm inside the kernel's activation
    load against the two steps in fp64: single-row groups stage x in shared
    memory (any alignment of the norm weights, w_off = 1 float); four-row
    groups at K = 1024 (N > 5292 on 148 SMs) and shapes outside the streaming
    kernel go through the scratch path."""
    from quartz_b200 import device as qd
    g = torch.Generator().manual_seed(N + K)
    q = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8).to(cuda_dev)
    s = (torch.rand(N, ng, generator=g) * 1e-3 + 1e-4).to(cuda_dev)
    x = (torch.randn(K, generator=g) * 3).to(cuda_dev)
    w = (1 + 0.1 * torch.randn(K + w_off, generator=g)).to(cuda_dev)[w_off:]
    res = torch.randn(N, generator=g).to(cuda_dev)
    xn = _rms_ref(x, w, 1e-6).double()
    wd = (q.double().view(N, ng, K // ng) * s.double()[:, :, None]).view(N, K)
    ref = wd @ xn + res.double()
    _close(qd.gemv(q, s, x, residual=res, norm_w=w), ref, f"gemv+norm {N}x{K}")


@pytest.mark.parametrize("H,I", [(1024, 3072), (2048, 8192), (4096, 1536)])
def test_fused_mlp_with_folded_rmsnorm(cuda_dev, H, I):
    from quartz_b200 import device as qd
    g = torch.Generator().manual_seed(H + I)
    gu = torch.randint(-127, 128, (2 * I, H), generator=g, dtype=torch.int8).to(cuda_dev)
    gus = (torch.rand(2 * I, 1, generator=g) * 2e-4 + 1e-4).to(cuda_dev)
    dq = torch.randint(-127, 128, (H, I), generator=g, dtype=torch.int8).to(cuda_dev)
    ds = (torch.rand(H, 1, generator=g) * 2e-4 + 1e-4).to(cuda_dev)
    x = (torch.randn(H, generator=g) * 2).to(cuda_dev)
    w = (1 + 0.1 * torch.randn(H, generator=g)).to(cuda_dev)
    res = torch.randn(H, generator=g).to(cuda_dev)
    xn = _rms_ref(x, w, 1e-6).double()
    a = (gu.double() * gus.double()) @ xn
    gate, up = a[:I], a[I:]
    act = gate / (1 + torch.exp(-gate)) * up
    ref = (dq.double() * ds.double()) @ act + res.double()
    _close(qd.fused_mlp(gu, gus, x, dq, ds, residual=res, norm_w=w), ref, f"mlp+norm {H}x{I}")
