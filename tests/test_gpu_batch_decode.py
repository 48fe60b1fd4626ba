"""Batched decode on the GPU: B sequences in lockstep, quartz's decode step on
[B, 1] ids (quartz/models/common.py:79-88), where every matmul runs M = B rows
(quartz/kernels/int8.py:66-87) and the MLP takes the per-op path
(quartz/quantize.py:112-114).

* qz_attention_decode_qkv_batch against a torch fp64 restatement of
  quartz/attention.py:29-43 per sequence (tolerance 1e-4 * max|ref|), on the
  fused kernel's shapes and on shapes that take the per-sequence fallback;
* the batched engine's greedy tokens against the tokens quartz itself produced
  with the same B rows (tests/golden/golden_model.npz), eager and CUDA-graph
  replay, and the first step's top-8 logits of every row.
"""

import ctypes
import json
from pathlib import Path

import numpy as np
import pytest

from tests.test_gpu_decode import _close, _rms_ref, _rope_ref, _sdpa_ref

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

GOLD = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module", autouse=True)
def _clean_status():
    from quartz_b200 import device
    if torch.cuda.is_available():
        device.status(clear=True)
    yield
    if torch.cuda.is_available():
        device.check_status()


def _cases():
    return {c["id"]: c for c in json.loads((GOLD / "cases_model.json").read_text())["cases"]}


def _golden(cid, what):
    with np.load(GOLD / "golden_model.npz") as z:
        return z[f"{cid}__{what}"]


@pytest.mark.parametrize("qk_norm", [True, False])
@pytest.mark.parametrize("B,nq,nkv,hd,pos,max_ctx", [(3, 16, 8, 128, 512, 640),
                                                     (16, 32, 8, 64, 100, 128),
                                                     (2, 32, 8, 128, 0, 16),
                                                     (5, 4, 2, 16, 39, 52),     # fallback
                                                     (4, 12, 2, 96, 70, 80)])   # fallback
def test_attention_decode_qkv_batch(cuda_dev, qk_norm, B, nq, nkv, hd, pos, max_ctx):
    """Norm + RoPE + append + attention for B sequences in one call; each
    sequence against the single-sequence references; other positions and the
    other sequences' caches untouched."""
    from quartz_b200 import _lib
    from quartz_b200.model import ModelSpec, rope_inv_freq
    lib = _lib.load()
    g = torch.Generator().manual_seed(B * 1000 + pos * 3 + hd)
    spec = ModelSpec(arch="Qwen3ForCausalLM", hidden=64, layers=1, n_heads=nq, n_kv=nkv,
                     head_dim=hd, inter=64, vocab=8, rope_theta=1e6, tie=True)
    inv = torch.from_numpy(rope_inv_freq(spec)).to(cuda_dev)
    rows = (nq + 2 * nkv) * hd
    qkv = torch.randn(B, rows, generator=g).to(cuda_dev)
    qn = (1 + 0.1 * torch.randn(hd, generator=g)).to(cuda_dev) if qk_norm else None
    kn = (1 + 0.1 * torch.randn(hd, generator=g)).to(cuda_dev) if qk_norm else None
    kc = torch.randn(B, nkv, max_ctx, hd, generator=g).to(cuda_dev)
    vc = torch.randn(B, nkv, max_ctx, hd, generator=g).to(cuda_dev)
    kc0, vc0 = kc.clone(), vc.clone()
    out = torch.full((B, nq * hd), float("nan"), device=cuda_dev)
    pos_dev = torch.tensor([pos], dtype=torch.int64, device=cuda_dev)
    nb = ctypes.c_int64(0)
    _lib.check(lib.qz_attention_decode_batch_workspace_bytes(B, nq, nkv, hd, max_ctx,
                                                             ctypes.byref(nb)))
    ws = torch.zeros(nb.value, dtype=torch.uint8, device=cuda_dev)
    st = torch.cuda.current_stream(cuda_dev).cuda_stream

    def call():
        _lib.check(lib.qz_attention_decode_qkv_batch(
            qkv.data_ptr(), rows, qn.data_ptr() if qk_norm else None,
            kn.data_ptr() if qk_norm else None, inv.data_ptr(), kc.data_ptr(), vc.data_ptr(),
            nkv * max_ctx * hd, out.data_ptr(), nq * hd, B, nq, nkv, hd, max_ctx, 0,
            pos_dev.data_ptr(), 1e-6, hd ** -0.5, ws.data_ptr(), ws.numel(), st))

    call()
    p = torch.tensor([float(pos)], device=cuda_dev)
    keep = [t for t in range(max_ctx) if t != pos]
    refs = []
    for b in range(B):
        parts = qkv[b].view(nq + 2 * nkv, hd)
        qh, kh, vh = parts[:nq], parts[nq:nq + nkv], parts[nq + nkv:]
        if qk_norm:
            qh, kh = _rms_ref(qh, qn, 1e-6), _rms_ref(kh, kn, 1e-6)
        qr = _rope_ref(qh[:, None], p, inv)[:, 0]
        kr = _rope_ref(kh[:, None], p, inv)[:, 0]
        _close(kc[b, :, pos], kr, f"seq {b} appended k")
        assert torch.equal(vc[b, :, pos], vh), f"seq {b} appended v"
        assert torch.equal(kc[b][:, keep], kc0[b][:, keep]), f"seq {b} k cache"
        assert torch.equal(vc[b][:, keep], vc0[b][:, keep]), f"seq {b} v cache"
        kref, vref = kc0[b].clone(), vc0[b].clone()
        kref[:, pos], vref[:, pos] = kr, vh
        ref = _sdpa_ref(qr[:, None], kref[:, :pos + 1], vref[:, :pos + 1], hd ** -0.5, nq // nkv)
        refs.append(ref.view(-1))
        _close(out[b], refs[b], f"seq {b} attention")
    call()            # again: the workspace's tickets were left ready
    for b in range(B):
        _close(out[b], refs[b], f"seq {b} attention, second call")


def _batch_engine(case, extra_ctx=0):
    from quartz_b200.decode import DecodeEngine
    from quartz_b200.model import ModelSpec, cached_int8_weights, norm_weights
    spec = ModelSpec.from_hf(case["cfg"], case["arch"])
    eng = DecodeEngine(spec, cached_int8_weights(spec), norm_weights(spec),
                       max_ctx=case["kv_len"] + case["steps"] + extra_ctx, max_prefill=1,
                       batch=case["batch"])
    return spec, eng


@pytest.mark.parametrize("cid", ["qwen3_small_kv_b3", "qwen3_0p6b_kv512_b2",
                                 "qwen3_0p6b_kv512_b4", "qwen3_0p6b_kv512_b8",
                                 "qwen3_0p6b_kv512_b16"])
def test_batch_engine_tokens_match_reference(cuda_dev, cid):
    """B sequences from a seeded [B, n_kv, 512, hd] cache each: greedy tokens of
    every row equal quartz's batched decode, eager (with the first step's
    top-8 logits per row) and through graph replay."""
    from quartz_b200.model import seeded_kv
    case = _cases()[cid]
    B = case["batch"]
    gold = _golden(cid, "tokens").tolist()
    top_ids = _golden(cid, "top_ids")
    top_vals = _golden(cid, "top_vals")
    spec, eng = _batch_engine(case)
    eng.load_kv(seeded_kv(spec, case["kv_len"], batch=B))
    first = eng.generate_batch(case["firsts"], 1, graph=False)
    for b in range(B):
        _close(eng.logits[b].cpu()[torch.from_numpy(top_ids[b])], torch.from_numpy(top_vals[b]),
               f"{cid} row {b} step-0 top-8 logits")
    assert first == gold[:1], "first step"
    eng.reset(case["kv_len"])
    toks = eng.generate_batch(case["firsts"], case["steps"], graph=False)
    assert toks == gold, "eager"
    eng.reset(case["kv_len"])
    toks = eng.generate_batch(case["firsts"], case["steps"], graph=True, unroll=8)
    assert toks == gold, "graph"
