"""CPU checks of the decode workload's host side: the synthetic int8 checkpoint
recipe reproduces quartz's own int8 tensors byte for byte (SHA-256 digests the
reference recorded), the RoPE frequencies equal the reference's, and the model
spec reads HF configs like quartz/config.py."""

import hashlib
import json
from pathlib import Path

import numpy as np
import pytest

from quartz_b200.model import (LLAMA_3P2_1B, QWEN3_0P6B, ModelSpec, leaf_names, norm_weights,
                               random_int8_weights, rope_inv_freq, seeded_kv)

HERE = Path(__file__).resolve().parent
CASES = {c["id"]: c for c in json.loads((HERE / "golden" / "cases_model.json").read_text())["cases"]}


def _golden(cid, key):
    with np.load(HERE / "golden" / "golden_model.npz") as z:
        return z[f"{cid}__{key}"]


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _spec(cid):
    c = CASES[cid]
    return ModelSpec.from_hf(c["cfg"], c["arch"])


@pytest.mark.parametrize("cid", ["qwen3_tiny_prompt", "llama_tiny_prompt", "qwen3_tiny_kv"])
def test_weight_digests_tiny(cid):
    spec = _spec(cid)
    w = {n: (q, s) for n, q, s in random_int8_weights(spec)}
    d = CASES[cid]["digests"]
    last = f"model.layers.{spec.layers - 1}.mlp.down_proj"
    assert _sha(w["model.embed_tokens"][0]) == d["embed_q"]
    assert _sha(w["model.embed_tokens"][1]) == d["embed_s"]
    assert _sha(w["model.layers.0.self_attn.q_proj"][0]) == d["q_proj0"]
    gu = np.concatenate([w["model.layers.0.mlp.gate_proj"][0], w["model.layers.0.mlp.up_proj"][0]])
    assert _sha(gu) == d["gu_q0"]
    assert _sha(w[last][0]) == d["down_last"]
    if "lm_head_q" in d:
        assert _sha(w["lm_head"][0]) == d["lm_head_q"]


def test_weight_digests_qwen3_0p6b():
    """The full Qwen3-0.6B draw (about 0.6 G values): embedding first, last layer's down."""
    spec = _spec("qwen3_0p6b_kv512")
    d = CASES["qwen3_0p6b_kv512"]["digests"]
    last = f"model.layers.{spec.layers - 1}.mlp.down_proj"
    for name, q, s in random_int8_weights(spec):
        if name == "model.embed_tokens":
            assert _sha(q) == d["embed_q"] and _sha(s) == d["embed_s"]
        elif name == "model.layers.0.self_attn.q_proj":
            assert _sha(q) == d["q_proj0"]
        elif name == last:
            assert _sha(q) == d["down_last"]


@pytest.mark.parametrize("cid", sorted(CASES))
def test_rope_inv_freq(cid):
    try:
        ref = _golden(cid, "inv_freq")
    except KeyError:
        pytest.skip("fixture predates the stored frequencies")
    got = rope_inv_freq(_spec(cid))
    assert got.dtype == np.float32 and np.array_equal(got, ref)


def test_leaf_order_and_norms():
    names = [n for n, _ in leaf_names(LLAMA_3P2_1B)]
    assert names[0] == "model.embed_tokens" and names[-1].endswith("layers.15.mlp.down_proj")
    assert names[1:8] == [f"model.layers.0.{p}" for p in
                          ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj",
                           "self_attn.o_proj", "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj")]
    untied = ModelSpec(**{**QWEN3_0P6B.__dict__, "tie": False})
    assert leaf_names(untied)[-1] == ("lm_head", (151936, 1024))
    n = norm_weights(QWEN3_0P6B)
    assert len(n) == 1 + 4 * 28 and all((v == 1).all() for v in n.values())
    assert not any("q_norm" in k for k in norm_weights(LLAMA_3P2_1B))


def test_spec_from_hf_and_bytes():
    s = ModelSpec.from_hf(dict(hidden_size=2048, num_hidden_layers=16, num_attention_heads=32,
                               num_key_value_heads=8, intermediate_size=8192, vocab_size=128256,
                               head_dim=None), "LlamaForCausalLM")
    assert s.head_dim == 64 and not s.qk_norm and s.qkv_rows == 3072
    # all-int8 Qwen3-0.6B streams about 0.6 GB of weights per token
    assert 0.59e9 < QWEN3_0P6B.int8_bytes_per_token() < 0.60e9
    with pytest.raises(ValueError):
        ModelSpec(**{**QWEN3_0P6B.__dict__, "arch": "GPT2LMHeadModel"})


def test_seeded_kv_shapes():
    spec = _spec("qwen3_tiny_kv")
    kv = list(seeded_kv(spec, 40))
    assert len(kv) == spec.layers
    k, v = kv[0]
    assert k.shape == (spec.n_kv, 40, spec.head_dim) and k.dtype == np.float32
    rng = np.random.default_rng(99)
    k0 = rng.standard_normal((1, spec.n_kv, 40, spec.head_dim), dtype=np.float32)
    assert np.array_equal(k, k0[0])


def _quartz_like(spec, fused_mlp):
    """An object tree shaped like a quantised quartz model
    (quartz/models/common.py, quartz/quantize.py), built from the synthetic
    checkpoint."""
    from types import SimpleNamespace as NS
    w = {n: (q, s) for n, q, s in random_int8_weights(spec)}
    lin = lambda n: NS(q=w[n][0], scale=w[n][1], weight=w[n][0])  # noqa: E731
    norm = lambda d: NS(weight=np.ones(d, np.float32))  # noqa: E731
    layers = []
    for i in range(spec.layers):
        p = f"model.layers.{i}."
        att = NS(q_proj=lin(p + "self_attn.q_proj"), k_proj=lin(p + "self_attn.k_proj"),
                 v_proj=lin(p + "self_attn.v_proj"), o_proj=lin(p + "self_attn.o_proj"))
        if spec.qk_norm:
            att.q_norm, att.k_norm = norm(spec.head_dim), norm(spec.head_dim)
        if fused_mlp:
            g, u, d = (w[p + "mlp." + n] for n in ("gate_proj", "up_proj", "down_proj"))
            mlp = NS(gu_q=np.concatenate([g[0], u[0]]), gu_s=np.concatenate([g[1], u[1]]),
                     down_q=d[0], down_s=d[1], inter=spec.inter, hidden=spec.hidden)
        else:
            mlp = NS(gate_proj=lin(p + "mlp.gate_proj"), up_proj=lin(p + "mlp.up_proj"),
                     down_proj=lin(p + "mlp.down_proj"))
        layers.append(NS(self_attn=att, mlp=mlp, input_layernorm=norm(spec.hidden),
                         post_attention_layernorm=norm(spec.hidden)))
    cfg = NS(hidden_size=spec.hidden, num_hidden_layers=spec.layers,
             num_attention_heads=spec.n_heads, num_key_value_heads=spec.n_kv,
             head_dim=spec.head_dim, intermediate_size=spec.inter, vocab_size=spec.vocab,
             rope_theta=spec.rope_theta, tie_word_embeddings=spec.tie,
             rope_scaling=spec.rope_scaling, rms_norm_eps=spec.eps, architectures=())
    net = type(spec.arch, (), {})()
    net.config = cfg
    net.model = NS(embed_tokens=lin("model.embed_tokens"), layers=layers, norm=norm(spec.hidden))
    if not spec.tie:
        net.lm_head = lin("lm_head")
    return net, w


@pytest.mark.parametrize("cid,fused", [("qwen3_tiny_kv", True), ("llama_tiny_prompt", False),
                                       ("llama_small_prompt", True)])
def test_quartz_checkpoint_reads_a_quartz_model(cid, fused):
    from quartz_b200.decode import quartz_checkpoint
    spec = _spec(cid)
    net, w = _quartz_like(spec, fused)
    got_spec, int8, norms = quartz_checkpoint(net)
    assert got_spec == spec and got_spec.rope_scaling == spec.rope_scaling
    assert set(int8) == set(w)
    for n, (q, s) in w.items():
        assert np.array_equal(int8[n][0], q) and np.array_equal(int8[n][1], s), n
    assert set(norms) == set(norm_weights(spec))


@pytest.mark.parametrize("cid,world", [("llama_small_prompt", 2), ("qwen3_small_kv", 2),
                                       ("qwen3_tiny_kv", 2)])
def test_tp_shard_reassembles(cid, world):
    """The ranks' parts of a checkpoint put back together give the full
    matrices: q/k/v and gate/up rows, o and down columns, lm_head vocab rows."""
    from quartz_b200.tp_decode import tp_shard
    spec = _spec(cid)
    w = {n: (q, s) for n, q, s in random_int8_weights(spec)}
    parts = [tp_shard(spec, w, r, world) for r in range(world)]
    assert all(p[0].n_heads * world == spec.n_heads and p[0].n_kv * world == spec.n_kv
               and p[0].inter * world == spec.inter for p in parts)
    for name, (q, s) in w.items():
        leaf = name.rsplit(".", 1)[-1]
        if name in ("model.embed_tokens",):
            assert all(np.array_equal(p[1][name][0], q) for p in parts)
        elif name == "lm_head":
            continue
        elif leaf in ("o_proj", "down_proj"):
            assert np.array_equal(np.concatenate([p[1][name][0] for p in parts], 1), q), name
            assert all(np.array_equal(p[1][name][1], s) for p in parts)
        else:
            assert np.array_equal(np.concatenate([p[1][name][0] for p in parts], 0), q), name
            assert np.array_equal(np.concatenate([p[1][name][1] for p in parts], 0), s), name
    lm = w["lm_head"] if "lm_head" in w else w["model.embed_tokens"]
    assert np.array_equal(np.concatenate([p[2][0] for p in parts]), lm[0])
    assert [p[2][2] for p in parts] == [0] + [p[2][3] for p in parts][:-1]
    with pytest.raises(ValueError):
        tp_shard(spec, w, 0, 3)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_tp_shard_eight_kv_heads(world):
    """Qwen3-8B's head counts (32 query / 8 kv, MLP a multiple of 8) split over
    1, 2, 4 and 8 ranks, on a small stand-in of the same head structure."""
    from quartz_b200.tp_decode import tp_shard
    spec = ModelSpec(arch="Qwen3ForCausalLM", hidden=64, layers=1, n_heads=32, n_kv=8,
                     head_dim=16, inter=96, vocab=50, rope_theta=1e6, tie=False)
    w = {n: (q, s) for n, q, s in random_int8_weights(spec)}
    parts = [tp_shard(spec, w, r, world) for r in range(world)]
    for local, lw, (lq, _, lo, hi) in parts:
        assert local.n_heads == 32 // world and local.n_kv == 8 // world
        assert lw["model.layers.0.self_attn.q_proj"][0].shape == (32 // world * 16, 64)
        assert lw["model.layers.0.self_attn.o_proj"][0].shape == (64, 32 // world * 16)
        assert lw["model.layers.0.mlp.down_proj"][0].shape == (64, 96 // world)
        assert lq.shape[0] == hi - lo
    assert sum(p[2][3] - p[2][2] for p in parts) == 50


def test_seeded_kv_batched_draws():
    """A batched cache draws [B, n_kv, T, hd] per layer from the same stream
    (keys then values, layer by layer), as the reference's batched fixtures do;
    batch=1 is the unbatched draw with a leading axis."""
    spec = _spec("qwen3_small_kv")
    one = list(seeded_kv(spec, 7))
    b1 = list(seeded_kv(spec, 7, batch=1))
    b3 = list(seeded_kv(spec, 7, batch=3))
    rng = np.random.default_rng(99)
    for (k1, v1), (kb1, vb1), (k3, v3) in zip(one, b1, b3):
        assert kb1.shape == (1,) + k1.shape and np.array_equal(kb1[0], k1)
        assert np.array_equal(vb1[0], v1)
        assert k3.shape == (3, spec.n_kv, 7, spec.head_dim)
        assert np.array_equal(k3, rng.standard_normal(k3.shape, dtype=np.float32))
        assert np.array_equal(v3, rng.standard_normal(v3.shape, dtype=np.float32))


def test_cached_int8_weights_round_trip(tmp_path):
    """The per-host checkpoint cache returns random_int8_weights' tensors, drawn
    once and then loaded (writable arrays) from its two flat files."""
    from quartz_b200.model import cached_int8_weights
    spec = _spec("qwen3_tiny_kv")
    want = list(random_int8_weights(spec))
    first = cached_int8_weights(spec, cache_dir=str(tmp_path))
    files = sorted(p.name for p in tmp_path.iterdir() if p.suffix == ".npy")
    assert len(files) == 2
    again = cached_int8_weights(spec, cache_dir=str(tmp_path))
    for (n0, q0, s0), (n1, q1, s1), (n2, q2, s2) in zip(want, first, again):
        assert n0 == n1 == n2
        assert np.array_equal(q0, q1) and np.array_equal(q0, q2)
        assert np.array_equal(s0, s1) and np.array_equal(s0, s2)
        assert q2.flags.writeable and q2.dtype == np.int8 and s2.dtype == np.float32
    # another seed is another file
    other = cached_int8_weights(spec, seed=5, cache_dir=str(tmp_path))
    assert not np.array_equal(other[1][1], want[1][1])
