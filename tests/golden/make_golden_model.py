"""Model-level golden fixtures: greedy decoding with the reference's own
all-int8 fused model (quartz, numpy + Numba) on seeded random-init weights.

    NUMBA_CACHE_DIR=/tmp/numba_cache PYTHONDONTWRITEBYTECODE=1 \
        python tests/golden/make_golden_model.py /root/reference [case,case,...]

Weights: every Linear and Embedding, in the reference's leaf order
(quartz/weights.py:70-82), gets ``rng.standard_normal(shape, float32) * 0.02``
from one ``np.random.default_rng(1234)``; RMSNorm weights are ones. The model
is quantised with ``QuantConfig(default="int8", fused=True)``
(quartz/quantize.py:134-169). Two ways to start decoding:

* ``prompt`` / ``prompt_rng``: prefill the prompt ids through the model (the
  M > 1 path), then decode greedily (quartz/generate.py:36-58);
* ``kv``: fill every layer's KV cache with ``kv_len`` positions of N(0, 1)
  keys then values from ``default_rng(99)`` (layer by layer), then decode from
  token ``first``.
* ``kv`` with ``batch`` B: B sequences decoded in lockstep through the
  reference's batched path (decode_logits on [B, 1] ids, so every matmul has
  M = B rows and the MLP takes quartz/quantize.py:112-114): the caches hold
  [B, n_kv, kv_len, head_dim] draws per layer (keys then values, layer by
  layer, from ``default_rng(99)``) and sequence b starts from ``firsts[b]``;
  tokens are stored [steps, B].

Stored per case (cases_model.json + golden_model.npz): the config, the greedy
tokens, each step's top-1/top-2 logit margin, the top-8 (id, logit) of every
step, the RoPE inverse frequencies, and SHA-256 digests of a few quantised tensors so the weight recipe can
be proven identical on our side.
"""

from __future__ import annotations

import hashlib
import json
import os
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

LLAMA3_SCALING = dict(rope_type="llama3", factor=32.0, low_freq_factor=1.0,
                      high_freq_factor=4.0, original_max_position_embeddings=8192)

CASES = [
    dict(id="qwen3_tiny_prompt", arch="Qwen3ForCausalLM",
         cfg=dict(hidden_size=64, num_hidden_layers=2, num_attention_heads=4,
                  num_key_value_heads=2, head_dim=16, intermediate_size=128, vocab_size=64,
                  rope_theta=10000.0, tie_word_embeddings=True),
         start="prompt", prompt=[1, 2, 3, 4, 5], steps=16),
    dict(id="llama_tiny_prompt", arch="LlamaForCausalLM",
         cfg=dict(hidden_size=64, num_hidden_layers=2, num_attention_heads=4,
                  num_key_value_heads=2, head_dim=16, intermediate_size=128, vocab_size=96,
                  rope_theta=500000.0, tie_word_embeddings=False, rope_scaling=LLAMA3_SCALING),
         start="prompt", prompt=[3, 1, 4, 1, 5, 9, 2], steps=16),
    dict(id="qwen3_tiny_kv", arch="Qwen3ForCausalLM",
         cfg=dict(hidden_size=64, num_hidden_layers=2, num_attention_heads=4,
                  num_key_value_heads=2, head_dim=16, intermediate_size=128, vocab_size=64,
                  rope_theta=10000.0, tie_word_embeddings=True),
         start="kv", kv_len=40, first=7, steps=12),
    # small models with the head sizes of the real ones (64 / 128)
    dict(id="qwen3_small_kv", arch="Qwen3ForCausalLM",
         cfg=dict(hidden_size=256, num_hidden_layers=3, num_attention_heads=4,
                  num_key_value_heads=2, head_dim=64, intermediate_size=512, vocab_size=1000,
                  rope_theta=1000000.0, tie_word_embeddings=True),
         start="kv", kv_len=100, first=3, steps=24),
    dict(id="llama_small_prompt", arch="LlamaForCausalLM",
         cfg=dict(hidden_size=512, num_hidden_layers=2, num_attention_heads=8,
                  num_key_value_heads=2, head_dim=128, intermediate_size=1024, vocab_size=2000,
                  rope_theta=500000.0, tie_word_embeddings=False, rope_scaling=LLAMA3_SCALING),
         start="prompt_rng", prompt_seed=11, prompt_len=37, steps=24),
    # Qwen3-0.6B architecture: 512 prefilled KV positions, 128 greedy tokens
    dict(id="qwen3_0p6b_kv512", arch="Qwen3ForCausalLM",
         cfg=dict(hidden_size=1024, num_hidden_layers=28, num_attention_heads=16,
                  num_key_value_heads=8, head_dim=128, intermediate_size=3072,
                  vocab_size=151936, rope_theta=1000000.0, tie_word_embeddings=True),
         start="kv", kv_len=512, first=42, steps=128),
    # batched decode (B sequences in lockstep, M = B rows per matmul)
    dict(id="qwen3_small_kv_b3", arch="Qwen3ForCausalLM",
         cfg=dict(hidden_size=256, num_hidden_layers=3, num_attention_heads=4,
                  num_key_value_heads=2, head_dim=64, intermediate_size=512, vocab_size=1000,
                  rope_theta=1000000.0, tie_word_embeddings=True),
         start="kv", kv_len=100, batch=3, firsts=[3, 17, 500], steps=24),
] + [
    dict(id=f"qwen3_0p6b_kv512_b{B}", arch="Qwen3ForCausalLM",
         cfg=dict(hidden_size=1024, num_hidden_layers=28, num_attention_heads=16,
                  num_key_value_heads=8, head_dim=128, intermediate_size=3072,
                  vocab_size=151936, rope_theta=1000000.0, tie_word_embeddings=True),
         start="kv", kv_len=512, batch=B, firsts=[(42 + 9973 * b) % 151936 for b in range(B)],
         steps=32)
    for B in (2, 4, 8, 16)
] + [
    # Llama-3.2-1B architecture: 512-token prefill, then greedy decoding
    dict(id="llama_1b_prompt512", arch="LlamaForCausalLM",
         cfg=dict(hidden_size=2048, num_hidden_layers=16, num_attention_heads=32,
                  num_key_value_heads=8, head_dim=64, intermediate_size=8192,
                  vocab_size=128256, rope_theta=500000.0, tie_word_embeddings=True,
                  rope_scaling=LLAMA3_SCALING),
         start="prompt_rng", prompt_seed=7, prompt_len=512, steps=256),
]


def _digest(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main(ref_root: str, only=None):
    os.environ.setdefault("NUMBA_CACHE_DIR", "/tmp/numba_cache")
    sys.path.insert(0, ref_root)
    from quartz.config import ModelConfig, QuantConfig
    from quartz.models import build_model
    from quartz.weights import _walk_leaves
    from quartz.ops import Linear, RMSNorm, Embedding
    from quartz.quantize import quantize_model
    from quartz.cache import make_cache

    out_json = HERE / "cases_model.json"
    out_npz = HERE / "golden_model.npz"
    records = json.loads(out_json.read_text())["cases"] if out_json.exists() else []
    arrays = dict(np.load(out_npz)) if out_npz.exists() else {}
    for case in CASES:
        if only and case["id"] not in only:
            continue
        t0 = time.time()
        case = dict(case)
        cfg = ModelConfig.from_dict(dict(case["cfg"], architectures=[case["arch"]]))
        net = build_model(cfg)
        rng = np.random.default_rng(1234)
        for _name, m in _walk_leaves(net):
            if isinstance(m, Linear):
                m.weight = rng.standard_normal((m.out_features, m.in_features),
                                               dtype=np.float32) * np.float32(0.02)
            elif isinstance(m, Embedding):
                m.weight = rng.standard_normal((m.num_embeddings, m.dims),
                                               dtype=np.float32) * np.float32(0.02)
            elif isinstance(m, RMSNorm):
                m.weight = np.ones(m.dims, np.float32)
        quantize_model(net, QuantConfig(default="int8", fused=True))
        L = cfg.num_hidden_layers
        cache = make_cache(L)
        B = case.get("batch", 1)
        if case["start"] == "kv":
            krng = np.random.default_rng(99)
            shape = (B, cfg.num_key_value_heads, case["kv_len"], cfg.head_dim)
            for c in cache:
                k = krng.standard_normal(shape, dtype=np.float32)
                v = krng.standard_normal(shape, dtype=np.float32)
                c.update_and_fetch(k, v)
            firsts = case.get("firsts", [case.get("first")])
            logits = net.decode_logits(np.array([[f] for f in firsts]), cache=cache)[:, -1, :]
        else:
            if case["start"] == "prompt_rng":
                case["prompt"] = np.random.default_rng(case["prompt_seed"]).integers(
                    0, cfg.vocab_size, case["prompt_len"]).tolist()
            logits = net.decode_logits(np.array([case["prompt"]]), cache=cache)[:, -1, :]
        toks, margins, top_ids, top_vals = [], [], [], []
        for step in range(case["steps"]):
            row_toks = []
            for b in range(B):
                row = logits[b]
                order = np.argsort(-row, kind="stable")[:8]
                row_toks.append(int(np.argmax(row)))
                margins.append(float(row[order[0]] - row[order[1]]))
                top_ids.append(order)
                top_vals.append(row[order])
            toks.append(row_toks if B > 1 else row_toks[0])
            if step + 1 < case["steps"]:
                logits = net.decode_logits(np.array([[t] for t in row_toks]),
                                           cache=cache)[:, -1, :]
        emb = net.model.embed_tokens
        l0 = net.model.layers[0]
        digests = dict(embed_q=_digest(emb.q), embed_s=_digest(emb.scale),
                       q_proj0=_digest(l0.self_attn.q_proj.q),
                       gu_q0=_digest(l0.mlp.gu_q),
                       down_last=_digest(net.model.layers[-1].mlp.down_q))
        if not cfg.tie_word_embeddings:
            digests["lm_head_q"] = _digest(net.lm_head.q)
        cid = case["id"]
        arrays[f"{cid}__tokens"] = np.array(toks, np.int64)
        arrays[f"{cid}__margins"] = np.array(margins, np.float32)
        arrays[f"{cid}__top_ids"] = np.array(top_ids, np.int64)
        arrays[f"{cid}__top_vals"] = np.array(top_vals, np.float32)
        arrays[f"{cid}__inv_freq"] = np.asarray(l0.self_attn.rope.inv_freq, np.float32)
        rec = dict(case)
        rec["digests"] = digests
        rec["seconds"] = round(time.time() - t0, 1)
        records = [r for r in records if r["id"] != cid] + [rec]
        print(f"{cid}: {toks[:12]}... min margin {min(margins):.3e} ({rec['seconds']} s)",
              flush=True)
        del net, cache
        np.savez_compressed(out_npz, **arrays)
        with open(out_json, "w") as f:
            json.dump(dict(generator="tests/golden/make_golden_model.py",
                           reference="mlelarge/quartz (quartz/models, quartz/quantize.py, "
                                     "quartz/kernels)",
                           weights="standard_normal(float32) * 0.02 in leaf order, seed 1234; "
                                   "norms ones; QuantConfig(default='int8', fused=True)",
                           cases=records), f, indent=1)


if __name__ == "__main__":
    if len(sys.argv) < 2:
        raise SystemExit("usage: make_golden_model.py <path of the quartz source tree> "
                         "[case,case,...]")
    main(sys.argv[1], only=sys.argv[2].split(",") if len(sys.argv) > 2 else None)
