"""CPU restatement of quartz's greedy decode step (test infrastructure only).

The checker for the device decode engine and the CPU decode baseline of
bench.py: quartz's all-int8 decoder for one token (M = 1) in numpy fp32 with
the int8 matmuls done by the oracle's C kernels (the restatement of
quartz/kernels/int8.py:24-38 and fused.py:27-65). Step by step it follows
quartz/models/common.py:29-78 (embedding, layers, final norm, lm_head on the
last position), quartz/models/qwen3.py:31-44 and llama.py:31-44 (projections,
Qwen3's per-head q/k RMSNorm before RoPE), quartz/ops.py:24-32 (RMSNorm),
quartz/rope.py:26-78 (half-split RoPE, llama3 frequency scaling),
quartz/cache.py:26-46 (KV append), quartz/attention.py:29-43 (GQA by repeat,
fp32 softmax) and quartz/sample.py:21-22 (greedy argmax).
"""

from __future__ import annotations

import numpy as np

from . import oracle as _k

QWEN3 = "Qwen3ForCausalLM"
LLAMA = "LlamaForCausalLM"


def rope_inv_freq(head_dim: int, base: float, scaling: dict | None) -> np.ndarray:
    """Per-pair inverse frequencies (quartz/rope.py:26-66)."""
    if scaling and scaling.get("rope_type") == "llama3":
        factor = scaling["factor"]
        low = scaling.get("low_freq_factor", 1.0)
        high = scaling.get("high_freq_factor", 4.0)
        old = scaling.get("original_max_position_embeddings", 8192)
        freqs = base ** (np.arange(0, head_dim, 2, dtype=np.float32) / head_dim)
        wavelens = 2 * np.pi * freqs
        freqs = np.where(wavelens > old / low, freqs * factor, freqs)
        medium = (wavelens > old / high) & (wavelens < old / low)
        smooth = (old / wavelens - low) / (high - low)
        smooth_freqs = freqs / ((1 - smooth) / factor + smooth)
        denom = np.where(medium, smooth_freqs, freqs).astype(np.float32)
        return (1.0 / denom).astype(np.float32)
    return (base ** (-(np.arange(0, head_dim, 2, dtype=np.float32) / head_dim))).astype(np.float32)


def _rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    x = x.astype(np.float32, copy=False)
    ms = np.mean(x * x, axis=-1, keepdims=True)
    return (x * (1.0 / np.sqrt(ms + eps)) * w).astype(np.float32)


def _rope(x: np.ndarray, pos: int, inv_freq: np.ndarray) -> np.ndarray:
    """x [heads, D] at position pos, half-split rotation."""
    d = x.shape[-1] // 2
    angle = np.float32(pos) * inv_freq
    c, s = np.cos(angle).astype(np.float32), np.sin(angle).astype(np.float32)
    out = np.empty_like(x)
    out[:, :d] = x[:, :d] * c - x[:, d:] * s
    out[:, d:] = x[:, d:] * c + x[:, :d] * s
    return out


class DecodePort:
    """One sequence: `cfg` is the HF-style config dict (hidden_size,
    num_hidden_layers, num_attention_heads, num_key_value_heads, head_dim,
    intermediate_size, vocab_size, rope_theta, rope_scaling,
    tie_word_embeddings, rms_norm_eps); int8: name -> (q, scale) in quartz's
    leaf names; norms: name -> fp32 weights."""

    def __init__(self, cfg: dict, arch: str, int8: dict, norms: dict, max_ctx: int):
        self.H = cfg["hidden_size"]
        self.L = cfg["num_hidden_layers"]
        self.nq = cfg["num_attention_heads"]
        self.nkv = cfg.get("num_key_value_heads") or self.nq
        self.hd = cfg.get("head_dim") or self.H // self.nq
        self.I = cfg["intermediate_size"]
        self.V = cfg["vocab_size"]
        self.eps = float(cfg.get("rms_norm_eps", 1e-6))
        self.qk_norm = arch == QWEN3
        self.tie = bool(cfg.get("tie_word_embeddings", False))
        self.inv_freq = rope_inv_freq(self.hd, float(cfg.get("rope_theta", 10000.0)),
                                      cfg.get("rope_scaling"))
        self.scale = self.hd ** -0.5
        self.w = int8
        self.n = norms
        self.gu = []
        for i in range(self.L):
            p = f"model.layers.{i}.mlp."
            gq, gs = int8[p + "gate_proj"]
            uq, us = int8[p + "up_proj"]
            self.gu.append((np.ascontiguousarray(np.concatenate([gq, uq])),
                            np.ascontiguousarray(np.concatenate([gs, us]))))
        self.k = np.zeros((self.L, self.nkv, max_ctx, self.hd), np.float32)
        self.v = np.zeros_like(self.k)
        self.pos = 0
        self.logits = None

    def load_kv(self, kv) -> None:
        T = 0
        for i, (k, v) in enumerate(kv):
            T = k.shape[1]
            self.k[i, :, :T] = k
            self.v[i, :, :T] = v
        self.pos = T

    def _lin(self, name: str, x: np.ndarray) -> np.ndarray:
        q, s = self.w[name]
        return _k.matmul_int8(q, s, x)

    def step(self, token: int) -> int:
        """Feed `token` at the current position; return the greedy next token."""
        H, hd, nq, nkv = self.H, self.hd, self.nq, self.nkv
        eq, es = self.w["model.embed_tokens"]
        ng = es.shape[1]
        h = (eq[token].astype(np.float32).reshape(ng, H // ng) * es[token][:, None]).reshape(H)
        pos = self.pos
        T = pos + 1
        n_rep = nq // nkv
        for i in range(self.L):
            p = f"model.layers.{i}."
            x = _rmsnorm(h, self.n[p + "input_layernorm"], self.eps)
            q = self._lin(p + "self_attn.q_proj", x).reshape(nq, hd)
            k = self._lin(p + "self_attn.k_proj", x).reshape(nkv, hd)
            v = self._lin(p + "self_attn.v_proj", x).reshape(nkv, hd)
            if self.qk_norm:
                q = _rmsnorm(q, self.n[p + "self_attn.q_norm"], self.eps)
                k = _rmsnorm(k, self.n[p + "self_attn.k_norm"], self.eps)
            q = _rope(q, pos, self.inv_freq)
            k = _rope(k, pos, self.inv_freq)
            self.k[i, :, pos] = k
            self.v[i, :, pos] = v
            K = np.repeat(self.k[i, :, :T], n_rep, axis=0)      # [nq, T, hd]
            Vv = np.repeat(self.v[i, :, :T], n_rep, axis=0)
            sc = np.einsum("hd,htd->ht", q, K).astype(np.float32) * np.float32(self.scale)
            sc = sc - sc.max(axis=-1, keepdims=True)
            e = np.exp(sc)
            pr = e / e.sum(axis=-1, keepdims=True)
            att = np.einsum("ht,htd->hd", pr, Vv).astype(np.float32).reshape(nq * hd)
            h = h + self._lin(p + "self_attn.o_proj", att)
            x = _rmsnorm(h, self.n[p + "post_attention_layernorm"], self.eps)
            gq, gs = self.gu[i]
            dq, ds = self.w[p + "mlp.down_proj"]
            out = np.empty(H, np.float32)
            _k.fused_mlp_decode(gq, gs, np.ascontiguousarray(x), dq, ds,
                                np.empty(self.I, np.float32), out)
            h = h + out
        x = _rmsnorm(h, self.n["model.norm"], self.eps)
        name = "model.embed_tokens" if self.tie else "lm_head"
        self.logits = self._lin(name, x)
        self.pos = T
        return int(np.argmax(self.logits))
