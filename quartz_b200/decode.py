"""All-int8 greedy decoding on one GPU: the device decode step around the int8 path.

quartz decodes with numpy on the host (quartz/generate.py:36-58): per token,
embedding gather -> per layer [RMSNorm -> q/k/v projections -> (Qwen3) q/k
RMSNorm -> RoPE -> KV append -> GQA attention -> o projection + residual ->
RMSNorm -> fused int8 MLP + residual] -> final RMSNorm -> lm_head -> argmax
(quartz/models/common.py:29-78, quartz/models/qwen3.py:31-45). ``DecodeEngine``
runs every one of those steps as a kernel of libquartz_b200 on device-resident
weights and KV cache, so a whole token is stream-ordered device work with no
host round trip, and ``generate`` replays it from a CUDA graph: the position
counter and the token live in device memory, the argmax kernel writes the
next token where the embedding gather of the next replay reads it, and the
only host traffic is the final token list.

Differences of form (not of results) from quartz:
* q, k and v are one stacked [(nq + 2 nkv) hd, H] int8 matrix (one GEMV
  instead of three; rows and scales are the three matrices' own);
* the RMSNorms are applied by the kernels that consume them (the qkv GEMV,
  the fused MLP, the lm_head GEMV normalise their input as they load it);
* the KV cache is preallocated [layers, n_kv, max_ctx, head_dim] fp32 instead
  of growing in 256-position steps (quartz/cache.py:26-46);
* prefill (M > 1) runs the tensor-core int8 GEMM and the causal prefill
  attention, decode (M = 1) the streaming GEMVs and the fused MLP, the same
  M split as quartz/quantize.py:99-114.
"""

from __future__ import annotations

import ctypes
from typing import Iterable, Mapping

import numpy as np
import torch

from . import _lib, device as qd
from .model import ARCHS, ModelSpec, rope_inv_freq


def _dev_f32(a, dev) -> torch.Tensor:
    if isinstance(a, torch.Tensor):
        return a.to(device=dev, dtype=torch.float32).contiguous()
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(dev)


def _dev_i8(a, dev) -> torch.Tensor:
    if isinstance(a, torch.Tensor):
        return a.to(device=dev, dtype=torch.int8).contiguous()
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.int8)).to(dev)


def _cat(parts):
    """Row concatenation of numpy arrays or torch tensors (not mixed)."""
    if isinstance(parts[0], torch.Tensor):
        return torch.cat(parts, 0)
    return np.concatenate(parts, 0)


class _Layer:
    __slots__ = ("qkv_q", "qkv_s", "o_q", "o_s", "gu_q", "gu_s", "down_q", "down_s", "in_w",
                 "post_w", "qn_w", "kn_w")


def quartz_checkpoint(net) -> tuple[ModelSpec, dict, dict]:
    """(spec, int8 weights, norm weights) of a quartz model quantised by
    ``quantize_model(net, QuantConfig(default="int8", ...))``
    (quartz/quantize.py:134-169), read from its module tree by attribute
    (quartz/models/common.py:17-78; no import of quartz): QuantizedLinear /
    QuantizedEmbedding leaves give (q, scale); a FusedMLP (quantize.py:87-97)
    gives its stacked gate|up rows back as gate and up; RMSNorm leaves give
    their weights. Arrays are not copied."""
    cfg = net.config
    arch = type(net).__name__
    if arch not in ARCHS:
        arch = (tuple(getattr(cfg, "architectures", ()) or ()) + (None,))[0]
    spec = ModelSpec(arch=arch, hidden=cfg.hidden_size, layers=cfg.num_hidden_layers,
                     n_heads=cfg.num_attention_heads, n_kv=cfg.num_key_value_heads,
                     head_dim=cfg.head_dim, inter=cfg.intermediate_size, vocab=cfg.vocab_size,
                     rope_theta=float(cfg.rope_theta), tie=bool(cfg.tie_word_embeddings),
                     rope_scaling=getattr(cfg, "rope_scaling", None),
                     eps=float(getattr(cfg, "rms_norm_eps", 1e-6)))

    def q8(leaf, name):
        if not (hasattr(leaf, "q") and hasattr(leaf, "scale")):
            raise ValueError(f"{name} is not int8-quantised (quantise with "
                             f"QuantConfig(default='int8'))")
        return np.asarray(leaf.q), np.asarray(leaf.scale)

    m = net.model
    int8 = {"model.embed_tokens": q8(m.embed_tokens, "model.embed_tokens")}
    norms = {"model.norm": np.asarray(m.norm.weight)}
    for i, layer in enumerate(m.layers):
        p = f"model.layers.{i}."
        att = layer.self_attn
        for n in ("q_proj", "k_proj", "v_proj", "o_proj"):
            int8[p + "self_attn." + n] = q8(getattr(att, n), p + "self_attn." + n)
        mlp = layer.mlp
        if hasattr(mlp, "gu_q"):
            I = int(mlp.inter)
            int8[p + "mlp.gate_proj"] = (np.asarray(mlp.gu_q)[:I], np.asarray(mlp.gu_s)[:I])
            int8[p + "mlp.up_proj"] = (np.asarray(mlp.gu_q)[I:], np.asarray(mlp.gu_s)[I:])
            int8[p + "mlp.down_proj"] = (np.asarray(mlp.down_q), np.asarray(mlp.down_s))
        else:
            for n in ("gate_proj", "up_proj", "down_proj"):
                int8[p + "mlp." + n] = q8(getattr(mlp, n), p + "mlp." + n)
        norms[p + "input_layernorm"] = np.asarray(layer.input_layernorm.weight)
        norms[p + "post_attention_layernorm"] = np.asarray(layer.post_attention_layernorm.weight)
        if spec.qk_norm:
            norms[p + "self_attn.q_norm"] = np.asarray(att.q_norm.weight)
            norms[p + "self_attn.k_norm"] = np.asarray(att.k_norm.weight)
    if not spec.tie:
        int8["lm_head"] = q8(net.lm_head, "lm_head")
    return spec, int8, norms


class DecodeEngine:
    """Device-resident all-int8 decoder for one sequence.

    weights: name -> (q int8 [out, in], scale fp32 [out, ng]) for every Linear
    and the embedding (names as quartz.model.leaf_names), name -> fp32 vector for
    the RMSNorms (quartz.model.norm_weights). Iterables of (name, q, scale) are
    accepted for the int8 tensors so a large checkpoint streams to the device.
    """

    def __init__(self, spec: ModelSpec, int8_weights: Mapping | Iterable, norms: Mapping,
                 *, max_ctx: int, max_prefill: int = 512, device=None,
                 persistent: bool = False, fold_norms: bool = True, batch: int = 1):
        """batch: sequences decoded in lockstep (quartz's decode_logits on [B, 1]
        ids, quartz/models/common.py:79-88): every step runs B rows through the
        int8 GEMMs (M = B, quartz/kernels/int8.py:66-87, 106-107), the per-op
        MLP (quartz/quantize.py:112-114) and a batched attention over B caches
        sharing one position. batch > 1 decodes through generate_batch and has
        no prefill (sequences start from a loaded cache)."""
        self.spec = spec
        self.batch = int(batch)
        if self.batch < 1:
            raise ValueError("batch must be >= 1")
        if self.batch > 1:
            persistent = False
        self.dev = torch.device("cuda", qd.ensure_device(device))
        dev = self.dev
        self.lib = _lib.load()
        self.max_ctx = int(max_ctx)
        self.max_prefill = max(1, int(max_prefill))
        S = spec
        H, hd = S.hidden, S.head_dim
        self.layers = [_Layer() for _ in range(S.layers)]
        self.embed_q = self.embed_s = self.lm_q = self.lm_s = None
        leaves = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")
        pending: dict[int, dict[str, tuple]] = {}

        def upload_layer(i: int, w: dict) -> None:
            L = self.layers[i]
            if len({w[n][1].shape[1] for n in ("q_proj", "k_proj", "v_proj")}) != 1:
                raise ValueError("q/k/v scales must share a group count")
            L.qkv_q = _dev_i8(_cat([w[n][0] for n in ("q_proj", "k_proj", "v_proj")]), dev)
            L.qkv_s = _dev_f32(_cat([w[n][1] for n in ("q_proj", "k_proj", "v_proj")]), dev)
            L.o_q, L.o_s = _dev_i8(w["o_proj"][0], dev), _dev_f32(w["o_proj"][1], dev)
            # gate rows over up rows, the layout of quartz/quantize.py:95-96
            L.gu_q = _dev_i8(_cat([w["gate_proj"][0], w["up_proj"][0]]), dev)
            L.gu_s = _dev_f32(_cat([w["gate_proj"][1], w["up_proj"][1]]), dev)
            L.down_q, L.down_s = _dev_i8(w["down_proj"][0], dev), _dev_f32(w["down_proj"][1], dev)

        pairs = ((n, *qs) for n, qs in int8_weights.items()) \
            if isinstance(int8_weights, Mapping) else int8_weights
        for name, q, s in pairs:
            if name == "model.embed_tokens":
                self.embed_q, self.embed_s = _dev_i8(q, dev), _dev_f32(s, dev)
                continue
            if name == "lm_head":
                self.lm_q, self.lm_s = _dev_i8(q, dev), _dev_f32(s, dev)
                continue
            parts = name.split(".")
            if (len(parts) != 5 or parts[:2] != ["model", "layers"] or parts[4] not in leaves
                    or not 0 <= int(parts[2]) < S.layers):
                raise KeyError(f"unexpected weight {name!r}")
            i = int(parts[2])
            w = pending.setdefault(i, {})
            w[parts[4]] = (q, s)
            if len(w) == len(leaves):      # layer complete: upload and drop the host copies
                upload_layer(i, pending.pop(i))
        if pending:
            raise ValueError(f"incomplete weights for layers {sorted(pending)}")
        if self.embed_q is None:
            raise ValueError("missing model.embed_tokens")
        if S.tie:
            self.lm_q, self.lm_s = self.embed_q, self.embed_s
        elif self.lm_q is None:
            raise ValueError("missing lm_head (tie_word_embeddings is false)")
        for i, L in enumerate(self.layers):
            p = f"model.layers.{i}."
            for attr in ("qkv_q", "o_q", "gu_q", "down_q"):
                if not hasattr(L, attr):
                    raise ValueError(f"layer {i} lacks {attr}")
            L.in_w = _dev_f32(norms[p + "input_layernorm"], dev)
            L.post_w = _dev_f32(norms[p + "post_attention_layernorm"], dev)
            if S.qk_norm:
                L.qn_w = _dev_f32(norms[p + "self_attn.q_norm"], dev)
                L.kn_w = _dev_f32(norms[p + "self_attn.k_norm"], dev)
            else:
                L.qn_w = L.kn_w = None
        self.norm_w = _dev_f32(norms["model.norm"], dev)
        self.inv_freq = _dev_f32(rope_inv_freq(S), dev)
        self.attn_scale = float(hd ** -0.5)
        self.ng = self.layers[0].qkv_s.shape[1] if self.layers else 1

        # KV cache and activation buffers
        f32 = dict(dtype=torch.float32, device=dev)
        B = self.batch
        cache_shape = ((S.layers, S.n_kv, self.max_ctx, hd) if B == 1 else
                       (S.layers, B, S.n_kv, self.max_ctx, hd))
        self.k_cache = torch.zeros(cache_shape, **f32)
        self.v_cache = torch.zeros(cache_shape, **f32)
        Mx = max(self.max_prefill, B)
        self.h_a = torch.zeros((Mx, H), **f32)
        self.h_b = torch.zeros((Mx, H), **f32)
        self.xn = torch.zeros((Mx, H), **f32)
        self.qkv = torch.zeros((Mx, S.qkv_rows), **f32)
        self.qo = torch.zeros((Mx, S.n_heads * hd), **f32)
        self.ao = torch.zeros((Mx, S.n_heads * hd), **f32)
        self.gu = torch.zeros((Mx, 2 * S.inter), **f32) if Mx > 1 else None
        self.act = torch.zeros((Mx, S.inter), **f32) if Mx > 1 else None
        self.abuf = torch.zeros(S.inter, **f32)
        self.logits = torch.zeros(S.vocab, **f32) if B == 1 else torch.zeros((B, S.vocab), **f32)
        self.keys = torch.zeros(max(8, B), dtype=torch.int64, device=dev)
        self.tok = torch.zeros(B, dtype=torch.int64, device=dev)
        self.ids = torch.zeros(Mx, dtype=torch.int64, device=dev)
        self.pos_dev = torch.zeros(1, dtype=torch.int64, device=dev)
        self.pos = 0
        self.mlp_ws = torch.zeros(self.lib.qz_mlp_workspace_bytes() // 4, dtype=torch.int32,
                                  device=dev)
        b = ctypes.c_int64(0)
        with torch.cuda.device(dev):
            if B == 1:
                _lib.check(self.lib.qz_attention_decode_workspace_bytes(
                    S.n_heads, S.n_kv, hd, self.max_ctx, ctypes.byref(b)))
            else:
                _lib.check(self.lib.qz_attention_decode_batch_workspace_bytes(
                    B, S.n_heads, S.n_kv, hd, self.max_ctx, ctypes.byref(b)))
        self.attn_ws = torch.zeros(b.value, dtype=torch.uint8, device=dev)
        self.gemm_ws = None
        if Mx > 1:
            need = 0
            shapes = [(S.qkv_rows, H), (H, S.n_heads * hd), (2 * S.inter, H), (H, S.inter)]
            if B > 1:
                shapes.append((self.lm_q.shape[0], H))      # the lm_head runs M = B rows
            for N, K in shapes:
                b = ctypes.c_int64(0)
                _lib.check(self.lib.qz_gemm_w8_workspace_bytes(Mx, N, K, ctypes.byref(b)))
                need = max(need, b.value)
            self.gemm_ws = torch.empty(need, dtype=torch.uint8, device=dev)
        self._graph = None
        self._graph_steps = 0
        self.trace = None   # set to a device uint64 tensor to record phase stamps
        self.fold_norms = bool(fold_norms)   # RMSNorms inside the consuming kernels
        self.persistent = bool(persistent) and self._setup_persistent()

    def _setup_persistent(self) -> bool:
        """Use the one-launch persistent kernel (qz_decode_layers) for all layers
        of a decode token when the shapes allow it (per-row scales, head_dim 64
        or 128, ...). Measured on B200 it is parity-exact but not faster than the
        per-op launches replayed from a CUDA graph (both latency-bound at about
        35 us per Qwen3-0.6B layer), so it is opt-in."""
        S, lib = self.spec, self.lib
        per_row = all(t.shape[1] == 1 for L in self.layers
                      for t in (L.qkv_s, L.o_s, L.gu_s, L.down_s)) and self.embed_s.shape[1] == 1
        if not per_row:
            return False
        with torch.cuda.device(self.dev):
            if lib.qz_decode_layers_supported(S.hidden, S.inter, S.n_heads, S.n_kv, S.head_dim,
                                              self.max_ctx) != 0:
                return False
            b = ctypes.c_int64(0)
            _lib.check(lib.qz_decode_step_workspace_bytes(S.hidden, S.inter, S.n_heads, S.n_kv,
                                                          S.head_dim, self.max_ctx,
                                                          ctypes.byref(b)))
        self.step_ws = torch.zeros(b.value, dtype=torch.uint8, device=self.dev)
        # qz_decoder_layer records (14 pointers each) in device memory
        recs = []
        for li, L in enumerate(self.layers):
            recs.append([t.data_ptr() if t is not None else 0 for t in (
                L.qkv_q, L.qkv_s, L.o_q, L.o_s, L.gu_q, L.gu_s, L.down_q, L.down_s, L.in_w,
                L.post_w, L.qn_w, L.kn_w, self.k_cache[li], self.v_cache[li])])
        self.layer_recs = torch.tensor(recs, dtype=torch.int64).to(self.dev)
        return True

    @classmethod
    def from_quartz(cls, net, **kw) -> "DecodeEngine":
        """An engine on the int8 weights of a quantised quartz model (see
        quartz_checkpoint); keyword arguments as the constructor's."""
        spec, int8, norms = quartz_checkpoint(net)
        return cls(spec, int8, norms, **kw)

    # ------------------------------------------------------------------ state
    def reset(self, pos: int = 0) -> None:
        """Forget the sequence: the next token is written at position `pos`."""
        if not 0 <= pos <= self.max_ctx:
            raise ValueError("position outside the cache")
        self.pos = int(pos)
        self.pos_dev.fill_(self.pos)

    def load_kv(self, kv: Iterable) -> None:
        """Fill the cache from per-layer (K, V) [n_kv, T, head_dim] arrays
        ([batch, n_kv, T, head_dim] for a batched engine) and set the position
        to T (the prefilled-cache start, like calling quartz's update_and_fetch
        once per layer, quartz/cache.py:26-46)."""
        T = None
        n = 0
        B = self.batch
        for i, (k, v) in enumerate(kv):
            k = torch.as_tensor(np.ascontiguousarray(k, np.float32))
            v = torch.as_tensor(np.ascontiguousarray(v, np.float32))
            t = k.shape[-2]
            if T is None:
                T = t
            want = (self.spec.n_kv, T, self.spec.head_dim) if B == 1 else \
                (B, self.spec.n_kv, T, self.spec.head_dim)
            if tuple(k.shape) != want or v.shape != k.shape:
                raise ValueError("K/V must be [n_kv, T, head_dim] ([batch, n_kv, T, head_dim] "
                                 "for a batched engine) with one T for all layers")
            if T > self.max_ctx:
                raise ValueError("prefilled context exceeds max_ctx")
            self.k_cache[i, ..., :T, :].copy_(k)
            self.v_cache[i, ..., :T, :].copy_(v)
            n += 1
        if n != self.spec.layers:
            raise ValueError(f"expected K/V for {self.spec.layers} layers, got {n}")
        self.reset(T)

    # ------------------------------------------------------------- the token
    def _stream(self) -> int:
        return torch.cuda.current_stream(self.dev).cuda_stream

    def _decode_ops(self, st: int) -> None:
        """One token at position *pos_dev: reads self.tok, writes self.tok and
        advances pos_dev. Every call is a libquartz_b200 launch on stream st."""
        if self.batch > 1:
            return self._decode_ops_batch(st)
        S, lib, chk = self.spec, self.lib, _lib.check
        H, hd, nq, nkv = S.hidden, S.head_dim, S.n_heads, S.n_kv
        p = lambda t: t.data_ptr()  # noqa: E731
        h_a, h_b, xn = p(self.h_a), p(self.h_b), p(self.xn)
        if self.persistent:
            chk(lib.qz_decode_layers(p(self.layer_recs), S.layers, p(self.embed_q), p(self.embed_s),
                                     S.vocab, p(self.tok), p(self.pos_dev), p(self.inv_freq),
                                     p(self.norm_w), xn, H, S.inter, nq, nkv, hd, self.max_ctx,
                                     S.eps, self.attn_scale, p(self.step_ws),
                                     self.step_ws.numel(), qd._ptr(self.trace), st))
            chk(lib.qz_gemv_w8(p(self.lm_q), p(self.lm_s), self.lm_s.shape[1], xn,
                               p(self.logits), S.vocab, H, None, st))
            chk(lib.qz_argmax(p(self.logits), 1, S.vocab, p(self.keys), p(self.tok),
                              p(self.pos_dev), 1, st))
            return
        chk(lib.qz_embed_gather(p(self.embed_q), p(self.embed_s), self.embed_s.shape[1],
                                p(self.tok), 1, S.vocab, H, h_a, st))
        for li, L in enumerate(self.layers):
            kc, vc = p(self.k_cache[li]), p(self.v_cache[li])
            if self.fold_norms:
                # the input RMSNorm happens inside the qkv GEMV's activation load
                chk(lib.qz_gemv_w8_rmsnorm(p(L.qkv_q), p(L.qkv_s), L.qkv_s.shape[1], h_a,
                                           p(L.in_w), S.eps, p(self.qkv), S.qkv_rows, H, None,
                                           xn, st))
            else:
                chk(lib.qz_rmsnorm(h_a, p(L.in_w), xn, 1, H, S.eps, st))
                chk(lib.qz_gemv_w8(p(L.qkv_q), p(L.qkv_s), L.qkv_s.shape[1], xn, p(self.qkv),
                                   S.qkv_rows, H, None, st))
            chk(lib.qz_attention_decode_qkv(p(self.qkv), qd._ptr(L.qn_w), qd._ptr(L.kn_w),
                                            p(self.inv_freq), kc, vc, p(self.ao), nq, nkv, hd,
                                            self.max_ctx, 0, p(self.pos_dev), S.eps,
                                            self.attn_scale, p(self.attn_ws),
                                            self.attn_ws.numel(), st))
            chk(lib.qz_gemv_w8(p(L.o_q), p(L.o_s), L.o_s.shape[1], p(self.ao), h_b, H, nq * hd,
                               h_a, st))
            if self.fold_norms:
                # the post-attention RMSNorm happens inside the MLP's activation staging
                chk(lib.qz_fused_mlp_decode_rmsnorm(p(L.gu_q), p(L.gu_s), L.gu_s.shape[1], h_b,
                                                    p(L.post_w), S.eps, p(L.down_q),
                                                    p(L.down_s), L.down_s.shape[1], p(self.abuf),
                                                    h_a, h_b, H, S.inter, p(self.mlp_ws), xn, st))
            else:
                chk(lib.qz_rmsnorm(h_b, p(L.post_w), xn, 1, H, S.eps, st))
                chk(lib.qz_fused_mlp_decode(p(L.gu_q), p(L.gu_s), L.gu_s.shape[1], xn,
                                            p(L.down_q), p(L.down_s), L.down_s.shape[1],
                                            p(self.abuf), h_a, h_b, H, S.inter, p(self.mlp_ws),
                                            st))
        if self.fold_norms:
            chk(lib.qz_gemv_w8_rmsnorm(p(self.lm_q), p(self.lm_s), self.lm_s.shape[1], h_a,
                                       p(self.norm_w), S.eps, p(self.logits), S.vocab, H, None,
                                       xn, st))
        else:
            chk(lib.qz_rmsnorm(h_a, p(self.norm_w), xn, 1, H, S.eps, st))
            chk(lib.qz_gemv_w8(p(self.lm_q), p(self.lm_s), self.lm_s.shape[1], xn,
                               p(self.logits), S.vocab, H, None, st))
        chk(lib.qz_argmax(p(self.logits), 1, S.vocab, p(self.keys), p(self.tok), p(self.pos_dev),
                          1, st))

    def _gemm_act(self, q, s, x: int, act: int, norm_w: int | None, y: int, M: int, N: int,
                  K: int, residual: int | None, st: int) -> None:
        """The int8 GEMM of M > 1 rows on an activation of x: its RMSNorm
        (act QZ_ACT_RMSNORM, weight norm_w) or silu(g) * u of its [g | u] rows
        (QZ_ACT_SILU_MUL). With fold_norms and a tensor-path shape the
        activation is computed inside the GEMM's limb split (one kernel less);
        otherwise qz_rmsnorm / qz_silu_mul write it first. Both give the same
        values."""
        lib, chk = self.lib, _lib.check
        ws, wsb = self.gemm_ws.data_ptr(), self.gemm_ws.numel()
        if self.fold_norms and s.shape[1] == 1 and K % 16 == 0:
            chk(lib.qz_gemm_w8_act_ws(q.data_ptr(), s.data_ptr(), 1, x, act, norm_w,
                                      self.spec.eps, y, M, N, K, residual, ws, wsb, st))
            return
        if act == _lib.QZ_ACT_RMSNORM:
            chk(lib.qz_rmsnorm(x, norm_w, self.xn.data_ptr(), M, K, self.spec.eps, st))
            src = self.xn.data_ptr()
        else:
            chk(lib.qz_silu_mul(x, self.act.data_ptr(), M, K, st))
            src = self.act.data_ptr()
        chk(lib.qz_gemm_w8_ws(q.data_ptr(), s.data_ptr(), s.shape[1], src, y, M, N, K, residual,
                              ws, wsb, st))

    def _batch_layer_attn(self, li: int, L, st: int) -> None:
        """RMSNorm, q/k/v GEMM and the batched attention of layer li for the
        B rows in h_a; the attention output goes to ao."""
        S, lib, chk = self.spec, self.lib, _lib.check
        B, H, hd, nq, nkv = self.batch, S.hidden, S.head_dim, S.n_heads, S.n_kv
        p = lambda t: t.data_ptr()  # noqa: E731
        self._gemm_act(L.qkv_q, L.qkv_s, p(self.h_a), _lib.QZ_ACT_RMSNORM, p(L.in_w),
                       p(self.qkv), B, S.qkv_rows, H, None, st)
        chk(lib.qz_attention_decode_qkv_batch(
            p(self.qkv), self.qkv.shape[1], qd._ptr(L.qn_w), qd._ptr(L.kn_w), p(self.inv_freq),
            p(self.k_cache[li]), p(self.v_cache[li]), nkv * self.max_ctx * hd, p(self.ao),
            self.ao.shape[1], B, nq, nkv, hd, self.max_ctx, 0, p(self.pos_dev), S.eps,
            self.attn_scale, p(self.attn_ws), self.attn_ws.numel(), st))

    def _decode_ops_batch(self, st: int) -> None:
        """One step of B sequences at position *pos_dev: reads tok [B], writes
        tok [B] and advances pos_dev. quartz's batched decode step: every
        linear is the int8 GEMM on B rows (w8a32_gemm), the MLP the per-op
        path with the clipped SiLU (quartz/quantize.py:112-114)."""
        S, lib, chk = self.spec, self.lib, _lib.check
        B, H, hd, nq, I = self.batch, S.hidden, S.head_dim, S.n_heads, S.inter
        p = lambda t: t.data_ptr()  # noqa: E731
        h_a, h_b = p(self.h_a), p(self.h_b)
        ws, wsb = p(self.gemm_ws), self.gemm_ws.numel()
        chk(lib.qz_embed_gather(p(self.embed_q), p(self.embed_s), self.embed_s.shape[1],
                                p(self.tok), B, S.vocab, H, h_a, st))
        for li, L in enumerate(self.layers):
            self._batch_layer_attn(li, L, st)
            chk(lib.qz_gemm_w8_ws(p(L.o_q), p(L.o_s), L.o_s.shape[1], p(self.ao), h_b, B, H,
                                  nq * hd, h_a, ws, wsb, st))
            self._gemm_act(L.gu_q, L.gu_s, h_b, _lib.QZ_ACT_RMSNORM, p(L.post_w), p(self.gu),
                           B, 2 * I, H, None, st)
            self._gemm_act(L.down_q, L.down_s, p(self.gu), _lib.QZ_ACT_SILU_MUL, None, h_a,
                           B, H, I, h_b, st)
        V = self.lm_q.shape[0]
        self._gemm_act(self.lm_q, self.lm_s, h_a, _lib.QZ_ACT_RMSNORM, p(self.norm_w),
                       p(self.logits), B, V, H, None, st)
        chk(lib.qz_argmax(p(self.logits), B, V, p(self.keys), p(self.tok), p(self.pos_dev), 1,
                          st))

    def _gemm_launches(self, M: int, N: int) -> int:
        """Kernels one qz_gemm_w8_ws call launches for M > 1 rows on the tensor
        path: the activation split and the GEMM, plus the split-K finish when
        the output tiles alone leave SMs idle."""
        sms = torch.cuda.get_device_properties(self.dev).multi_processor_count
        m16 = -(-M // 16) * 16
        mt = 128 if m16 >= 128 else (64 if m16 > 32 else m16)
        tiles = -(-N // 128) * (-(-M // mt))
        return 3 if tiles < sms else 2

    def _prologue_launches(self, s, K: int) -> int:
        """Launches of the RMSNorm / silu before a GEMM of K columns with
        scales s: none when _gemm_act computes it inside the limb split."""
        return 0 if self.fold_norms and s.shape[1] == 1 and K % 16 == 0 else 1

    def _launches_per_token(self) -> int:
        if self.batch > 1:
            # per step (B tokens): embed, per layer (rmsnorm, qkv GEMM, attention, o GEMM,
            # rmsnorm, gate/up GEMM, silu, down GEMM), final rmsnorm, lm_head GEMM, argmax x2;
            # a norm or the silu inside its GEMM's limb split launches nothing of its own
            S, B, g, pre = self.spec, self.batch, self._gemm_launches, self._prologue_launches
            L0 = self.layers[0]
            per_layer = (1 + pre(L0.qkv_s, S.hidden) + g(B, S.qkv_rows) + g(B, S.hidden)
                         + pre(L0.gu_s, S.hidden) + g(B, 2 * S.inter)
                         + pre(L0.down_s, S.inter) + g(B, S.hidden))
            return (1 + per_layer * S.layers + pre(self.lm_s, S.hidden)
                    + g(B, self.lm_q.shape[0]) + 2)
        if self.persistent:
            return 4   # decode_layers, lm_head GEMV, argmax + finish
        # embed + per layer (qkv with its norm, attention, o, mlp with its norm) + lm with
        # the final norm, argmax x2; attention is one launch for the fused kernel's shapes;
        # one more launch per norm when they are not folded. The library folds a norm
        # into a GEMV unless it keeps x in registers (K = 1024 with four-row groups:
        # more than 36 * (SMs - 1) rows), where the norm is a pass of its own.
        S = self.spec
        sms = torch.cuda.get_device_properties(self.dev).multi_processor_count

        def norm_pass(n_rows: int, k: int) -> int:
            return int(not self.fold_norms or (k == 1024 and n_rows > 36 * (sms - 1)))

        per_layer = 4 + norm_pass(S.qkv_rows, S.hidden) + (0 if self.fold_norms else 1)
        return 1 + per_layer * S.layers + 3 + norm_pass(S.vocab, S.hidden)

    def prefill(self, ids: Iterable[int]) -> int:
        """Run the prompt ids at the current position; return the greedy next token
        (quartz/generate.py:50 then quartz/models/common.py:69-78 on the last row)."""
        if self.batch > 1:
            raise ValueError("a batched engine decodes through generate_batch")
        ids = [int(t) for t in ids]
        M = len(ids)
        S = self.spec
        if M == 0:
            raise ValueError("empty prompt: nothing to prefill")
        if any(t < 0 or t >= S.vocab for t in ids):
            raise ValueError("token id outside the vocabulary")
        if self.pos + M > self.max_ctx:
            raise ValueError("prompt does not fit in the cache")
        if M == 1:
            return self.decode(ids[0])
        if M > self.max_prefill:
            raise ValueError(f"prompt of {M} tokens exceeds max_prefill={self.max_prefill}")
        st = self._stream()
        lib, chk = self.lib, _lib.check
        H, hd, nq, nkv, I = S.hidden, S.head_dim, S.n_heads, S.n_kv, S.inter
        p = lambda t: t.data_ptr()  # noqa: E731
        self.ids[:M].copy_(torch.tensor(ids, dtype=torch.int64))
        h_a, h_b, xn = p(self.h_a), p(self.h_b), p(self.xn)
        ws, wsb = p(self.gemm_ws), self.gemm_ws.numel()
        pos0 = self.pos
        chk(lib.qz_embed_gather(p(self.embed_q), p(self.embed_s), self.embed_s.shape[1],
                                p(self.ids), M, S.vocab, H, h_a, st))
        for li, L in enumerate(self.layers):
            kc, vc = p(self.k_cache[li]), p(self.v_cache[li])
            self._gemm_act(L.qkv_q, L.qkv_s, h_a, _lib.QZ_ACT_RMSNORM, p(L.in_w), p(self.qkv),
                           M, S.qkv_rows, H, None, st)
            chk(lib.qz_qk_rope(p(self.qkv), qd._ptr(L.qn_w), qd._ptr(L.kn_w), p(self.inv_freq),
                               p(self.qo), kc, vc, M, nq, nkv, hd, self.max_ctx, pos0, None,
                               S.eps, st))
            chk(lib.qz_attention_prefill(p(self.qo), kc, vc, p(self.ao), M, nq, nkv, hd,
                                         self.max_ctx, pos0, self.attn_scale, st))
            chk(lib.qz_gemm_w8_ws(p(L.o_q), p(L.o_s), L.o_s.shape[1], p(self.ao), h_b, M, H,
                                  nq * hd, h_a, ws, wsb, st))
            self._gemm_act(L.gu_q, L.gu_s, h_b, _lib.QZ_ACT_RMSNORM, p(L.post_w), p(self.gu),
                           M, 2 * I, H, None, st)
            self._gemm_act(L.down_q, L.down_s, p(self.gu), _lib.QZ_ACT_SILU_MUL, None, h_a,
                           M, H, I, h_b, st)
        last = h_a + (M - 1) * H * 4
        chk(lib.qz_rmsnorm(last, p(self.norm_w), xn, 1, H, S.eps, st))
        chk(lib.qz_gemv_w8(p(self.lm_q), p(self.lm_s), self.lm_s.shape[1], xn, p(self.logits),
                           S.vocab, H, None, st))
        self.pos_dev.fill_(pos0)
        chk(lib.qz_argmax(p(self.logits), 1, S.vocab, p(self.keys), p(self.tok), p(self.pos_dev),
                          M, st))
        self.pos = pos0 + M
        return int(self.tok.item())

    def decode(self, token: int) -> int:
        """One eager decode step from `token`; returns the greedy next token."""
        if self.batch > 1:
            raise ValueError("a batched engine decodes through generate_batch")
        if not 0 <= token < self.spec.vocab:
            raise ValueError("token id outside the vocabulary")
        if self.pos >= self.max_ctx:
            raise ValueError("the cache is full")
        self.tok.fill_(int(token))
        self.pos_dev.fill_(self.pos)
        self._decode_ops(self._stream())
        self.pos += 1
        return int(self.tok.item())

    # ----------------------------------------------------------- graph replay
    def capture(self, steps: int = 8) -> None:
        """Capture `steps` consecutive decode steps (each followed by a copy of
        its token into a device history slot) into one CUDA graph."""
        steps = max(1, int(steps))
        self._graph = None
        self.hist = torch.zeros(steps if self.batch == 1 else (steps, self.batch),
                                dtype=torch.int64, device=self.dev)
        # One eager step first, so every launch path (kernel attributes, the
        # cooperative-launch form) is settled outside the capture. It writes the
        # cache row at the current position, which the next real step rewrites;
        # token and device position are restored.
        tok0 = self.tok.clone()
        if self.pos < self.max_ctx:
            self.pos_dev.fill_(self.pos)
            self._decode_ops(self._stream())
            self.tok.copy_(tok0)
            self.pos_dev.fill_(self.pos)
        side = torch.cuda.Stream(self.dev)
        side.wait_stream(torch.cuda.current_stream(self.dev))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            with torch.cuda.graph(g, stream=side):
                st = side.cuda_stream
                for i in range(steps):
                    self._decode_ops(st)
                    self.hist[i:i + 1].copy_(self.tok.view(1, -1) if self.batch > 1 else self.tok)
        torch.cuda.current_stream(self.dev).wait_stream(side)
        self._graph = g
        self._graph_steps = steps

    def replay(self) -> torch.Tensor:
        """Run the captured steps from the current device token and position;
        returns the device history of their tokens."""
        if self._graph is None:
            raise RuntimeError("capture() first")
        if self.pos + self._graph_steps > self.max_ctx:
            raise ValueError("the cache would overflow")
        self._graph.replay()
        self.pos += self._graph_steps
        return self.hist

    def generate(self, first: int, steps: int, *, graph: bool = True, unroll: int = 8
                 ) -> list[int]:
        """Greedy tokens after feeding `first` at the current position: the
        decode loop of quartz/generate.py:52-58 (without EOS handling), `steps`
        tokens, the first being the argmax of `first`'s logits."""
        if self.batch > 1:
            raise ValueError("a batched engine decodes through generate_batch")
        if steps <= 0:
            return []
        if self.pos + steps > self.max_ctx:
            raise ValueError("generation would overflow the cache")
        if not 0 <= first < self.spec.vocab:
            raise ValueError("token id outside the vocabulary")
        if not graph:
            out, tok = [], first
            for _ in range(steps):
                tok = self.decode(tok)
                out.append(tok)
            return out
        if self._graph is None or self._graph_steps != unroll:
            self.capture(unroll)
        out = torch.empty(steps, dtype=torch.int64, device=self.dev)
        self.tok.fill_(int(first))
        self.pos_dev.fill_(self.pos)
        st = self._stream()
        done = 0
        while steps - done >= self._graph_steps:
            h = self.replay()
            out[done:done + self._graph_steps].copy_(h)
            done += self._graph_steps
        while done < steps:
            self._decode_ops(st)
            out[done:done + 1].copy_(self.tok)
            self.pos += 1
            done += 1
        return out.cpu().tolist()

    def generate_batch(self, firsts, steps: int, *, graph: bool = True, unroll: int = 8
                       ) -> list[list[int]]:
        """Greedy tokens of the B sequences after feeding firsts[b] to sequence b
        at the current (shared) position: `steps` rows of B tokens, row 0 the
        argmax of each sequence's logits for its first token."""
        firsts = [int(t) for t in firsts]
        if len(firsts) != self.batch:
            raise ValueError(f"expected {self.batch} first tokens, got {len(firsts)}")
        if any(t < 0 or t >= self.spec.vocab for t in firsts):
            raise ValueError("token id outside the vocabulary")
        if steps <= 0:
            return []
        if self.pos + steps > self.max_ctx:
            raise ValueError("generation would overflow the cache")
        self.tok.copy_(torch.tensor(firsts, dtype=torch.int64))
        self.pos_dev.fill_(self.pos)
        st = self._stream()
        out = torch.empty((steps, self.batch), dtype=torch.int64, device=self.dev)
        done = 0
        if graph:
            if self._graph is None or self._graph_steps != unroll:
                self.capture(unroll)
                self.tok.copy_(torch.tensor(firsts, dtype=torch.int64))
            self.pos_dev.fill_(self.pos)
            while steps - done >= self._graph_steps:
                h = self.replay()
                out[done:done + self._graph_steps].copy_(h.view(self._graph_steps, self.batch))
                done += self._graph_steps
        while done < steps:
            self._decode_ops(st)
            out[done].copy_(self.tok)
            self.pos += 1
            done += 1
        return out.cpu().tolist()
