"""Tensor-parallel greedy decoding: one sequence over P GPUs (one process each).

quartz decodes on one CPU (quartz/generate.py:36-58). For models whose int8
weights outgrow one GPU's bandwidth budget per token (Qwen3-8B: 7.5 GB), the
decode step is split Megatron-style over the ranks of a process group:

* attention by heads: rank r owns query heads [r nq/P, (r+1) nq/P) and the kv
  heads they read (quartz repeats kv head g to the n_rep adjacent query heads,
  quartz/attention.py:36-38, so the split keeps whole groups); its stacked
  q/k/v rows, its slice of every KV cache and the matching columns of o_proj;
* MLP by units: gate/up rows [r I/P, (r+1) I/P) and the matching down columns
  (the split quartz_b200.sharding.ShardedMLP uses);
* lm_head by vocab rows: greedy decoding needs only the argmax, so every rank
  reduces its logits to (max, first index of max) and one all-gather of those
  pairs picks the token, ties to the lowest global index as np.argmax
  (quartz/sample.py:21-22).

Per layer the o-projection and the MLP down-projection produce partial [H]
sums; rank 0 folds the residual into its partial and one all-reduce (sum)
completes each. The embedding table and the RMSNorms are replicated. Every
rank ends each step with the same token and position.
"""

from __future__ import annotations

import ctypes
from typing import Iterable, Mapping

import numpy as np
import torch
import torch.distributed as dist

from . import _lib
from .decode import DecodeEngine
from .model import ModelSpec
from .sharding import shard_range


def tp_shard(spec: ModelSpec, int8_weights: Mapping | Iterable, rank: int, world: int
             ) -> tuple[ModelSpec, dict, tuple[np.ndarray, np.ndarray, int, int]]:
    """This rank's part of a checkpoint: (local spec, local int8 weights,
    (lm_head q rows, scale rows, lo, hi)). The local spec has the rank's head
    and unit counts, the full hidden size and vocabulary (the embedding table
    is replicated); its lm_head is the embedding's (``tie``), which the engine
    replaces by the vocab shard."""
    if spec.n_kv % world or spec.n_heads % world or spec.inter % world:
        raise ValueError(f"{world} ranks do not divide the kv heads ({spec.n_kv}), query heads "
                         f"({spec.n_heads}) and MLP units ({spec.inter}) evenly")
    hd = spec.head_dim
    nq_r, nkv_r, i_r = spec.n_heads // world, spec.n_kv // world, spec.inter // world
    local = ModelSpec(arch=spec.arch, hidden=spec.hidden, layers=spec.layers, n_heads=nq_r,
                      n_kv=nkv_r, head_dim=hd, inter=i_r, vocab=spec.vocab,
                      rope_theta=spec.rope_theta, tie=True, rope_scaling=spec.rope_scaling,
                      eps=spec.eps)
    qlo, qhi = rank * nq_r * hd, (rank + 1) * nq_r * hd       # q rows / o columns
    klo, khi = rank * nkv_r * hd, (rank + 1) * nkv_r * hd     # k and v rows
    ulo, uhi = rank * i_r, (rank + 1) * i_r                   # MLP units
    pairs = ((n, *qs) for n, qs in int8_weights.items()) \
        if isinstance(int8_weights, Mapping) else int8_weights
    out: dict[str, tuple[np.ndarray, np.ndarray]] = {}
    lm = None
    for name, q, s in pairs:
        q, s = np.asarray(q), np.asarray(s)
        leaf = name.rsplit(".", 1)[-1]
        if name == "model.embed_tokens":
            out[name] = (q, s)
            if spec.tie:
                lm = (q, s)
            continue
        if name == "lm_head":
            lm = (q, s)
            continue
        if leaf == "q_proj":
            out[name] = (q[qlo:qhi], s[qlo:qhi])
        elif leaf in ("k_proj", "v_proj"):
            out[name] = (q[klo:khi], s[klo:khi])
        elif leaf == "o_proj":
            ng = s.shape[1]
            if ng != 1:
                raise ValueError("o_proj with grouped scales is not split over heads here")
            out[name] = (np.ascontiguousarray(q[:, qlo:qhi]), s)
        elif leaf in ("gate_proj", "up_proj"):
            out[name] = (q[ulo:uhi], s[ulo:uhi])
        elif leaf == "down_proj":
            if s.shape[1] != 1:
                raise ValueError("down_proj with grouped scales is not split over units here")
            out[name] = (np.ascontiguousarray(q[:, ulo:uhi]), s)
        else:
            raise KeyError(f"unexpected weight {name!r}")
    if lm is None:
        raise ValueError("missing lm_head (tie_word_embeddings is false)")
    vlo, vhi = shard_range(spec.vocab, world, rank)
    lm_local = (np.ascontiguousarray(lm[0][vlo:vhi]), np.ascontiguousarray(lm[1][vlo:vhi]),
                vlo, vhi)
    return local, out, lm_local


class TPDecodeEngine(DecodeEngine):
    """DecodeEngine over the ranks of `group` (NCCL; one GPU per rank). All
    ranks must construct it with the same checkpoint and call the same
    methods in the same order. Decoding through the persistent kernel is not
    offered here (its layers have no collective step)."""

    def __init__(self, spec: ModelSpec, int8_weights: Mapping | Iterable | None, norms: Mapping,
                 *, group=None, max_ctx: int, max_prefill: int = 512, device=None,
                 presharded=None, allreduce: str = "fused", batch: int = 1):
        """int8_weights: the full checkpoint (every rank slices its part with
        tp_shard), or None with presharded = tp_shard(...)'s result for this
        rank (arrays may be torch tensors already on the device).
        allreduce: how the per-token [H] partials are summed. "fused": the
        o-projection GEMV and the fused MLP push their rows to the ranks from
        their epilogues and the following RMSNorm sums them as it reads
        (no collective launches); "peer": the peer-memory all-reduce kernel
        (quartz_b200.comm); "nccl": the process group's all-reduce. Prefill's
        [M, H] sums always use NCCL.
        batch: sequences decoded in lockstep (DecodeEngine's batch); their
        [B, H] partial sums go through the peer all-reduce kernel ("fused" and
        "peer") or NCCL ("nccl"), since the in-kernel push serves one row."""
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.full_spec = spec
        local, w, (lq, ls, vlo, vhi) = (presharded if presharded is not None else
                                        tp_shard(spec, int8_weights, self.rank, self.world))
        super().__init__(local, w, norms, max_ctx=max_ctx, max_prefill=max_prefill,
                         device=device, persistent=False, batch=batch)
        self.lm_q = _to_dev(lq, torch.int8, self.dev)
        self.lm_s = _to_dev(ls, torch.float32, self.dev)
        self.vlo, self.vhi = vlo, vhi
        B = self.batch
        n_local = max(vhi - vlo, 1)
        self.logits = torch.zeros(n_local if B == 1 else (B, n_local), dtype=torch.float32,
                                  device=self.dev)
        self.ltok = torch.zeros(B, dtype=torch.int64, device=self.dev)
        self.pair = torch.zeros((B, 2), dtype=torch.float64, device=self.dev)
        self.pairs = torch.zeros((self.world * B, 2), dtype=torch.float64, device=self.dev)
        if allreduce not in ("fused", "peer", "nccl"):
            raise ValueError("allreduce must be 'fused', 'peer' or 'nccl'")
        self.peer = None
        self.fused_ar = allreduce == "fused" and self.world > 1 and B == 1
        if allreduce in ("fused", "peer") and self.world > 1:
            from .comm import PeerAllReduce
            self.peer = PeerAllReduce(self.spec.hidden * B, group=group, device=self.dev)
        if self.fused_ar:
            self.peer_sum = ctypes.byref(self.peer.ps)

    def close(self) -> None:
        """Release the graph (it may hold collectives) and the peer buffers;
        every rank calls it before the process group goes."""
        self._graph = None
        if self.peer is not None:
            self.peer.close()
            self.peer = None

    def load_kv(self, kv: Iterable) -> None:
        """Per layer full (K, V) [n_kv, T, head_dim]: this rank keeps its kv heads."""
        n = self.spec.n_kv
        lo = self.rank * n
        ax = 0 if self.batch == 1 else 1      # batched caches are [B, n_kv, T, hd]
        sl = (slice(None),) * ax + (slice(lo, lo + n),)
        super().load_kv((np.asarray(k)[sl], np.asarray(v)[sl]) for k, v in kv)

    # -------------------------------------------------------------- collectives
    def _all_reduce(self, t: torch.Tensor) -> None:
        if self.peer is not None and t.numel() <= self.peer.n_max:
            self.peer(t)
        else:
            dist.all_reduce(t, op=dist.ReduceOp.SUM, group=self.group)

    def _pick_token(self, st: int, pos_step: int) -> None:
        """Greedy token over the vocab shards: local argmax, then one all-gather
        of (max value, global index) and the lowest index among the maxima."""
        S, lib, chk = self.spec, self.lib, _lib.check
        B = self.batch
        n_local = self.vhi - self.vlo
        if n_local > 0:
            chk(lib.qz_argmax(self.logits.data_ptr(), B, n_local, self.keys.data_ptr(),
                              self.ltok.data_ptr(), None, 0, st))
            self.pair[:, 0].copy_(self.logits.view(B, -1).gather(1, self.ltok.view(B, 1))[:, 0])
            self.pair[:, 1].copy_(self.ltok + self.vlo)
        else:
            self.pair[:, 0].fill_(float("-inf"))
            self.pair[:, 1].fill_(float(S.vocab))
        dist.all_gather_into_tensor(self.pairs, self.pair, group=self.group)
        vals = self.pairs[:, 0].view(self.world, B)
        idx = self.pairs[:, 1].view(self.world, B)
        best = vals.max(dim=0, keepdim=True).values
        cand = torch.where(vals == best, idx, torch.full_like(idx, float("inf")))
        self.tok.copy_(cand.min(dim=0).values.to(torch.int64))
        self.pos_dev.add_(pos_step)

    # ------------------------------------------------------------- the token
    def _decode_ops_fused(self, st: int) -> None:
        """The token with the all-reduces inside the kernels: producers push,
        the next RMSNorm sums (see the constructor's allreduce="fused")."""
        S, lib, chk = self.spec, self.lib, _lib.check
        H, hd, nq, nkv = S.hidden, S.head_dim, S.n_heads, S.n_kv
        p = lambda t: t.data_ptr()  # noqa: E731
        h_a, h_b, xn = p(self.h_a), p(self.h_b), p(self.xn)
        first = self.rank == 0
        ps = self.peer_sum
        chk(lib.qz_embed_gather(p(self.embed_q), p(self.embed_s), self.embed_s.shape[1],
                                p(self.tok), 1, S.vocab, H, h_a, st))
        chk(lib.qz_rmsnorm(h_a, p(self.layers[0].in_w), xn, 1, H, S.eps, st))
        for li, L in enumerate(self.layers):
            kc, vc = p(self.k_cache[li]), p(self.v_cache[li])
            chk(lib.qz_gemv_w8(p(L.qkv_q), p(L.qkv_s), L.qkv_s.shape[1], xn, p(self.qkv),
                               S.qkv_rows, H, None, st))
            chk(lib.qz_attention_decode_qkv(p(self.qkv), _ptr(L.qn_w), _ptr(L.kn_w),
                                            p(self.inv_freq), kc, vc, p(self.ao), nq, nkv, hd,
                                            self.max_ctx, 0, p(self.pos_dev), S.eps,
                                            self.attn_scale, p(self.attn_ws),
                                            self.attn_ws.numel(), st))
            # o-projection partials (rank 0 adds the residual) go to every rank
            chk(lib.qz_gemv_w8_peer(p(L.o_q), p(L.o_s), L.o_s.shape[1], p(self.ao), H, nq * hd,
                                    h_a if first else None, ps, st))
            chk(lib.qz_rmsnorm_peer_sum(ps, H, p(L.post_w), S.eps, h_b, xn, st))
            chk(lib.qz_fused_mlp_decode_peer(p(L.gu_q), p(L.gu_s), L.gu_s.shape[1], xn,
                                             p(L.down_q), p(L.down_s), L.down_s.shape[1],
                                             p(self.abuf), h_b if first else None, H, S.inter,
                                             p(self.mlp_ws), ps, st))
            # the sum, normalised for what comes next (the next layer or the lm_head)
            nw = self.layers[li + 1].in_w if li + 1 < len(self.layers) else self.norm_w
            chk(lib.qz_rmsnorm_peer_sum(ps, H, p(nw), S.eps, h_a, xn, st))
        n_local = self.vhi - self.vlo
        if n_local > 0:
            chk(lib.qz_gemv_w8(p(self.lm_q), p(self.lm_s), self.lm_s.shape[1], xn,
                               p(self.logits), n_local, H, None, st))
        self._pick_token(st, 1)

    def _decode_ops_batch(self, st: int) -> None:
        """One step of the B sequences on this rank's shard: every rank runs its
        heads and units over all B rows; the o-projection and down-projection
        [B, H] partials (rank 0 carrying the residual) are summed by one
        all-reduce each; the lm_head by vocab rows with a per-row pick."""
        S, lib, chk = self.spec, self.lib, _lib.check
        B, H, hd, nq, I = self.batch, S.hidden, S.head_dim, S.n_heads, S.inter
        p = lambda t: t.data_ptr()  # noqa: E731
        h_a, h_b = p(self.h_a), p(self.h_b)
        ws, wsb = p(self.gemm_ws), self.gemm_ws.numel()
        first = self.rank == 0
        chk(lib.qz_embed_gather(p(self.embed_q), p(self.embed_s), self.embed_s.shape[1],
                                p(self.tok), B, S.vocab, H, h_a, st))
        for li, L in enumerate(self.layers):
            self._batch_layer_attn(li, L, st)
            chk(lib.qz_gemm_w8_ws(p(L.o_q), p(L.o_s), L.o_s.shape[1], p(self.ao), h_b, B, H,
                                  nq * hd, h_a if first else None, ws, wsb, st))
            self._all_reduce(self.h_b[:B])
            self._gemm_act(L.gu_q, L.gu_s, h_b, _lib.QZ_ACT_RMSNORM, p(L.post_w), p(self.gu),
                           B, 2 * I, H, None, st)
            self._gemm_act(L.down_q, L.down_s, p(self.gu), _lib.QZ_ACT_SILU_MUL, None, h_a,
                           B, H, I, h_b if first else None, st)
            self._all_reduce(self.h_a[:B])
        n_local = self.vhi - self.vlo
        if n_local > 0:
            self._gemm_act(self.lm_q, self.lm_s, h_a, _lib.QZ_ACT_RMSNORM, p(self.norm_w),
                           p(self.logits), B, n_local, H, None, st)
        self._pick_token(st, 1)

    def _decode_ops(self, st: int) -> None:
        if self.batch > 1:
            return self._decode_ops_batch(st)
        if self.fused_ar:
            return self._decode_ops_fused(st)
        S, lib, chk = self.spec, self.lib, _lib.check
        H, hd, nq, nkv = S.hidden, S.head_dim, S.n_heads, S.n_kv
        p = lambda t: t.data_ptr()  # noqa: E731
        h_a, h_b, xn = p(self.h_a), p(self.h_b), p(self.xn)
        first = self.rank == 0
        chk(lib.qz_embed_gather(p(self.embed_q), p(self.embed_s), self.embed_s.shape[1],
                                p(self.tok), 1, S.vocab, H, h_a, st))
        for li, L in enumerate(self.layers):
            kc, vc = p(self.k_cache[li]), p(self.v_cache[li])
            chk(lib.qz_rmsnorm(h_a, p(L.in_w), xn, 1, H, S.eps, st))
            chk(lib.qz_gemv_w8(p(L.qkv_q), p(L.qkv_s), L.qkv_s.shape[1], xn, p(self.qkv),
                               S.qkv_rows, H, None, st))
            chk(lib.qz_attention_decode_qkv(p(self.qkv), _ptr(L.qn_w), _ptr(L.kn_w),
                                            p(self.inv_freq), kc, vc, p(self.ao), nq, nkv, hd,
                                            self.max_ctx, 0, p(self.pos_dev), S.eps,
                                            self.attn_scale, p(self.attn_ws),
                                            self.attn_ws.numel(), st))
            # partial o-projection; rank 0 carries the residual
            chk(lib.qz_gemv_w8(p(L.o_q), p(L.o_s), L.o_s.shape[1], p(self.ao), h_b, H, nq * hd,
                               h_a if first else None, st))
            self._all_reduce(self.h_b[0])
            chk(lib.qz_rmsnorm(h_b, p(L.post_w), xn, 1, H, S.eps, st))
            chk(lib.qz_fused_mlp_decode(p(L.gu_q), p(L.gu_s), L.gu_s.shape[1], xn, p(L.down_q),
                                        p(L.down_s), L.down_s.shape[1], p(self.abuf), h_a,
                                        h_b if first else None, H, S.inter, p(self.mlp_ws), st))
            self._all_reduce(self.h_a[0])
        chk(lib.qz_rmsnorm(h_a, p(self.norm_w), xn, 1, H, S.eps, st))
        n_local = self.vhi - self.vlo
        if n_local > 0:
            chk(lib.qz_gemv_w8(p(self.lm_q), p(self.lm_s), self.lm_s.shape[1], xn,
                               p(self.logits), n_local, H, None, st))
        self._pick_token(st, 1)

    def _launches_per_token(self) -> int:
        if self.batch > 1:
            # per step: embed, per layer (qkv GEMM with its norm, attention, o GEMM,
            # [peer all-reduce], gate/up GEMM with its norm, down GEMM with the silu,
            # [peer all-reduce]), lm_head GEMM with the final norm, argmax x2 (NCCL
            # collectives and the torch ops of the vocab pick are not counted)
            S, B, g, pre = self.spec, self.batch, self._gemm_launches, self._prologue_launches
            L0, ar = self.layers[0], int(self.peer is not None)
            per_layer = (1 + pre(L0.qkv_s, S.hidden) + g(B, S.qkv_rows) + g(B, S.hidden) + ar
                         + pre(L0.gu_s, S.hidden) + g(B, 2 * S.inter)
                         + pre(L0.down_s, S.inter) + g(B, S.hidden) + ar)
            n_local = self.vhi - self.vlo
            lm = pre(self.lm_s, S.hidden) + g(B, n_local) + 2 if n_local > 0 else 0
            return 1 + per_layer * S.layers + lm
        if self.fused_ar:
            # embed, rmsnorm + per layer (qkv, attention, o, peer sum, mlp, peer sum) + lm, argmax
            return 2 + 6 * self.spec.layers + 2
        # embed + per layer (rmsnorm, qkv, attention, o, all-reduce, rmsnorm, mlp, all-reduce)
        # + norm, lm, argmax x2
        return 1 + (8 if self.peer is not None else 6) * self.spec.layers + 4

    def prefill(self, ids) -> int:
        """The prompt through the tensor-core GEMMs on each rank's shard, two
        all-reduces of [M, H] partials per layer; returns the greedy token."""
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
        first = self.rank == 0
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
            chk(lib.qz_qk_rope(p(self.qkv), _ptr(L.qn_w), _ptr(L.kn_w), p(self.inv_freq),
                               p(self.qo), kc, vc, M, nq, nkv, hd, self.max_ctx, pos0, None,
                               S.eps, st))
            chk(lib.qz_attention_prefill(p(self.qo), kc, vc, p(self.ao), M, nq, nkv, hd,
                                         self.max_ctx, pos0, self.attn_scale, st))
            chk(lib.qz_gemm_w8_ws(p(L.o_q), p(L.o_s), L.o_s.shape[1], p(self.ao), h_b, M, H,
                                  nq * hd, h_a if first else None, ws, wsb, st))
            self._all_reduce(self.h_b[:M])
            self._gemm_act(L.gu_q, L.gu_s, h_b, _lib.QZ_ACT_RMSNORM, p(L.post_w), p(self.gu),
                           M, 2 * I, H, None, st)
            self._gemm_act(L.down_q, L.down_s, p(self.gu), _lib.QZ_ACT_SILU_MUL, None, h_a,
                           M, H, I, h_b if first else None, st)
            self._all_reduce(self.h_a[:M])
        last = h_a + (M - 1) * H * 4
        chk(lib.qz_rmsnorm(last, p(self.norm_w), xn, 1, H, S.eps, st))
        n_local = self.vhi - self.vlo
        if n_local > 0:
            chk(lib.qz_gemv_w8(p(self.lm_q), p(self.lm_s), self.lm_s.shape[1], xn,
                               p(self.logits), n_local, H, None, st))
        self.pos_dev.fill_(pos0)
        self._pick_token(st, M)
        self.pos = pos0 + M
        return int(self.tok.item())


def _ptr(t):
    return None if t is None else t.data_ptr()


def _to_dev(a, dtype, dev) -> torch.Tensor:
    if isinstance(a, torch.Tensor):
        return a.to(device=dev, dtype=dtype).contiguous()
    return torch.from_numpy(np.ascontiguousarray(a)).to(device=dev, dtype=dtype)


def random_tp_shard(spec: ModelSpec, rank: int, world: int, device, seed: int = 1234):
    """A rank's shard of a synthetic checkpoint drawn on the device (int8
    uniform in [-127, 127], per-row scales in [1e-4, 3e-4]): what tp_shard
    returns, for benchmarks whose timing does not depend on the values."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed + 7919 * rank)
    hd, H = spec.head_dim, spec.hidden
    nq, nkv, I = spec.n_heads // world, spec.n_kv // world, spec.inter // world
    local = ModelSpec(arch=spec.arch, hidden=H, layers=spec.layers, n_heads=nq, n_kv=nkv,
                      head_dim=hd, inter=I, vocab=spec.vocab, rope_theta=spec.rope_theta,
                      tie=True, rope_scaling=spec.rope_scaling, eps=spec.eps)

    def q_(n, k):
        return torch.randint(-127, 128, (n, k), dtype=torch.int8, device=device, generator=gen)

    def s_(n):
        return torch.rand((n, 1), device=device, generator=gen) * 2e-4 + 1e-4

    w = {"model.embed_tokens": (q_(spec.vocab, H), s_(spec.vocab))}
    for i in range(spec.layers):
        p = f"model.layers.{i}."
        w[p + "self_attn.q_proj"] = (q_(nq * hd, H), s_(nq * hd))
        w[p + "self_attn.k_proj"] = (q_(nkv * hd, H), s_(nkv * hd))
        w[p + "self_attn.v_proj"] = (q_(nkv * hd, H), s_(nkv * hd))
        w[p + "self_attn.o_proj"] = (q_(H, nq * hd), s_(H))
        w[p + "mlp.gate_proj"] = (q_(I, H), s_(I))
        w[p + "mlp.up_proj"] = (q_(I, H), s_(I))
        w[p + "mlp.down_proj"] = (q_(H, I), s_(H))
    vlo, vhi = shard_range(spec.vocab, world, rank)
    return local, w, (q_(vhi - vlo, H), s_(vhi - vlo), vlo, vhi)
