"""Tensor / vocab parallelism for the int8 path over torch.distributed (NCCL).

quartz itself is single-process (no parallelism beyond its CPU thread pool);
these are the partitions the B200 build adds for models whose lm_head and MLP
outgrow one GPU's bandwidth budget (e.g. Qwen3-8B):

* ShardedLMHead -- vocab (column) parallel: rank r owns the contiguous vocab
  rows [lo_r, hi_r) of q and scale. Greedy decoding needs only the argmax, so
  each rank reduces its logits to (max, first index of max) per row and one
  all-gather of those pairs picks the winner, ties going to the lowest global
  index exactly as np.argmax over the full row (quartz/sample.py:21-22).
  ``logits()`` all-gathers the full rows when they are needed.
* ShardedMLP -- gate/up column-parallel, down row-parallel: rank r owns the
  intermediate units [lo_r, hi_r): their gate and up rows (stacked gate-first,
  as quartz/quantize.py:95-96 stacks them) and the matching columns of down.
  Each rank computes a partial [M, H] down projection; one all-reduce (sum)
  completes it and the residual is added after the reduce. A per-row down
  scale distributes over the partial sums; per-group down scales need shard
  boundaries on group boundaries, which the unit split respects.

Local compute goes through an ``ops`` object with ``gemv``, ``gemm``,
``fused_mlp`` and ``silu_mul`` (default: the CUDA kernels in
quartz_b200.device), so the partition logic can also run on CPU ranks.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def shard_range(n: int, world: int, rank: int, align: int = 1) -> tuple[int, int]:
    """Balanced contiguous split of [0, n) into `world` parts on multiples of
    `align` (the last part takes the remainder): the range of part `rank`."""
    if n % align:
        raise ValueError(f"{n} is not a multiple of the alignment {align}")
    units = n // align
    lo = units * rank // world
    hi = units * (rank + 1) // world
    return lo * align, hi * align


def _world(group) -> tuple[int, int]:
    return dist.get_rank(group), dist.get_world_size(group)


def _unit_alignment(intermediate: int, ngd: int) -> int:
    """Shard boundaries of the intermediate units: free with a per-row down
    scale (ngd == 1), on down-scale group boundaries otherwise."""
    return 1 if ngd == 1 else intermediate // ngd


def _default_ops():
    from . import device
    return device


class ShardedLMHead:
    """Vocab-parallel int8 lm_head. q: [V, H] int8, scale: [V, ng] fp32 (full
    tensors, any device; this rank keeps only its rows)."""

    def __init__(self, q: torch.Tensor, scale: torch.Tensor, *, group=None, device=None,
                 ops=None):
        self.group = group
        self.rank, self.world = _world(group)
        self.ops = ops or _default_ops()
        V, H = q.shape
        self.V, self.H = V, H
        self.lo, self.hi = shard_range(V, self.world, self.rank)
        dev = device if device is not None else q.device
        self.q = q[self.lo:self.hi].contiguous().to(dev)
        self.scale = scale[self.lo:self.hi].contiguous().to(dev)
        self.device = self.q.device
        # all_gather needs equal sizes: shards are padded to the largest one
        self.pad = max(hi - lo for lo, hi in (shard_range(V, self.world, r)
                                              for r in range(self.world)))

    @classmethod
    def from_local(cls, q_local: torch.Tensor, s_local: torch.Tensor, vocab: int, *, group=None,
                   ops=None) -> "ShardedLMHead":
        """Wrap this rank's own rows (those shard_range(vocab, world, rank) names)."""
        self = cls.__new__(cls)
        self.group = group
        self.rank, self.world = _world(group)
        self.ops = ops or _default_ops()
        self.V, self.H = vocab, q_local.shape[1]
        self.lo, self.hi = shard_range(vocab, self.world, self.rank)
        if q_local.shape[0] != self.hi - self.lo:
            raise ValueError("q_local does not hold this rank's vocab rows")
        self.q, self.scale, self.device = q_local, s_local, q_local.device
        self.pad = max(hi - lo for lo, hi in (shard_range(vocab, self.world, r)
                                              for r in range(self.world)))
        return self

    def local_logits(self, h: torch.Tensor) -> torch.Tensor:
        """[M, hi - lo] logits of this rank's vocab rows for h [M, H]."""
        h2 = h.reshape(-1, self.H).to(torch.float32).contiguous()
        if h2.shape[0] == 1:
            return self.ops.gemv(self.q, self.scale, h2[0]).reshape(1, -1)
        return self.ops.gemm(self.q, self.scale, h2)

    def argmax(self, h: torch.Tensor) -> torch.Tensor:
        """Greedy token per row of h: int64 [M], identical on every rank."""
        loc = self.local_logits(h)
        M = loc.shape[0]
        if loc.shape[1] > 0:
            val, idx = loc.max(dim=1)          # first index of the max, like np.argmax
        else:
            val = torch.full((M,), float("-inf"), device=loc.device)
            idx = torch.zeros(M, dtype=torch.int64, device=loc.device)
        pair = torch.stack([val.to(torch.float64), (idx + self.lo).to(torch.float64)], dim=1)
        out = torch.empty((self.world * M, 2), dtype=torch.float64, device=pair.device)
        dist.all_gather_into_tensor(out, pair.contiguous(), group=self.group)
        out = out.view(self.world, M, 2)
        vals, gidx = out[..., 0], out[..., 1]
        best = vals.max(dim=0).values
        # lowest global index among the ranks holding the maximum
        cand = torch.where(vals == best.unsqueeze(0), gidx, torch.full_like(gidx, float("inf")))
        return cand.min(dim=0).values.to(torch.int64)

    def logits(self, h: torch.Tensor) -> torch.Tensor:
        """Full [M, V] logits on every rank."""
        loc = self.local_logits(h)
        M = loc.shape[0]
        padded = torch.zeros((M, self.pad), dtype=torch.float32, device=loc.device)
        padded[:, :loc.shape[1]] = loc
        out = torch.empty((self.world * M, self.pad), dtype=torch.float32, device=loc.device)
        dist.all_gather_into_tensor(out, padded.contiguous(), group=self.group)
        out = out.view(self.world, M, self.pad)
        parts = []
        for r in range(self.world):
            lo, hi = shard_range(self.V, self.world, r)
            parts.append(out[r, :, :hi - lo])
        return torch.cat(parts, dim=1)


class ShardedMLP:
    """Tensor-parallel int8 SwiGLU MLP. Full tensors: gate/up q [I, H] with
    scales [I, ng]; down q [H, I] with scale [H, ngd]."""

    def __init__(self, gate_q, gate_s, up_q, up_s, down_q, down_s, *, group=None, device=None,
                 ops=None):
        self.group = group
        self.rank, self.world = _world(group)
        self.ops = ops or _default_ops()
        I, H = gate_q.shape
        self.I, self.H = I, H
        ngd = down_s.shape[1]
        if I % ngd:
            raise ValueError("down scale groups do not tile the intermediate size")
        align = _unit_alignment(I, ngd)
        self.lo, self.hi = shard_range(I, self.world, self.rank, align=align)
        dev = device if device is not None else gate_q.device
        lo, hi = self.lo, self.hi
        self.gu_q = torch.cat([gate_q[lo:hi], up_q[lo:hi]], 0).contiguous().to(dev)
        self.gu_s = torch.cat([gate_s[lo:hi], up_s[lo:hi]], 0).contiguous().to(dev)
        self.down_q = down_q[:, lo:hi].contiguous().to(dev)
        # one scale per down row applies to every partial sum; per-group scales
        # go with their groups
        ds = down_s if ngd == 1 else down_s[:, lo // align:hi // align]
        self.down_s = ds.contiguous().to(dev)
        self.device = self.gu_q.device

    @classmethod
    def from_local(cls, gu_q, gu_s, down_q, down_s, intermediate: int, *, group=None,
                   ops=None) -> "ShardedMLP":
        """Wrap this rank's own units: stacked gate|up rows [2 I_r, H] and the
        matching down columns [H, I_r] (units shard_range(I, world, rank))."""
        self = cls.__new__(cls)
        self.group = group
        self.rank, self.world = _world(group)
        self.ops = ops or _default_ops()
        self.I, self.H = intermediate, gu_q.shape[1]
        self.lo, self.hi = shard_range(intermediate, self.world, self.rank,
                                       align=_unit_alignment(intermediate, down_s.shape[1]))
        self.gu_q, self.gu_s, self.down_q, self.down_s = gu_q, gu_s, down_q, down_s
        self.device = gu_q.device
        return self

    def partial(self, x: torch.Tensor) -> torch.Tensor:
        """This rank's [M, H] share of down(silu(gate.x) * (up.x))."""
        x2 = x.reshape(-1, self.H).to(torch.float32).contiguous()
        M = x2.shape[0]
        if self.hi == self.lo:
            return torch.zeros((M, self.H), dtype=torch.float32, device=self.device)
        if M == 1:
            # quartz/kernels/fused.py:27-65 on the local units
            return self.ops.fused_mlp(self.gu_q, self.gu_s, x2[0], self.down_q,
                                      self.down_s).reshape(1, self.H)
        # quartz/quantize.py:112-114 on the local units
        gu = self.ops.gemm(self.gu_q, self.gu_s, x2)
        a = self.ops.silu_mul(gu)
        return self.ops.gemm(self.down_q, self.down_s, a)

    def __call__(self, x: torch.Tensor, residual: torch.Tensor | None = None) -> torch.Tensor:
        out = self.partial(x)
        dist.all_reduce(out, op=dist.ReduceOp.SUM, group=self.group)
        if residual is not None:
            out = out + residual.reshape(out.shape)
        return out.reshape(*x.shape[:-1], self.H)
