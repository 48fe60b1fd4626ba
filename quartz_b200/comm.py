"""Peer-memory all-reduce over the GPUs of one node (qz_allreduce_sum).

Every rank allocates one communication buffer with the library (its own
cudaMalloc, so its CUDA IPC handle covers exactly that range), the ranks swap
handles once through the process group, and each rank maps its peers'
buffers. A sum is then one kernel per rank that pushes its values, each
tagged with the call's epoch in one 8-byte word, to every peer over NVLink,
polls (bounded) until the peers' words of this call have arrived and adds
them in rank order, so every rank gets bit-identical results. Small messages only:
the [H] partials of a tensor-parallel decode step, where a library
all-reduce's fixed latency dominates.
"""

from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib


class PeerSum(ctypes.Structure):
    """qz_peer_sum: every rank's buffer as mapped here, this rank, the rank
    count, the buffers' n_max."""
    _fields_ = [("buffers", ctypes.c_void_p * 8), ("rank", ctypes.c_int),
                ("ranks", ctypes.c_int), ("n_max", ctypes.c_int64)]


class PeerAllReduce:
    """In-place sums of fp32 CUDA tensors of at most `n_max` elements over the
    ranks of `group` (one GPU per rank, peer access between them). Every rank
    must make the same calls in the same order. Call close() (or drop the
    object) before destroying the process group's GPUs' contexts."""

    def __init__(self, n_max: int, *, group=None, device=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.n_max = (int(n_max) + 3) // 4 * 4
        self.lib = _lib.load()
        self.dev = torch.device("cuda", torch.cuda.current_device() if device is None
                                else torch.device(device).index)
        nb = ctypes.c_int64(0)
        _lib.check(self.lib.qz_comm_buffer_bytes(self.world, self.n_max, ctypes.byref(nb)))
        self._own = ctypes.c_void_p()
        self._opened: list[int] = []
        with torch.cuda.device(self.dev):
            _lib.check(self.lib.qz_comm_alloc(nb.value, ctypes.byref(self._own)))
            handle = ctypes.create_string_buffer(64)
            _lib.check(self.lib.qz_ipc_handle(self._own, handle))
            handles: list = [None] * self.world
            dist.all_gather_object(handles, bytes(handle.raw), group=group)
            ptrs = []
            for r, h in enumerate(handles):
                if r == self.rank:
                    ptrs.append(self._own.value)
                    continue
                p = ctypes.c_void_p()
                _lib.check(self.lib.qz_ipc_open(ctypes.create_string_buffer(h, 64), ctypes.byref(p)))
                self._opened.append(p.value)
                ptrs.append(p.value)
        self._peers = (ctypes.c_void_p * self.world)(*ptrs)
        self.ps = PeerSum((ctypes.c_void_p * 8)(*ptrs), self.rank, self.world, self.n_max)
        dist.barrier(group=group)

    def __call__(self, t: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """Sum of `t` over the ranks, into `out` (default: in place)."""
        out = t if out is None else out
        n = t.numel()
        if t.dtype != torch.float32 or not t.is_contiguous() or out.numel() != n:
            raise ValueError("fp32 contiguous tensors of equal size expected")
        if n > self.n_max:
            raise ValueError(f"{n} elements: at most {self.n_max}")
        _lib.check(self.lib.qz_allreduce_sum(t.data_ptr(), out.data_ptr(), n, self.n_max,
                                             self._peers, self.rank, self.world,
                                             torch.cuda.current_stream(self.dev).cuda_stream))
        return out

    def close(self, barrier: bool = True) -> None:
        """Unmap the peers' buffers, wait for every rank to have done the same
        (so no process still maps this rank's buffer), free it."""
        if self._own is None:
            return
        torch.cuda.synchronize(self.dev)
        with torch.cuda.device(self.dev):
            for p in self._opened:
                self.lib.qz_ipc_close(ctypes.c_void_p(p))
            self._opened = []
            if barrier and dist.is_initialized():
                dist.barrier(group=self.group)
            self.lib.qz_comm_free(self._own)
        self._own = None

    def __del__(self):
        try:
            self.close(barrier=False)
        except Exception:
            pass
