"""Host-array plumbing for the numpy-signature entry points.

* A device-resident cache of weight arrays. quartz quantises its weights once
  at load (quartz/quantize.py:134-169) and never mutates them afterwards, so
  each int8 weight and scale array is copied to the GPU on first use and reused
  while the numpy array is alive (a weakref finalizer evicts it when the array
  is freed, so a new array at a recycled address never hits a stale entry).
  Call ``invalidate(arr)`` after mutating a weight in place.
* Pinned staging buffers for per-call activations and outputs.
"""

from __future__ import annotations

import threading
import weakref

import numpy as np
import torch

_lock = threading.Lock()
_cache: dict[tuple, torch.Tensor] = {}
# id(array) -> (weakref to it, device, tensor): the per-call lookup of an
# array object seen before, without rebuilding its key from
# __array_interface__ (about 1.5 us a key on the host)
_fast: dict[int, tuple] = {}


def _key(a: np.ndarray, dev: int) -> tuple:
    return (a.__array_interface__["data"][0], a.shape, a.strides, a.dtype.str, dev)


def _evict(key) -> None:
    with _lock:
        _cache.pop(key, None)


def _drop_fast(ident: int, ref) -> None:
    with _lock:
        e = _fast.get(ident)
        if e is not None and e[0] is ref:
            del _fast[ident]


def resident(a: np.ndarray, dev: int) -> torch.Tensor:
    """Device copy of a (C-contiguous) weight array, cached for the array's lifetime."""
    e = _fast.get(id(a))
    ref = None
    if e is not None and e[0]() is a:
        if e[1] == dev:
            return e[2]
        ref = e[0]   # the same object on another device: keep its finalizer
    key = _key(a, dev)
    t = _cache.get(key)
    if t is None:
        src = torch.from_numpy(np.ascontiguousarray(a))
        t = src.to(torch.device("cuda", dev), non_blocking=False)
        with _lock:
            _cache[key] = t
        try:
            weakref.finalize(a, _evict, key)
        except TypeError:
            # Objects without weakref support (not ndarrays) are not cached.
            _evict(key)
            return t
    if ref is None:
        try:
            ref = weakref.ref(a)
            weakref.finalize(a, _drop_fast, id(a), ref)
        except TypeError:
            return t
    with _lock:
        _fast[id(a)] = (ref, dev, t)
    return t


def invalidate(a: np.ndarray | None = None) -> None:
    """Drop the cached device copy of `a` (all cached weights when None)."""
    with _lock:
        if a is None:
            _cache.clear()
            _fast.clear()
        else:
            for k in [k for k in _cache if k[:4] == _key(a, 0)[:4]]:
                del _cache[k]
            kk = _key(a, 0)[:4]
            for i in [i for i, e in _fast.items()
                      if e[0]() is not None and _key(e[0](), 0)[:4] == kk]:
                del _fast[i]


def cached_bytes() -> int:
    return sum(t.numel() * t.element_size() for t in _cache.values())


class _Staging:
    """Grow-only pinned host buffers and device buffers, one set per device."""

    def __init__(self, dev: int):
        self.dev = dev
        self.bufs: dict[str, torch.Tensor] = {}
        self.io = None

    def get(self, name: str, nbytes: int, pinned: bool) -> torch.Tensor:
        b = self.bufs.get(name)
        if b is None or b.numel() < nbytes:
            self.io = None   # cached raw pointers may name the buffer being replaced
            n = max(nbytes, 4096)
            if pinned:
                b = torch.empty(n, dtype=torch.uint8, pin_memory=True)
            else:
                b = torch.empty(n, dtype=torch.uint8, device=torch.device("cuda", self.dev))
            self.bufs[name] = b
        return b


_staging: dict[int, _Staging] = {}


def staging(dev: int) -> _Staging:
    s = _staging.get(dev)
    if s is None:
        s = _staging[dev] = _Staging(dev)
    return s


def io_ptrs(dev: int, x_bytes: int, y_bytes: int) -> tuple[int, int, int, int]:
    """Raw pointers (pinned x, pinned y, device x, device y) of the GEMV's
    staging buffers with at least these sizes; cached while they fit."""
    st = staging(dev)
    p = getattr(st, "io", None)
    if p is not None and p[0] >= x_bytes and p[1] >= y_bytes:
        return p[2]
    xb, yb = max(x_bytes, 4096), max(y_bytes, 4096)
    bufs = (st.get("x.h", xb, pinned=True), st.get("y.h", yb, pinned=True),
            st.get("x.d", xb, pinned=False), st.get("y.d", yb, pinned=False))
    ptrs = tuple(b.data_ptr() for b in bufs)
    st.io = (min(b.numel() for b in (bufs[0], bufs[2])),
             min(b.numel() for b in (bufs[1], bufs[3])), ptrs)
    return ptrs


def to_device(a: np.ndarray, name: str, dev: int) -> torch.Tensor:
    """Copy a float32 host array to a per-call device buffer through pinned memory."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    st = staging(dev)
    nbytes = a.nbytes
    host = st.get(name + ".h", nbytes, pinned=True)
    dbuf = st.get(name + ".d", nbytes, pinned=False)
    hv = host[:nbytes].view(torch.float32)
    hv.numpy()[...] = a.reshape(-1)
    dv = dbuf[:nbytes].view(torch.float32)
    dv.copy_(hv, non_blocking=True)
    return dv.view(a.shape)


def out_buffer(shape, name: str, dev: int) -> torch.Tensor:
    n = int(np.prod(shape)) * 4
    dbuf = staging(dev).get(name + ".d", n, pinned=False)
    return dbuf[:n].view(torch.float32).view(tuple(shape))


def to_host(t: torch.Tensor, out: np.ndarray, name: str) -> None:
    """Copy a device float32 tensor into the numpy array `out` (synchronising)."""
    nbytes = t.numel() * 4
    host = staging(t.device.index).get(name + ".h", nbytes, pinned=True)
    hv = host[:nbytes].view(torch.float32)
    hv.copy_(t.reshape(-1), non_blocking=True)
    torch.cuda.current_stream(t.device).synchronize()
    out.reshape(-1)[...] = hv.numpy()
