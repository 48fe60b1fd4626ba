"""Drop-in replacements for quartz/kernels/int8.py, running on a B200.

Same names, argument order, out-parameter convention and errors as the
reference module; the arithmetic runs in the sm_100a kernels of
libquartz_b200.so. Arguments may be numpy arrays (the reference's contract:
results are in `y` / `Y` when the call returns) or CUDA torch tensors (no host
copies; stream-ordered like any torch op).

Weights passed as numpy arrays are copied to the GPU once and kept resident
(see quartz_b200/_host.py); activations and outputs travel per call.
"""

from __future__ import annotations

import numpy as np
import torch

from .. import _host, _lib
from .. import device as _dev

# The reference routes int8 GEMVs below this many weight bytes to a serial
# Numba twin (quartz/kernels/int8.py:45, 101-105) because a CPU thread-pool
# fork-join costs more than the work. On the GPU the same split is a launch
# shape (grid = min(row groups, SMs)); the constant is kept for callers that
# read it.
PRANGE_BYTES = 2_500_000


def _is_torch(*xs) -> bool:
    return any(isinstance(x, torch.Tensor) for x in xs)


def _dev_index() -> int:
    return _dev.ensure_device()


# The current stream's raw handle without building a torch.cuda.Stream object
# (a few microseconds a call on the host, which the numpy GEMV pays every call).
_raw_stream_fn = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _raw_stream(d: int) -> int:
    if _raw_stream_fn is not None:
        return _raw_stream_fn(d)
    return torch.cuda.current_stream(d).cuda_stream


def _check_np(q, scale):
    if not isinstance(q, np.ndarray) or q.dtype != np.int8 or q.ndim != 2:
        raise TypeError("q must be a 2-D int8 numpy array")
    if not isinstance(scale, np.ndarray) or scale.dtype != np.float32 or scale.ndim != 2:
        raise TypeError("scale must be a 2-D float32 numpy array")
    if scale.shape[0] != q.shape[0]:
        raise ValueError("scale and q disagree on the number of rows")
    if q.shape[1] % scale.shape[1]:
        raise ValueError(f"scale has {scale.shape[1]} groups that do not tile K={q.shape[1]}")


def _check_out(y, shape, name):
    if not isinstance(y, np.ndarray) or y.dtype != np.float32 or y.shape != tuple(shape):
        raise TypeError(f"{name} must be a float32 numpy array of shape {tuple(shape)}")
    if not y.flags["C_CONTIGUOUS"] or not y.flags["WRITEABLE"]:
        raise ValueError(f"{name} must be C-contiguous and writeable")


def w8a32_gemv(q, scale, x, y) -> None:
    """One activation row against int8 weights: y[n] = sum over scale groups g
    of scale[n, g] * sum_j x[g*G + j] * q[n, g*G + j], with q [N, K] int8,
    scale [N, ng] float32 (G = K / ng), x [K] and the output y [N] float32,
    written in place. Same signature as quartz/kernels/int8.py:24-38."""
    if _is_torch(q, scale, x, y):
        _dev.gemv(q, scale, x.reshape(-1), y)
        return
    _check_np(q, scale)
    N, K = q.shape
    if x.shape != (K,):
        raise ValueError(f"x must have shape ({K},), got {x.shape}")
    _check_out(y, (N,), "y")
    d = _dev_index()
    qd, sd = _host.resident(q, d), _host.resident(scale, d)
    if x.dtype != np.float32 or not x.flags["C_CONTIGUOUS"]:
        x = np.ascontiguousarray(x, dtype=np.float32)
    # one library call: x in through pinned memory, the GEMV, y back in chunks
    xp, yp, xdv, ydv = _host.io_ptrs(d, 4 * K, 4 * N)
    _lib.check(_lib.load().qz_gemv_w8_host(
        qd.data_ptr(), sd.data_ptr(), scale.shape[1], x.__array_interface__["data"][0],
        y.__array_interface__["data"][0], N, K, xp, yp, xdv, ydv, _raw_stream(d)))


def w8a32_gemv_serial(q, scale, x, y) -> None:
    """The reference's serial twin (quartz/kernels/int8.py:48-63). Same kernel,
    so the output is bit-identical to w8a32_gemv, as the reference guarantees."""
    w8a32_gemv(q, scale, x, y)


def w8a32_gemm(q, scale, X, Y) -> None:
    """Several activation rows at once: Y[m] = the GEMV of X[m] for every m,
    with X [M, K] and the output Y [M, N] float32 written in place; runs on
    the tensor cores. Same signature as quartz/kernels/int8.py:66-87."""
    if _is_torch(q, scale, X, Y):
        _dev.gemm(q, scale, X, Y)
        return
    _check_np(q, scale)
    N, K = q.shape
    if X.ndim != 2 or X.shape[1] != K:
        raise ValueError(f"X must have shape (M, {K}), got {X.shape}")
    M = X.shape[0]
    _check_out(Y, (M, N), "Y")
    d = _dev_index()
    qd, sd = _host.resident(q, d), _host.resident(scale, d)
    Xd = _host.to_device(X, "x", d)
    Yd = _host.out_buffer((M, N), "y", d)
    _dev.gemm(qd, sd, Xd, Yd)
    _host.to_host(Yd, Y, "y")


def matmul_int8(q, scale, x):
    """y = x @ dequant(q, scale).T for x of shape (..., K). quartz/kernels/int8.py:90-108.

    Raises ValueError when the scale groups do not tile K. M == 1 runs the
    HBM-streaming GEMV, M > 1 the GEMM. Returns a new array (numpy in, numpy
    out; CUDA tensor in, CUDA tensor out).
    """
    lead = tuple(x.shape[:-1])
    K = x.shape[-1]
    ng = scale.shape[1]
    if K % ng != 0:
        raise ValueError(f"scale has {ng} groups that do not tile K={K}")
    N = q.shape[0]
    if _is_torch(q, scale, x):
        xm = x.reshape(-1, K).to(torch.float32).contiguous()
        return _dev.gemm(q, scale, xm).reshape(*lead, N)
    xm = np.ascontiguousarray(x.reshape(-1, K), dtype=np.float32)
    M = xm.shape[0]
    y = np.empty((M, N), dtype=np.float32)
    if M == 1:
        w8a32_gemv(q, scale, xm[0], y[0])
    else:
        w8a32_gemm(q, scale, xm, y)
    return y.reshape(*lead, N)


def warmup() -> None:
    """Initialise the device and run each kernel once on tiny inputs (the
    reference JIT-compiles here, quartz/kernels/int8.py:111-117)."""
    q = np.ones((2, 4), dtype=np.int8)
    s = np.ones((2, 1), dtype=np.float32)
    w8a32_gemv(q, s, np.ones(4, np.float32), np.zeros(2, np.float32))
    w8a32_gemv_serial(q, s, np.ones(4, np.float32), np.zeros(2, np.float32))
    w8a32_gemm(q, s, np.ones((2, 4), np.float32), np.zeros((2, 2), np.float32))
    q16 = np.ones((8, 32), dtype=np.int8)
    s16 = np.ones((8, 1), dtype=np.float32)
    w8a32_gemv(q16, s16, np.ones(32, np.float32), np.zeros(8, np.float32))
