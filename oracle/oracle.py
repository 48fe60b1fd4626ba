"""ctypes front end of the C oracle plus numpy restatements of the host glue.

TEST INFRASTRUCTURE ONLY -- the checker and the CPU baseline, never the product.

* ``w8a32_gemv`` / ``w8a32_gemm`` / ``fused_mlp_decode`` call qz_oracle.c, the
  loop-for-loop restatement of quartz/kernels/int8.py:24-87 and
  quartz/kernels/fused.py:27-65, with the reference's argument order and
  out-parameter convention.
* ``matmul_int8`` restates the dispatcher quartz/kernels/int8.py:90-108
  (flatten to [M, K], K % ng check, M == 1 -> GEMV, else GEMM).
* ``mlp_per_op`` restates the M > 1 FusedMLP fallback quartz/quantize.py:112-114
  with the clipped silu of quartz/ops.py:35-37.
* ``w4a32_gemv`` is the int4 GEMV in numpy: the int8 GEMV's group sums on
  weights unpacked from two-per-byte nibbles. quartz has no 4-bit kernel, so
  this one is pinned to nothing but its own definition (parity unpinned).
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_lib = None

_i8p = ctypes.POINTER(ctypes.c_int8)
_f32p = ctypes.POINTER(ctypes.c_float)
_i64 = ctypes.c_int64


def _has_avx512() -> bool:
    try:
        with open("/proc/cpuinfo") as f:
            flags = f.read()
        return "avx512f" in flags and "avx512bw" in flags and "avx512vl" in flags
    except OSError:
        return False


def build() -> None:
    """Compile the oracle shared objects with its Makefile (gcc + OpenMP)."""
    subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)


def load():
    """Load (building if needed) the oracle library for this host's ISA level."""
    global _lib
    if _lib is not None:
        return _lib
    name = "libqz_oracle_v4.so" if _has_avx512() else "libqz_oracle_v3.so"
    path = _HERE / name
    if not path.exists():
        build()
    lib = ctypes.CDLL(str(path))
    lib.qzo_w8a32_gemv.argtypes = [_i8p, _f32p, _i64, _i64, _i64, _f32p, _f32p]
    lib.qzo_w8a32_gemm.argtypes = [_i8p, _f32p, _i64, _i64, _i64, _f32p, _i64, _f32p]
    lib.qzo_fused_mlp_decode.argtypes = [_i8p, _f32p, _i64, _i64, _i64, _f32p,
                                         _i8p, _f32p, _i64, _f32p, _f32p]
    lib.qzo_set_threads.argtypes = [ctypes.c_int]
    lib.qzo_get_threads.restype = ctypes.c_int
    lib.isa = name
    _lib = lib
    return lib


def set_threads(n: int) -> None:
    load().qzo_set_threads(int(n))


def threads() -> int:
    return int(load().qzo_get_threads())


def _p(a, t):
    return a.ctypes.data_as(t)


def _check(q, scale, K):
    if q.dtype != np.int8 or q.ndim != 2 or not q.flags["C_CONTIGUOUS"]:
        raise TypeError("q must be a C-contiguous 2-D int8 array")
    if scale.dtype != np.float32 or scale.ndim != 2 or not scale.flags["C_CONTIGUOUS"]:
        raise TypeError("scale must be a C-contiguous 2-D float32 array")
    if scale.shape[0] != q.shape[0] or q.shape[1] != K or K % scale.shape[1]:
        raise ValueError("inconsistent q / scale / K shapes")


def w8a32_gemv(q, scale, x, y) -> None:
    """int8.py:24-38: y[n] = sum_g scale[n,g] * sum_j x[gG+j] * q[n,gG+j]."""
    N, K = q.shape
    _check(q, scale, K)
    assert x.dtype == np.float32 and x.flags["C_CONTIGUOUS"] and x.shape == (K,)
    assert y.dtype == np.float32 and y.flags["C_CONTIGUOUS"] and y.shape == (N,)
    load().qzo_w8a32_gemv(_p(q, _i8p), _p(scale, _f32p), N, K, scale.shape[1],
                          _p(x, _f32p), _p(y, _f32p))


# int8.py:48-63 computes the same rows serially; the row results are identical.
w8a32_gemv_serial = w8a32_gemv


def w8a32_gemm(q, scale, X, Y) -> None:
    """int8.py:66-87: Y[m, n] for every row m of X."""
    N, K = q.shape
    _check(q, scale, K)
    M = X.shape[0]
    assert X.dtype == np.float32 and X.flags["C_CONTIGUOUS"] and X.shape == (M, K)
    assert Y.dtype == np.float32 and Y.flags["C_CONTIGUOUS"] and Y.shape == (M, N)
    load().qzo_w8a32_gemm(_p(q, _i8p), _p(scale, _f32p), N, K, scale.shape[1],
                          _p(X, _f32p), M, _p(Y, _f32p))


def matmul_int8(q, scale, x):
    """int8.py:90-108: y = x @ dequant(q, scale).T for x of shape (..., K)."""
    lead = x.shape[:-1]
    K = x.shape[-1]
    ng = scale.shape[1]
    if K % ng != 0:
        raise ValueError(f"scale has {ng} groups that do not tile K={K}")
    xm = np.ascontiguousarray(x.reshape(-1, K), dtype=np.float32)
    M = xm.shape[0]
    N = q.shape[0]
    y = np.empty((M, N), dtype=np.float32)
    if M == 1:
        w8a32_gemv(q, scale, xm[0], y[0])
    else:
        w8a32_gemm(q, scale, xm, y)
    return y.reshape(*lead, N)


def w4a32_gemv(q4, scale, x, y) -> None:
    """int4 GEMV restated in numpy (no reference counterpart: quartz keeps
    4-bit weights as future work, quartz/config.py:98). q4 (N, K/2) uint8,
    element 2i in the low nibble of byte i, 2i+1 in the high one, two's
    complement; y[n] = sum_g scale[n,g] * sum_j f32(q[n, gG+j]) x[gG+j], the
    group sums of int8.py:24-38, accumulated in float64 and rounded once."""
    q4 = np.asarray(q4, dtype=np.uint8)
    lo = (q4 & 0x0F).astype(np.int16)
    hi = (q4 >> 4).astype(np.int16)
    q = np.empty(q4.shape[:-1] + (2 * q4.shape[-1],), np.int16)
    q[..., 0::2] = np.where(lo > 7, lo - 16, lo)
    q[..., 1::2] = np.where(hi > 7, hi - 16, hi)
    N, K = q.shape
    ng = scale.shape[1]
    G = K // ng
    part = (q.reshape(N, ng, G).astype(np.float64) * np.asarray(x, np.float64).reshape(1, ng, G)).sum(-1)
    y[...] = (part * scale.astype(np.float64)).sum(-1).astype(np.float32)


def fused_mlp_decode(gu_q, gu_s, x, down_q, down_s, abuf, out) -> None:
    """fused.py:27-65: out = down(silu(gate.x) * (up.x)), unclipped exp in silu."""
    I2, H = gu_q.shape
    I = I2 // 2
    _check(gu_q, gu_s, H)
    _check(down_q, down_s, I)
    assert down_q.shape == (H, I)
    for a, n in ((x, H), (abuf, I), (out, H)):
        assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"] and a.shape == (n,)
    load().qzo_fused_mlp_decode(_p(gu_q, _i8p), _p(gu_s, _f32p), I, H, gu_s.shape[1],
                                _p(x, _f32p), _p(down_q, _i8p), _p(down_s, _f32p),
                                down_s.shape[1], _p(abuf, _f32p), _p(out, _f32p))


def silu_clipped(x):
    """ops.py:35-37: x * sigmoid(x) with the exponent clipped to [-88, 88]."""
    return x * (1.0 / (1.0 + np.exp(-np.clip(x, -88.0, 88.0))))


def mlp_per_op(gu_q, gu_s, down_q, down_s, x):
    """quantize.py:112-114: stacked gate|up GEMM, split, clipped silu * up, down."""
    I = gu_q.shape[0] // 2
    gu = matmul_int8(gu_q, gu_s, x)
    return matmul_int8(down_q, down_s, silu_clipped(gu[..., :I]) * gu[..., I:])
