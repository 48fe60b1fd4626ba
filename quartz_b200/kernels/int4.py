"""int4 weight GEMV with the numpy signature of the int8 path.

quartz itself has no 4-bit kernel (its config keeps a ``bits`` field for it
as future work, quartz/config.py:98); this is the same call as
``w8a32_gemv`` (quartz/kernels/int8.py:24-38) for weights packed two per
byte by ``quartz_b200.quantize.quantize_symmetric_int4``, halving the bytes
the GEMV streams. Numpy arguments: results in ``y`` on return; CUDA tensors:
stream-ordered, no host copies.
"""

from __future__ import annotations

import numpy as np
import torch

from .. import _host
from .. import device as _dev


def w4a32_gemv(q4, scale, x, y) -> None:
    """Decode GEMV (M=1) on int4 weights. q4:(N,K/2) uint8 packed; scale:(N,ng)
    f32; x:(K,) f32; y:(N,) f32 out. y[n] = sum_g scale[n,g] * sum_j x[gG+j] q[n,gG+j].
    K and K // ng must be multiples of 32; exact for |x| < 2^43."""
    if any(isinstance(t, torch.Tensor) for t in (q4, scale, x, y)):
        _dev.gemv_w4(q4, scale, x.reshape(-1), y)
        return
    if not isinstance(q4, np.ndarray) or q4.dtype != np.uint8 or q4.ndim != 2:
        raise TypeError("q4 must be a 2-D uint8 numpy array (two int4 weights per byte)")
    if not isinstance(scale, np.ndarray) or scale.dtype != np.float32 or scale.ndim != 2:
        raise TypeError("scale must be a 2-D float32 numpy array")
    N, K = q4.shape[0], 2 * q4.shape[1]
    if scale.shape[0] != N:
        raise ValueError("scale and q4 disagree on the number of rows")
    if K % scale.shape[1]:
        raise ValueError(f"scale has {scale.shape[1]} groups that do not tile K={K}")
    if x.shape != (K,):
        raise ValueError(f"x must have shape ({K},), got {x.shape}")
    if not isinstance(y, np.ndarray) or y.dtype != np.float32 or y.shape != (N,):
        raise TypeError(f"y must be a float32 numpy array of shape ({N},)")
    if not y.flags["C_CONTIGUOUS"] or not y.flags["WRITEABLE"]:
        raise ValueError("y must be C-contiguous and writeable")
    d = _dev.ensure_device()
    qd, sd = _host.resident(q4, d), _host.resident(scale, d)
    xd = _host.to_device(x, "x", d)
    yd = _host.out_buffer((N,), "y", d)
    _dev.gemv_w4(qd, sd, xd, yd)
    _host.to_host(yd, y, "y")
