"""Drop-in replacement for quartz/kernels/fused.py, running on a B200.

``fused_mlp_decode`` keeps the reference's signature and out-parameters
(quartz/kernels/fused.py:27-65): out[H] = down(silu(gate.x) * (up.x)) with
gate|up stacked as gu_q [2I, H]. On the GPU it is one cooperative kernel:
gate/up GEMV pair + SiLU gate into abuf, a grid-wide barrier, then the down
GEMV -- the down weights stream into shared memory while phase 1 finishes.
"""

from __future__ import annotations

import numpy as np

from .. import _host
from .. import device as _dev
from .int8 import _check_np, _check_out, _is_torch


def fused_mlp_decode(gu_q, gu_s, x, down_q, down_s, abuf, out) -> None:
    """The MLP body of one token on the GPU: for each intermediate unit n,
    abuf[n] = silu(g_n . x) * (u_n . x), where g_n and u_n are rows n and
    I + n of the stacked int8 matrix gu_q [2I, H] (scales gu_s [2I, ng]);
    then out[h] = sum_n down_q[h, n] * abuf[n], scaled by down_s [H, ng_d].
    x [H] is the already-normalised activation. Both abuf [I] and out [H] are
    written in place, as in the reference's signature."""
    if _is_torch(gu_q, gu_s, x, down_q, down_s, abuf, out):
        _dev.fused_mlp(gu_q, gu_s, x.reshape(-1), down_q, down_s, abuf, out)
        return
    _check_np(gu_q, gu_s)
    _check_np(down_q, down_s)
    I2, H = gu_q.shape
    I = I2 // 2
    if I2 != 2 * I or down_q.shape != (H, I):
        raise ValueError(f"shape mismatch: gu_q {gu_q.shape}, down_q {down_q.shape}")
    if x.shape != (H,):
        raise ValueError(f"x must have shape ({H},), got {x.shape}")
    _check_out(abuf, (I,), "abuf")
    _check_out(out, (H,), "out")
    d = _dev.ensure_device()
    gq, gs = _host.resident(gu_q, d), _host.resident(gu_s, d)
    dq, ds = _host.resident(down_q, d), _host.resident(down_s, d)
    xd = _host.to_device(x, "x", d)
    ad = _host.out_buffer((I,), "abuf", d)
    od = _host.out_buffer((H,), "y", d)
    _dev.fused_mlp(gq, gs, xd, dq, ds, ad, od)
    _host.to_host(ad, abuf, "abuf")
    _host.to_host(od, out, "y")


def warmup_fused() -> None:
    """Run the fused kernel once on tiny inputs (quartz/kernels/fused.py:68-76)."""
    ii, h = 4, 2
    gu = np.ones((2 * ii, h), np.int8)
    gs = np.ones((2 * ii, 1), np.float32)
    dq = np.ones((h, ii), np.int8)
    ds = np.ones((h, 1), np.float32)
    fused_mlp_decode(gu, gs, np.ones(h, np.float32), dq, ds,
                     np.empty(ii, np.float32), np.empty(h, np.float32))
    ii, h = 64, 32
    fused_mlp_decode(np.ones((2 * ii, h), np.int8), np.ones((2 * ii, 1), np.float32),
                     np.ones(h, np.float32), np.ones((h, ii), np.int8),
                     np.ones((h, 1), np.float32), np.empty(ii, np.float32),
                     np.empty(h, np.float32))
