"""Load-time symmetric int8 (and int4) quantisers (host, numpy) and the dequantising row gather.

These produce the operands of the int8 weight-only path; they run once at model
load, never on the decode hot path, so they stay numpy on the host.

Format (identical to quartz/quantize.py:26-48 so that the same fp32 weights give
the same int8 bytes on both sides): ``w ~= q * scale`` with q int8 in [-127, 127]
and one fp32 scale per group of ``G = K // ng`` consecutive input-dim elements
(``group_size=None`` is one scale per output row). A group whose absmax is zero
gets scale 1.0. Rounding is numpy's round-half-to-even.
"""

from __future__ import annotations

import numpy as np


def quantize_symmetric(W: np.ndarray, group_size: int | None = None):
    """(N, K) fp32 -> (q int8 (N, K) C-contiguous, scale fp32 (N, ng)).

    Follows quartz/quantize.py:26-38: the scale is computed in float64 from the
    fp32 absmax then cast to fp32; q = clip(round(W / scale), -127, 127), where
    the division is fp32 / fp32 (numpy promotes nothing here).
    """
    W = np.ascontiguousarray(W, dtype=np.float32)
    N, K = W.shape
    G = group_size or K
    if K % G != 0:
        raise ValueError(f"group_size {G} does not divide input dim {K}")
    if W.size >= _PARALLEL_ELEMS and N >= 2 * _THREADS:
        # rows are independent: quantise row blocks on host threads (numpy
        # releases the GIL in these loops); the bytes are those of one pass
        from concurrent.futures import ThreadPoolExecutor
        b = [N * i // _THREADS for i in range(_THREADS + 1)]
        with ThreadPoolExecutor(_THREADS) as ex:
            parts = list(ex.map(lambda i: _quantize_rows(W[b[i]:b[i + 1]], G), range(_THREADS)))
        return (np.ascontiguousarray(np.concatenate([p[0] for p in parts])),
                np.ascontiguousarray(np.concatenate([p[1] for p in parts])))
    return _quantize_rows(W, G)


_PARALLEL_ELEMS = 1 << 24
_THREADS = 8


def _quantize_rows(W: np.ndarray, G: int):
    N, K = W.shape
    ng = K // G
    Wg = W.reshape(N, ng, G)
    scale = (np.abs(Wg).max(axis=2) / 127.0).astype(np.float32)
    scale[scale == 0] = 1.0
    q = np.clip(np.round(Wg / scale[:, :, None]), -127, 127).astype(np.int8).reshape(N, K)
    return np.ascontiguousarray(q), np.ascontiguousarray(scale)


def dequantize_symmetric(q: np.ndarray, scale: np.ndarray, group_size: int | None = None) -> np.ndarray:
    """fp32 (..., K) from int8 q (..., K) and scale (..., ng) (quartz/quantize.py:41-48)."""
    shp = q.shape
    K = shp[-1]
    ng = scale.shape[-1]
    G = K // ng
    qf = q.astype(np.float32).reshape(*shp[:-1], ng, G)
    return (qf * scale[..., None]).reshape(shp).astype(np.float32)


def quantize_symmetric_int4(W: np.ndarray, group_size: int | None = None):
    """(N, K) fp32 -> (q4 uint8 (N, K // 2) packed, scale fp32 (N, ng)).

    The 4-bit twin of ``quantize_symmetric`` (quartz keeps 4-bit weights as
    future work, quartz/config.py:98): scale = absmax / 7 per group (1.0 for
    an all-zero group), q = clip(round_half_even(W / scale), -7, 7), packed
    two per byte by ``pack_int4``. K must be even.
    """
    W = np.ascontiguousarray(W, dtype=np.float32)
    N, K = W.shape
    G = group_size or K
    if K % G != 0:
        raise ValueError(f"group_size {G} does not divide input dim {K}")
    if K % 2:
        raise ValueError("int4 packing needs an even input dim")
    ng = K // G
    Wg = W.reshape(N, ng, G)
    scale = (np.abs(Wg).max(axis=2) / 7.0).astype(np.float32)
    scale[scale == 0] = 1.0
    q = np.clip(np.round(Wg / scale[:, :, None]), -7, 7).astype(np.int8).reshape(N, K)
    return pack_int4(q), np.ascontiguousarray(scale)


def pack_int4(q: np.ndarray) -> np.ndarray:
    """int8 (..., K) in [-8, 7] -> uint8 (..., K // 2): element 2i in the low
    nibble of byte i, element 2i + 1 in the high nibble, two's complement."""
    q = np.asarray(q, dtype=np.int8)
    if q.shape[-1] % 2:
        raise ValueError("int4 packing needs an even last dim")
    u = q.astype(np.uint8) & 0x0F
    return np.ascontiguousarray(u[..., 0::2] | (u[..., 1::2] << 4))


def unpack_int4(q4: np.ndarray) -> np.ndarray:
    """uint8 (..., K // 2) -> int8 (..., K), the inverse of ``pack_int4``."""
    q4 = np.asarray(q4, dtype=np.uint8)
    lo = (q4 & 0x0F).astype(np.int8)
    hi = (q4 >> 4).astype(np.int8)
    lo = np.where(lo > 7, lo - 16, lo).astype(np.int8)
    hi = np.where(hi > 7, hi - 16, hi).astype(np.int8)
    out = np.empty(q4.shape[:-1] + (2 * q4.shape[-1],), np.int8)
    out[..., 0::2] = lo
    out[..., 1::2] = hi
    return out


def stack_gate_up(gate_q, gate_s, up_q, up_s):
    """Stack gate rows over up rows -> ([2I, H] int8, [2I, ng] fp32).

    The fused MLP reads intermediate unit n from rows n (gate) and n + I (up) of
    one tensor, the layout quartz/quantize.py:95-96 builds.
    """
    gu_q = np.ascontiguousarray(np.concatenate([gate_q, up_q], axis=0))
    gu_s = np.ascontiguousarray(np.concatenate([gate_s, up_s], axis=0))
    return gu_q, gu_s
