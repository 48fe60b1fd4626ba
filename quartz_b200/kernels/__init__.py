"""B200 kernel layer: the drop-in for quartz's ``quartz.kernels`` package
(quartz/kernels/__init__.py:10-12) plus its ``fused`` module."""

from __future__ import annotations

from .int8 import (w8a32_gemv, w8a32_gemv_serial, w8a32_gemm, matmul_int8, warmup,
                   PRANGE_BYTES)
from .fused import fused_mlp_decode, warmup_fused
from .int4 import w4a32_gemv

__all__ = ["w8a32_gemv", "w8a32_gemm", "matmul_int8", "warmup"]
