"""CPU oracle for the int8 weight-only path (test infrastructure only).

Imported by tests/, by ``__graft_entry__.smoke()`` as the checker, and by
bench.py's CPU-baseline leg. The shipped package never imports it.
"""

from .oracle import (  # noqa: F401
    load,
    threads,
    set_threads,
    w8a32_gemv,
    w4a32_gemv,
    w8a32_gemv_serial,
    w8a32_gemm,
    matmul_int8,
    fused_mlp_decode,
    mlp_per_op,
    silu_clipped,
)
