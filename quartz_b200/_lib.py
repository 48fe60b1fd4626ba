"""ctypes binding of libquartz_b200.so (the C ABI in include/quartz_b200.h).

Loading fails loudly: there is no CPU fallback behind this package. A missing
library, a host without CUDA, or a GPU that is not sm_100 raises.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libquartz_b200.so"

QZ_OK = 0
QZ_ERR_INVALID = 1
QZ_ERR_CUDA = 2
QZ_ERR_UNSUPPORTED = 3

# Every symbol include/quartz_b200.h declares, with its ctypes signature.
# activation prologues of qz_gemm_w8_act_ws (include/quartz_b200.h)
QZ_ACT_NONE, QZ_ACT_RMSNORM, QZ_ACT_SILU_MUL = 0, 1, 2
_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int
SIGNATURES = {
    "qz_version": ([], _int),
    "qz_init": ([_int], _int),
    "qz_last_error": ([ctypes.c_char_p, ctypes.c_size_t], _int),
    "qz_gemv_w8": ([_vp, _vp, _i64, _vp, _vp, _i64, _i64, _vp, _vp], _int),
    "qz_gemv_w4": ([_vp, _vp, _i64, _vp, _vp, _i64, _i64, _vp, _vp], _int),
    "qz_gemv_w8_host": ([_vp, _vp, _i64, _vp, _vp, _i64, _i64, _vp, _vp, _vp, _vp, _vp], _int),
    "qz_gemm_w8": ([_vp, _vp, _i64, _vp, _vp, _i64, _i64, _i64, _vp, _vp], _int),
    "qz_fused_mlp_decode": ([_vp, _vp, _i64, _vp, _vp, _vp, _i64, _vp, _vp, _vp, _i64, _i64,
                             _vp, _vp], _int),
    "qz_gemm_w8_workspace_bytes": ([_i64, _i64, _i64, ctypes.POINTER(_i64)], _int),
    "qz_gemm_w8_ws": ([_vp, _vp, _i64, _vp, _vp, _i64, _i64, _i64, _vp, _vp, ctypes.c_size_t, _vp],
                      _int),
    "qz_gemm_w8_act_ws": ([_vp, _vp, _i64, _vp, _int, _vp, ctypes.c_float, _vp, _i64, _i64, _i64,
                           _vp, _vp, ctypes.c_size_t, _vp], _int),
    "qz_mlp_workspace_bytes": ([], _int),
    "qz_fused_mlp_decode_noalloc": ([_vp, _vp, _i64, _vp, _vp, _vp, _i64, _vp, _vp, _i64, _i64,
                                     _vp], _int),
    "qz_silu_mul": ([_vp, _vp, _i64, _i64, _vp], _int),
    "qz_gemv_w8_rmsnorm": ([_vp, _vp, _i64, _vp, _vp, ctypes.c_float, _vp, _i64, _i64, _vp, _vp,
                            _vp], _int),
    "qz_fused_mlp_decode_rmsnorm": ([_vp, _vp, _i64, _vp, _vp, ctypes.c_float, _vp, _vp, _i64,
                                     _vp, _vp, _vp, _i64, _i64, _vp, _vp, _vp], _int),
    "qz_embed_gather": ([_vp, _vp, _i64, _vp, _i64, _i64, _i64, _vp, _vp], _int),
    "qz_rmsnorm": ([_vp, _vp, _vp, _i64, _i64, ctypes.c_float, _vp], _int),
    "qz_qk_rope": ([_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _int, _int, _int, _i64, _i64, _vp,
                    ctypes.c_float, _vp], _int),
    "qz_attention_decode_workspace_bytes": ([_int, _int, _int, _i64, ctypes.POINTER(_i64)], _int),
    "qz_attention_decode_qkv": ([_vp, _vp, _vp, _vp, _vp, _vp, _vp, _int, _int, _int, _i64, _i64,
                                 _vp, ctypes.c_float, ctypes.c_float, _vp, ctypes.c_size_t, _vp],
                                _int),
    "qz_attention_decode_batch_workspace_bytes": ([_int, _int, _int, _int, _i64,
                                                   ctypes.POINTER(_i64)], _int),
    "qz_attention_decode_qkv_batch": ([_vp, _i64, _vp, _vp, _vp, _vp, _vp, _i64, _vp, _i64, _int,
                                       _int, _int, _int, _i64, _i64, _vp, ctypes.c_float,
                                       ctypes.c_float, _vp, ctypes.c_size_t, _vp], _int),
    "qz_attention_decode": ([_vp, _vp, _vp, _vp, _int, _int, _int, _i64, _i64, _vp, _i64,
                             ctypes.c_float, _vp, ctypes.c_size_t, _vp], _int),
    "qz_attention_prefill": ([_vp, _vp, _vp, _vp, _i64, _int, _int, _int, _i64, _i64,
                              ctypes.c_float, _vp], _int),
    "qz_argmax": ([_vp, _i64, _i64, _vp, _vp, _vp, _i64, _vp], _int),
    "qz_decode_step_workspace_bytes": ([_int, _int, _int, _int, _int, _i64, ctypes.POINTER(_i64)],
                                       _int),
    "qz_decode_layers_supported": ([_int, _int, _int, _int, _int, _i64], _int),
    "qz_comm_buffer_bytes": ([_int, _i64, ctypes.POINTER(_i64)], _int),
    "qz_comm_alloc": ([_i64, ctypes.POINTER(_vp)], _int),
    "qz_comm_free": ([_vp], _int),
    "qz_ipc_handle": ([_vp, _vp], _int),
    "qz_ipc_open": ([_vp, ctypes.POINTER(_vp)], _int),
    "qz_ipc_close": ([_vp], _int),
    "qz_allreduce_sum": ([_vp, _vp, _i64, _i64, _vp, _int, _int, _vp], _int),
    "qz_gemv_w8_peer": ([_vp, _vp, _i64, _vp, _i64, _i64, _vp, _vp, _vp], _int),
    "qz_fused_mlp_decode_peer": ([_vp, _vp, _i64, _vp, _vp, _vp, _i64, _vp, _vp, _i64, _i64,
                                  _vp, _vp, _vp], _int),
    "qz_rmsnorm_peer_sum": ([_vp, _i64, _vp, ctypes.c_float, _vp, _vp, _vp], _int),
    "qz_decode_layers": ([_vp, _int, _vp, _vp, _i64, _vp, _vp, _vp, _vp, _vp, _int, _int, _int,
                          _int, _int, _i64, ctypes.c_float, ctypes.c_float, _vp, ctypes.c_size_t,
                          _vp, _vp], _int),
    "qz_device_status": ([ctypes.POINTER(ctypes.c_uint32), _int], _int),
    "qz_sync": ([_vp], _int),
}

_lib = None
_lock = threading.Lock()


class QuartzError(RuntimeError):
    """A CUDA-side failure reported through the C ABI."""


def load():
    """Load the library (no CUDA context is created by loading)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise ImportError(
                    f"{LIB_PATH} is missing: build it with `python -m quartz_b200.build`")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (args, res) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.argtypes = args
                fn.restype = res
            _lib = lib
    return _lib


def last_error() -> str:
    lib = load()
    n = lib.qz_last_error(None, 0)
    buf = ctypes.create_string_buffer(n + 1)
    lib.qz_last_error(buf, n + 1)
    return buf.value.decode(errors="replace")


def check(rc: int) -> None:
    if rc == QZ_OK:
        return
    msg = last_error()
    if rc == QZ_ERR_INVALID:
        raise ValueError(msg)
    raise QuartzError(msg)


def device_status(clear: bool = False) -> tuple[int, int, int, int]:
    words = (ctypes.c_uint32 * 4)()
    check(load().qz_device_status(words, 1 if clear else 0))
    return tuple(int(w) for w in words)
