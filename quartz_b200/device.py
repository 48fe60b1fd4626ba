"""Device-level entry points over torch CUDA tensors (no host copies).

Each function validates its tensors, then calls the C ABI on the current torch
stream. Outputs may be passed in (written in place, like the reference's
out-parameters) or are allocated here. torch is used only for device memory
and streams.

    gemv(q, scale, x)            -> y        quartz/kernels/int8.py:24-38
    gemm(q, scale, X)            -> Y        quartz/kernels/int8.py:66-87
    fused_mlp(gu_q, gu_s, x, down_q, down_s)  -> out   quartz/kernels/fused.py:27-65
    silu_mul(gu)                 -> a        quartz/quantize.py:112-114 (+ ops.py:35-37)
"""

from __future__ import annotations

import threading

import torch

from . import _lib

_init_lock = threading.Lock()
_ready_devices: set[int] = set()
_mlp_ws: dict[int, torch.Tensor] = {}
_gemm_ws: dict[int, torch.Tensor] = {}


def _stream_ptr(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def ensure_device(dev: torch.device | int | None = None) -> int:
    """qz_init once per device (checks that it is an sm_100 GPU)."""
    if not torch.cuda.is_available():
        raise RuntimeError("quartz_b200 needs a CUDA device; none is available")
    if dev is None:
        idx = torch.cuda.current_device()
    elif isinstance(dev, int):
        idx = dev
    else:
        idx = dev.index if dev.index is not None else torch.cuda.current_device()
    if idx not in _ready_devices:
        with _init_lock:
            if idx not in _ready_devices:
                with torch.cuda.device(idx):
                    _lib.check(_lib.load().qz_init(idx))
                _ready_devices.add(idx)
    return idx


def _same_device(dev: torch.device, *ts) -> None:
    for t in ts:
        if t is not None and t.device != dev:
            raise ValueError(f"all tensors must be on {dev}, found one on {t.device}")


def _need(t: torch.Tensor, dtype, name: str, ndim: int | None = None) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")
    if ndim is not None and t.dim() != ndim:
        raise ValueError(f"{name} must be {ndim}-D, got shape {tuple(t.shape)}")


def _weights(q, scale, name="q"):
    _need(q, torch.int8, name, 2)
    _need(scale, torch.float32, name + " scale", 2)
    N, K = q.shape
    if scale.shape[0] != N:
        raise ValueError(f"{name}: scale has {scale.shape[0]} rows, weights have {N}")
    ng = scale.shape[1]
    if ng < 1 or K % ng:
        raise ValueError(f"scale has {ng} groups that do not tile K={K}")
    return N, K, ng


def _ptr(t):
    return None if t is None else t.data_ptr()


def gemv(q, scale, x, y=None, residual=None):
    """y[n] = sum_g scale[n,g] sum_{j<G} x[gG+j] q[n,gG+j] (+ residual[n])."""
    N, K, ng = _weights(q, scale)
    ensure_device(q.device)
    _need(x, torch.float32, "x")
    if x.numel() != K:
        raise ValueError(f"x has {x.numel()} elements, expected K={K}")
    if y is None:
        y = torch.empty(N, dtype=torch.float32, device=q.device)
    _need(y, torch.float32, "y")
    if y.numel() != N:
        raise ValueError(f"y has {y.numel()} elements, expected N={N}")
    if residual is not None:
        _need(residual, torch.float32, "residual")
        if residual.numel() != N:
            raise ValueError("residual must have N elements")
    _same_device(q.device, scale, x, y, residual)
    with torch.cuda.device(q.device):
        _lib.check(_lib.load().qz_gemv_w8(q.data_ptr(), scale.data_ptr(), ng, x.data_ptr(),
                                          y.data_ptr(), N, K, _ptr(residual),
                                          _stream_ptr(q.device)))
    return y


def gemm(q, scale, X, Y=None, residual=None):
    """Y[m, n] for each row m of X [M, K] (+ residual[m, n])."""
    N, K, ng = _weights(q, scale)
    ensure_device(q.device)
    _need(X, torch.float32, "X")
    if X.dim() != 2 or X.shape[1] != K:
        raise ValueError(f"X must be [M, {K}], got {tuple(X.shape)}")
    M = X.shape[0]
    if Y is None:
        Y = torch.empty((M, N), dtype=torch.float32, device=q.device)
    _need(Y, torch.float32, "Y")
    if Y.numel() != M * N:
        raise ValueError(f"Y must hold M*N = {M * N} elements")
    if residual is not None:
        _need(residual, torch.float32, "residual")
        if residual.numel() != M * N:
            raise ValueError("residual must have M*N elements")
    _same_device(q.device, scale, X, Y, residual)
    ws = gemm_workspace(q.device, M, N, K)
    with torch.cuda.device(q.device):
        _lib.check(_lib.load().qz_gemm_w8_ws(q.data_ptr(), scale.data_ptr(), ng, X.data_ptr(),
                                             Y.data_ptr(), M, N, K, _ptr(residual),
                                             _ptr(ws), 0 if ws is None else ws.numel(),
                                             _stream_ptr(q.device)))
    return Y


def gemm_workspace(device, M: int, N: int, K: int):
    """Grow-only per-device workspace for the tensor-core GEMM (None when M < 2).

    The GEMM's activation split is stream-ordered on the current stream; two
    streams must not share this buffer concurrently.
    """
    import ctypes
    idx = ensure_device(device)
    need = ctypes.c_int64(0)
    _lib.check(_lib.load().qz_gemm_w8_workspace_bytes(M, N, K, ctypes.byref(need)))
    if need.value == 0:
        return None
    ws = _gemm_ws.get(idx)
    if ws is None or ws.numel() < need.value:
        ws = torch.empty(max(need.value, 1 << 20), dtype=torch.uint8,
                         device=torch.device("cuda", idx))
        _gemm_ws[idx] = ws
    return ws


def mlp_workspace(device) -> torch.Tensor:
    """Per-device grid-barrier words for the fused MLP (zeroed once)."""
    idx = ensure_device(device)
    ws = _mlp_ws.get(idx)
    if ws is None:
        nbytes = _lib.load().qz_mlp_workspace_bytes()
        ws = torch.zeros(nbytes // 4, dtype=torch.int32, device=torch.device("cuda", idx))
        _mlp_ws[idx] = ws
    return ws


def fused_mlp(gu_q, gu_s, x, down_q, down_s, abuf=None, out=None, residual=None):
    """out = down(silu(gate.x) * (up.x)) (+ residual) for one token (M = 1)."""
    I2, H = gu_q.shape
    _, _, ng = _weights(gu_q, gu_s, "gu_q")
    Hd, I, ngd = _weights(down_q, down_s, "down_q")
    if I2 != 2 * I or Hd != H:
        raise ValueError(f"shape mismatch: gu_q {tuple(gu_q.shape)}, down_q {tuple(down_q.shape)}")
    dev = gu_q.device
    _need(x, torch.float32, "x")
    if x.numel() != H:
        raise ValueError(f"x has {x.numel()} elements, expected H={H}")
    if abuf is None:
        abuf = torch.empty(I, dtype=torch.float32, device=dev)
    if out is None:
        out = torch.empty(H, dtype=torch.float32, device=dev)
    _need(abuf, torch.float32, "abuf")
    _need(out, torch.float32, "out")
    if abuf.numel() != I or out.numel() != H:
        raise ValueError("abuf must have I elements and out H elements")
    if residual is not None:
        _need(residual, torch.float32, "residual")
        if residual.numel() != H:
            raise ValueError("residual must have H elements")
    _same_device(dev, gu_s, x, down_q, down_s, abuf, out, residual)
    ws = mlp_workspace(dev)
    with torch.cuda.device(dev):
        _lib.check(_lib.load().qz_fused_mlp_decode(
            gu_q.data_ptr(), gu_s.data_ptr(), ng, x.data_ptr(), down_q.data_ptr(),
            down_s.data_ptr(), ngd, abuf.data_ptr(), out.data_ptr(), _ptr(residual), H, I,
            ws.data_ptr(), _stream_ptr(dev)))
    return out


def silu_mul(gu, a=None):
    """a[m, i] = silu_clipped(gu[m, i]) * gu[m, I + i] for gu [M, 2I]."""
    _need(gu, torch.float32, "gu")
    ensure_device(gu.device)
    M = gu.numel() // gu.shape[-1]
    I2 = gu.shape[-1]
    if I2 % 2:
        raise ValueError("gu's last dimension must be even")
    I = I2 // 2
    if a is None:
        a = torch.empty((*gu.shape[:-1], I), dtype=torch.float32, device=gu.device)
    _need(a, torch.float32, "a")
    if a.numel() != M * I:
        raise ValueError(f"a must hold M*I = {M * I} elements")
    _same_device(gu.device, a)
    with torch.cuda.device(gu.device):
        _lib.check(_lib.load().qz_silu_mul(gu.data_ptr(), a.data_ptr(), M, I,
                                           _stream_ptr(gu.device)))
    return a


def status(clear: bool = False, device=None):
    """Device status word {error bits, first site, its block, count} (synchronises)."""
    idx = ensure_device(device)
    with torch.cuda.device(idx):
        return _lib.device_status(clear)


def check_status(device=None) -> None:
    """Raise if any kernel on the device reported a failed wait; clears the word."""
    bits, site, block, count = status(clear=True, device=device)
    if bits:
        raise _lib.QuartzError(
            f"device kernels reported {count} failed wait(s): bits=0x{bits:x} "
            f"first site=0x{site:x} block={block}")
