"""Device-level entry points over torch CUDA tensors (no host copies).

Each function validates its tensors, then calls the C ABI on the current torch
stream. Outputs may be passed in (written in place, like the reference's
out-parameters) or are allocated here. torch is used only for device memory
and streams.

    gemv(q, scale, x)            -> y        quartz/kernels/int8.py:24-38
    gemm(q, scale, X)            -> Y        quartz/kernels/int8.py:66-87
    fused_mlp(gu_q, gu_s, x, down_q, down_s)  -> out   quartz/kernels/fused.py:27-65
    silu_mul(gu)                 -> a        quartz/quantize.py:112-114 (+ ops.py:35-37)

Decode-step glue (the fp32 work between the int8 matmuls of one token):

    embed_gather(q, scale, ids)  -> rows     quartz/quantize.py:78-80
    rmsnorm(x, w, eps)           -> y        quartz/ops.py:24-32
    qk_rope(qkv, ...)            -> q        quartz/models/qwen3.py:31-41, rope.py:47-78
    attention_decode(q, kc, vc, T)           quartz/attention.py:29-43 (one query row)
    attention_decode_qkv(qkv, ...)           the two above plus the KV append, one launch
    attention_prefill(q, kc, vc, pos0)       quartz/attention.py:15-43 (causal rows)
    argmax(logits)               -> tokens   quartz/sample.py:21-22
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
    if dev is None and _ready_devices:
        idx = torch.cuda.current_device()   # the per-call path: no availability probe
        if idx in _ready_devices:
            return idx
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


def gemv(q, scale, x, y=None, residual=None, norm_w=None, eps=1e-6):
    """y[n] = sum_g scale[n,g] sum_{j<G} x[gG+j] q[n,gG+j] (+ residual[n]).
    With norm_w, the GEMV of RMSNorm(x) * norm_w (normalised in the kernel)."""
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
    _same_device(q.device, scale, x, y, residual, norm_w)
    with torch.cuda.device(q.device):
        if norm_w is not None:
            _need(norm_w, torch.float32, "norm_w", 1)
            if norm_w.numel() != K:
                raise ValueError("norm_w must have K elements")
            scratch = torch.empty(K, dtype=torch.float32, device=q.device)
            _lib.check(_lib.load().qz_gemv_w8_rmsnorm(
                q.data_ptr(), scale.data_ptr(), ng, x.data_ptr(), norm_w.data_ptr(), float(eps),
                y.data_ptr(), N, K, _ptr(residual), scratch.data_ptr(), _stream_ptr(q.device)))
            return y
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


def gemv_w4(q4, scale, x, y=None, residual=None):
    """int4 weights: y[n] = sum_g scale[n,g] sum_{j<G} x[gG+j] q[n,gG+j]
    (+ residual[n]), q4 uint8 [N, K/2] packed two weights per byte
    (quartz_b200.quantize.pack_int4)."""
    if not isinstance(q4, torch.Tensor) or q4.dtype != torch.uint8 or q4.dim() != 2:
        raise TypeError("q4 must be a 2-D uint8 CUDA tensor")
    if not q4.is_cuda or not q4.is_contiguous():
        raise ValueError("q4 must be a contiguous CUDA tensor")
    N, K = q4.shape[0], 2 * q4.shape[1]
    _need(scale, torch.float32, "scale", 2)
    if scale.shape[0] != N:
        raise ValueError("scale and q4 disagree on the number of rows")
    ng = scale.shape[1]
    ensure_device(q4.device)
    _need(x, torch.float32, "x")
    if x.numel() != K:
        raise ValueError(f"x has {x.numel()} elements, expected K={K}")
    if y is None:
        y = torch.empty(N, dtype=torch.float32, device=q4.device)
    _need(y, torch.float32, "y")
    if y.numel() != N:
        raise ValueError(f"y has {y.numel()} elements, expected N={N}")
    if residual is not None:
        _need(residual, torch.float32, "residual")
    _same_device(q4.device, scale, x, y, residual)
    with torch.cuda.device(q4.device):
        _lib.check(_lib.load().qz_gemv_w4(q4.data_ptr(), scale.data_ptr(), ng, x.data_ptr(),
                                          y.data_ptr(), N, K, _ptr(residual),
                                          _stream_ptr(q4.device)))
    return y


def fused_mlp(gu_q, gu_s, x, down_q, down_s, abuf=None, out=None, residual=None, norm_w=None,
              eps=1e-6):
    """out = down(silu(gate.x) * (up.x)) (+ residual) for one token (M = 1).
    With norm_w, of RMSNorm(x) * norm_w (normalised in the kernel)."""
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
    if norm_w is not None:
        _need(norm_w, torch.float32, "norm_w", 1)
        if norm_w.numel() != H:
            raise ValueError("norm_w must have H elements")
        scratch = torch.empty(H, dtype=torch.float32, device=dev)
        with torch.cuda.device(dev):
            _lib.check(_lib.load().qz_fused_mlp_decode_rmsnorm(
                gu_q.data_ptr(), gu_s.data_ptr(), ng, x.data_ptr(), norm_w.data_ptr(), float(eps),
                down_q.data_ptr(), down_s.data_ptr(), ngd, abuf.data_ptr(), out.data_ptr(),
                _ptr(residual), H, I, ws.data_ptr(), scratch.data_ptr(), _stream_ptr(dev)))
        return out
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


# ---------------------------------------------------------------------------
# decode-step glue
# ---------------------------------------------------------------------------

_attn_ws: dict[int, torch.Tensor] = {}
_argmax_keys: dict[int, torch.Tensor] = {}


def embed_gather(q, scale, ids, out=None):
    """out[m, :] = q[ids[m], :] * scale[ids[m], group] (int64 ids on the device)."""
    V, H, ng = _weights(q, scale)
    ensure_device(q.device)
    _need(ids, torch.int64, "ids")
    M = ids.numel()
    if out is None:
        out = torch.empty((M, H), dtype=torch.float32, device=q.device)
    _need(out, torch.float32, "out")
    if out.numel() != M * H:
        raise ValueError(f"out must hold M*H = {M * H} elements")
    _same_device(q.device, scale, ids, out)
    with torch.cuda.device(q.device):
        _lib.check(_lib.load().qz_embed_gather(q.data_ptr(), scale.data_ptr(), ng, ids.data_ptr(),
                                               M, V, H, out.data_ptr(), _stream_ptr(q.device)))
    return out


def rmsnorm(x, w, eps=1e-6, out=None):
    """Row-wise x / sqrt(mean(x^2) + eps) * w over the last dimension."""
    _need(x, torch.float32, "x")
    _need(w, torch.float32, "w", 1)
    ensure_device(x.device)
    n = x.shape[-1]
    if w.numel() != n:
        raise ValueError(f"w has {w.numel()} elements, rows have {n}")
    rows = x.numel() // n if n else 0
    if out is None:
        out = torch.empty_like(x)
    _need(out, torch.float32, "out")
    if out.numel() != x.numel():
        raise ValueError("out must match x")
    _same_device(x.device, w, out)
    with torch.cuda.device(x.device):
        _lib.check(_lib.load().qz_rmsnorm(x.data_ptr(), w.data_ptr(), out.data_ptr(), rows, n,
                                          float(eps), _stream_ptr(x.device)))
    return out


def _cache_dims(kc, vc):
    _need(kc, torch.float32, "k_cache", 3)
    _need(vc, torch.float32, "v_cache", 3)
    if kc.shape != vc.shape:
        raise ValueError("k_cache and v_cache must have the same shape")
    return kc.shape   # (n_kv, max_ctx, head_dim)


def qk_rope(qkv, inv_freq, k_cache, v_cache, n_heads, pos0=0, pos_dev=None, q_norm=None,
            k_norm=None, eps=1e-6, q_out=None):
    """Split qkv [M, (nq + 2 nkv) hd] into q (normed, rotated; returned as [M, nq hd]) and the
    cache rows at positions pos0 + m (or *pos_dev + m)."""
    nkv, max_ctx, hd = _cache_dims(k_cache, v_cache)
    _need(qkv, torch.float32, "qkv")
    _need(inv_freq, torch.float32, "inv_freq", 1)
    ensure_device(qkv.device)
    width = (n_heads + 2 * nkv) * hd
    if qkv.shape[-1] != width:
        raise ValueError(f"qkv rows must have {width} elements")
    if inv_freq.numel() != hd // 2:
        raise ValueError("inv_freq must have head_dim / 2 elements")
    M = qkv.numel() // width
    for t, name in ((q_norm, "q_norm"), (k_norm, "k_norm")):
        if t is not None:
            _need(t, torch.float32, name, 1)
            if t.numel() != hd:
                raise ValueError(f"{name} must have head_dim elements")
    if (q_norm is None) != (k_norm is None):
        raise ValueError("pass both q_norm and k_norm or neither")
    if pos_dev is not None:
        _need(pos_dev, torch.int64, "pos_dev")
    if q_out is None:
        q_out = torch.empty((M, n_heads * hd), dtype=torch.float32, device=qkv.device)
    _need(q_out, torch.float32, "q_out")
    if q_out.numel() != M * n_heads * hd:
        raise ValueError("q_out must hold M * n_heads * head_dim elements")
    _same_device(qkv.device, inv_freq, k_cache, v_cache, q_norm, k_norm, pos_dev, q_out)
    with torch.cuda.device(qkv.device):
        _lib.check(_lib.load().qz_qk_rope(
            qkv.data_ptr(), _ptr(q_norm), _ptr(k_norm), inv_freq.data_ptr(), q_out.data_ptr(),
            k_cache.data_ptr(), v_cache.data_ptr(), M, n_heads, nkv, hd, max_ctx, int(pos0),
            _ptr(pos_dev), float(eps), _stream_ptr(qkv.device)))
    return q_out


def attention_workspace(device, n_heads: int, n_kv: int, head_dim: int, max_ctx: int
                        ) -> torch.Tensor:
    """Grow-only per-device workspace of the decode attention (zeroed when made;
    the kernels leave it zeroed where it must be)."""
    import ctypes
    idx = ensure_device(device)
    need = ctypes.c_int64(0)
    with torch.cuda.device(idx):
        _lib.check(_lib.load().qz_attention_decode_workspace_bytes(n_heads, n_kv, head_dim,
                                                                   max_ctx, ctypes.byref(need)))
    ws = _attn_ws.get(idx)
    if ws is None or ws.numel() < need.value:
        ws = torch.zeros(need.value, dtype=torch.uint8, device=torch.device("cuda", idx))
        _attn_ws[idx] = ws
    return ws


def attention_decode(q, k_cache, v_cache, T=None, T_dev=None, t_offset=0, scale=None, out=None,
                     workspace=None):
    """softmax(q K^T * scale) V for one query row per head over cache positions [0, T)
    (T = *T_dev + t_offset when T_dev is given). q: [n_heads * head_dim]."""
    nkv, max_ctx, hd = _cache_dims(k_cache, v_cache)
    _need(q, torch.float32, "q")
    ensure_device(q.device)
    if q.numel() % hd:
        raise ValueError("q must hold n_heads * head_dim elements")
    nq = q.numel() // hd
    if (T is None) == (T_dev is None):
        raise ValueError("pass exactly one of T and T_dev")
    if T_dev is not None:
        _need(T_dev, torch.int64, "T_dev")
    scale = hd ** -0.5 if scale is None else scale
    if out is None:
        out = torch.empty(nq * hd, dtype=torch.float32, device=q.device)
    _need(out, torch.float32, "out")
    if out.numel() != nq * hd:
        raise ValueError("out must hold n_heads * head_dim elements")
    ws = workspace if workspace is not None else attention_workspace(q.device, nq, nkv, hd,
                                                                      max_ctx)
    _same_device(q.device, k_cache, v_cache, T_dev, out, ws)
    with torch.cuda.device(q.device):
        _lib.check(_lib.load().qz_attention_decode(
            q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), out.data_ptr(), nq, nkv, hd,
            max_ctx, 0 if T is None else int(T), _ptr(T_dev), int(t_offset), float(scale),
            ws.data_ptr(), ws.numel(), _stream_ptr(q.device)))
    return out


def attention_decode_qkv(qkv, inv_freq, k_cache, v_cache, n_heads, pos0=0, pos_dev=None,
                         q_norm=None, k_norm=None, eps=1e-6, scale=None, out=None,
                         workspace=None):
    """The attention block of one decode token from its projection row qkv
    [(nq + 2 nkv) hd]: q/k norm (Qwen3), RoPE, k/v append at position pos0
    (or *pos_dev), attention over positions [0, pos]. Returns [nq * hd]."""
    nkv, max_ctx, hd = _cache_dims(k_cache, v_cache)
    _need(qkv, torch.float32, "qkv")
    _need(inv_freq, torch.float32, "inv_freq", 1)
    ensure_device(qkv.device)
    if qkv.numel() != (n_heads + 2 * nkv) * hd:
        raise ValueError(f"qkv must hold (n_heads + 2 n_kv) * head_dim elements")
    if inv_freq.numel() != hd // 2:
        raise ValueError("inv_freq must have head_dim / 2 elements")
    if (q_norm is None) != (k_norm is None):
        raise ValueError("pass both q_norm and k_norm or neither")
    for t, name in ((q_norm, "q_norm"), (k_norm, "k_norm")):
        if t is not None:
            _need(t, torch.float32, name, 1)
            if t.numel() != hd:
                raise ValueError(f"{name} must have head_dim elements")
    if pos_dev is not None:
        _need(pos_dev, torch.int64, "pos_dev")
    scale = hd ** -0.5 if scale is None else scale
    if out is None:
        out = torch.empty(n_heads * hd, dtype=torch.float32, device=qkv.device)
    _need(out, torch.float32, "out")
    if out.numel() != n_heads * hd:
        raise ValueError("out must hold n_heads * head_dim elements")
    ws = workspace if workspace is not None else attention_workspace(qkv.device, n_heads, nkv, hd,
                                                                      max_ctx)
    _same_device(qkv.device, inv_freq, k_cache, v_cache, q_norm, k_norm, pos_dev, out, ws)
    with torch.cuda.device(qkv.device):
        _lib.check(_lib.load().qz_attention_decode_qkv(
            qkv.data_ptr(), _ptr(q_norm), _ptr(k_norm), inv_freq.data_ptr(), k_cache.data_ptr(),
            v_cache.data_ptr(), out.data_ptr(), n_heads, nkv, hd, max_ctx, int(pos0),
            _ptr(pos_dev), float(eps), float(scale), ws.data_ptr(), ws.numel(),
            _stream_ptr(qkv.device)))
    return out


def attention_prefill(q, k_cache, v_cache, pos0, scale=None, out=None):
    """Causal attention of query rows q [M, n_heads * head_dim] at positions pos0 + m."""
    nkv, max_ctx, hd = _cache_dims(k_cache, v_cache)
    _need(q, torch.float32, "q", 2)
    ensure_device(q.device)
    M, width = q.shape
    if width % hd:
        raise ValueError("q rows must hold n_heads * head_dim elements")
    nq = width // hd
    scale = hd ** -0.5 if scale is None else scale
    if out is None:
        out = torch.empty_like(q)
    _need(out, torch.float32, "out")
    if out.numel() != q.numel():
        raise ValueError("out must match q")
    _same_device(q.device, k_cache, v_cache, out)
    with torch.cuda.device(q.device):
        _lib.check(_lib.load().qz_attention_prefill(
            q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), out.data_ptr(), M, nq, nkv, hd,
            max_ctx, int(pos0), float(scale), _stream_ptr(q.device)))
    return out


def argmax_keys(device, M: int) -> torch.Tensor:
    """Per-device zeroed uint64 scratch for argmax (kept zero between calls)."""
    idx = ensure_device(device)
    keys = _argmax_keys.get(idx)
    if keys is None or keys.numel() < M:
        keys = torch.zeros(max(M, 64), dtype=torch.int64, device=torch.device("cuda", idx))
        _argmax_keys[idx] = keys
    return keys


def argmax(logits, tokens=None, pos_dev=None, pos_step=0, keys=None):
    """Greedy token per row of logits [M, V] (first index of the maximum)."""
    _need(logits, torch.float32, "logits")
    ensure_device(logits.device)
    V = logits.shape[-1]
    M = logits.numel() // V
    if tokens is None:
        tokens = torch.empty(M, dtype=torch.int64, device=logits.device)
    _need(tokens, torch.int64, "tokens")
    if tokens.numel() != M:
        raise ValueError("tokens must have one element per row")
    if pos_dev is not None:
        _need(pos_dev, torch.int64, "pos_dev")
    keys = keys if keys is not None else argmax_keys(logits.device, M)
    _same_device(logits.device, tokens, pos_dev, keys)
    with torch.cuda.device(logits.device):
        _lib.check(_lib.load().qz_argmax(logits.data_ptr(), M, V, keys.data_ptr(),
                                         tokens.data_ptr(), _ptr(pos_dev), int(pos_step),
                                         _stream_ptr(logits.device)))
    return tokens
