"""Batched GEMM (M > 1) on the tensor cores against the CPU oracle.

quartz/kernels/int8.py:66-87 (w8a32_gemm) at the prefill shapes of the
Llama-3.2-1B workload (M = 512), batched decode rows (M = 2..16) on the Qwen3
lm_head, odd sizes (partial 128-row and 128-byte tiles, token padding) and
activations with outliers. Bar: max |err| <= 1e-4 * ||Y_ref||_inf.
"""

import numpy as np
import pytest

import oracle
from tests import _golden as G

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def _oracle_gemm(q, s, X):
    Y = np.empty((X.shape[0], q.shape[0]), np.float32)
    oracle.w8a32_gemm(q, s, np.ascontiguousarray(X), Y)
    return Y


@pytest.fixture(autouse=True, scope="module")
def _status():
    from quartz_b200 import device
    device.status(clear=True)
    yield
    device.check_status()


@pytest.mark.parametrize("N,K,M", [
    (2048, 2048, 512),    # Llama-1B q/o proj, 512-token prefill
    (512, 2048, 512),     # k/v proj
    (2048, 8192, 64),     # down proj, 64 rows
    (16384, 2048, 128),   # stacked gate|up
    (1000, 1040, 37),     # ragged rows, K not a multiple of 128, token padding
    (128, 64, 5),         # K smaller than one 128-byte tile
    (300, 4096, 2),
])
def test_tensor_gemm_vs_oracle(N, K, M):
    from quartz_b200 import device
    from quartz_b200.workloads import gemv_case
    c = gemv_case(N, K, M, seed=N + K + M)
    Y = device.gemm(_t(c.q), _t(c.scale), _t(c.x)).cpu().numpy()
    G.assert_close(Y, _oracle_gemm(c.q, c.scale, c.x), what=f"{N}x{K} M={M}")


@pytest.mark.parametrize("M", [2, 4, 8, 16])
def test_lm_head_batched_decode_rows(M):
    from quartz_b200 import device
    from quartz_b200.workloads import gemv_case
    c = gemv_case(151936, 1024, M, seed=M)
    Y = device.gemm(_t(c.q), _t(c.scale), _t(c.x)).cpu().numpy()
    ref = _oracle_gemm(c.q, c.scale, c.x)
    for m in range(M):
        G.assert_close(Y[m], ref[m], what=f"lm_head row {m} of {M}")


def test_tensor_gemm_residual_and_outliers():
    from quartz_b200 import device
    from quartz_b200.workloads import gemv_case
    c = gemv_case(1536, 2048, 24, seed=11)
    X = c.x.copy()
    X[3, 17] = 1000.0          # a massive activation in one channel
    X[7, :] *= 1e-3            # a tiny row
    X[9, :] = 0.0              # an all-zero row
    R = np.random.default_rng(12).standard_normal((24, 1536)).astype(np.float32)
    Y = device.gemm(_t(c.q), _t(c.scale), _t(X), residual=_t(R)).cpu().numpy()
    ref = _oracle_gemm(c.q, c.scale, X) + R
    for m in range(24):
        G.assert_close(Y[m], ref[m], what=f"row {m}")


def test_gemm_rows_equal_gemv_rows_tensor_path():
    """tests/test_kernels.py:36-47 at a tensor-path shape: each GEMM row matches
    the GEMV of that row (atol 1e-4)."""
    from quartz_b200 import device
    from quartz_b200.workloads import gemv_case
    c = gemv_case(4096, 1024, 8, seed=21)
    q, s = _t(c.q), _t(c.scale)
    Y = device.gemm(q, s, _t(c.x)).cpu().numpy()
    for m in range(8):
        y = device.gemv(q, s, _t(c.x[m])).cpu().numpy()
        assert np.allclose(Y[m], y, atol=1e-4)


def _gemm_ws(M, N, K):
    import ctypes
    from quartz_b200 import _lib
    b = ctypes.c_int64(0)
    _lib.check(_lib.load().qz_gemm_w8_workspace_bytes(M, N, K, ctypes.byref(b)))
    return torch.zeros(max(b.value, 256), dtype=torch.uint8, device="cuda")


@pytest.mark.parametrize("N,K,M,act", [
    (3072, 1024, 4, "rmsnorm"),     # Qwen3-0.6B shapes, decode rows: qkv after the input norm
    (6144, 1024, 16, "rmsnorm"),    # gate|up after the post-attention norm
    (1024, 3072, 16, "silu"),       # down after silu(gate) * up
    (2048, 8192, 512, "silu"),      # Llama-1B prefill down
    (3072, 2048, 512, "rmsnorm"),   # Llama-1B prefill qkv
    (300, 4112, 3, "rmsnorm"),      # K not a multiple of 128, ragged rows
    (256, 48, 2, "silu"),           # K below one 512-thread pass
])
def test_gemm_activation_prologue_equals_separate_kernels(N, K, M, act):
    """qz_gemm_w8_act_ws with the RMSNorm or silu(g) * u computed in the
    GEMM's limb split equals qz_rmsnorm / qz_silu_mul followed by
    qz_gemm_w8_ws (same activation values, so the same limbs), and both are
    within the oracle's tolerance of the fp32 reference."""
    from quartz_b200 import _lib
    from quartz_b200.workloads import gemv_case
    lib = _lib.load()
    st = torch.cuda.current_stream().cuda_stream
    c = gemv_case(N, K, M, seed=N + 3 * K + M)
    q, s = _t(c.q), _t(c.scale)
    rng = np.random.default_rng(K)
    eps = 1e-6
    if act == "rmsnorm":
        X = _t(c.x * 3.0)
        w = _t(rng.standard_normal(K).astype(np.float32))
        mid = torch.empty(M, K, device="cuda")
        _lib.check(lib.qz_rmsnorm(X.data_ptr(), w.data_ptr(), mid.data_ptr(), M, K, eps, st))
        code, wp = _lib.QZ_ACT_RMSNORM, w.data_ptr()
    else:
        X = _t(rng.standard_normal((M, 2 * K)).astype(np.float32) * 4.0)
        mid = torch.empty(M, K, device="cuda")
        _lib.check(lib.qz_silu_mul(X.data_ptr(), mid.data_ptr(), M, K, st))
        code, wp = _lib.QZ_ACT_SILU_MUL, None
    ws = _gemm_ws(M, N, K)
    R = _t(rng.standard_normal((M, N)).astype(np.float32))
    Y_sep = torch.empty(M, N, device="cuda")
    Y_fused = torch.empty(M, N, device="cuda")
    _lib.check(lib.qz_gemm_w8_ws(q.data_ptr(), s.data_ptr(), 1, mid.data_ptr(), Y_sep.data_ptr(),
                                 M, N, K, R.data_ptr(), ws.data_ptr(), ws.numel(), st))
    for _ in range(2):   # twice: the workspace holds the previous call's limbs
        _lib.check(lib.qz_gemm_w8_act_ws(q.data_ptr(), s.data_ptr(), 1, X.data_ptr(), code, wp,
                                         eps, Y_fused.data_ptr(), M, N, K, R.data_ptr(),
                                         ws.data_ptr(), ws.numel(), st))
        torch.cuda.synchronize()
        assert torch.equal(Y_fused, Y_sep), f"{act} {N}x{K} M={M}: fused prologue differs"
    ref = _oracle_gemm(c.q, c.scale, mid.cpu().numpy()) + R.cpu().numpy()
    G.assert_close(Y_fused.cpu().numpy(), ref, what=f"{act} {N}x{K} M={M}")


def test_gemm_activation_prologue_rejections():
    """Outside the tensor path (one row, group scales) the prologue entry
    refuses with QZ_ERR_UNSUPPORTED and queues nothing; an unknown act is an
    argument error."""
    from quartz_b200 import _lib
    from quartz_b200.workloads import gemv_case
    lib = _lib.load()
    st = torch.cuda.current_stream().cuda_stream
    c = gemv_case(256, 1024, 4, seed=5)
    q, s, X = _t(c.q), _t(c.scale), _t(c.x)
    w = torch.ones(1024, device="cuda")
    Y = torch.zeros(4, 256, device="cuda")
    ws = _gemm_ws(4, 256, 1024)
    args = (ws.data_ptr(), ws.numel(), st)
    with pytest.raises(_lib.QuartzError):
        _lib.check(lib.qz_gemm_w8_act_ws(q.data_ptr(), s.data_ptr(), 1, X.data_ptr(),
                                         _lib.QZ_ACT_RMSNORM, w.data_ptr(), 1e-6, Y.data_ptr(),
                                         1, 256, 1024, None, *args))
    cg = gemv_case(256, 1024, 4, seed=6, group_size=128)
    with pytest.raises(_lib.QuartzError):
        _lib.check(lib.qz_gemm_w8_act_ws(_t(cg.q).data_ptr(), _t(cg.scale).data_ptr(), 8,
                                         X.data_ptr(), _lib.QZ_ACT_RMSNORM, w.data_ptr(), 1e-6,
                                         Y.data_ptr(), 4, 256, 1024, None, *args))
    with pytest.raises(ValueError):
        _lib.check(lib.qz_gemm_w8_act_ws(q.data_ptr(), s.data_ptr(), 1, X.data_ptr(), 7,
                                         w.data_ptr(), 1e-6, Y.data_ptr(), 4, 256, 1024, None,
                                         *args))
    torch.cuda.synchronize()
    assert float(Y.abs().max()) == 0.0
