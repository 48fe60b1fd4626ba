"""CUDA parity: the sm_100a kernels against the reference's golden outputs and
against the CPU oracle, through the public numpy-signature API and the C ABI.

Bar: max |err| <= 1e-4 * ||y_ref||_inf per output (fp32 outputs).
"""

import numpy as np
import pytest

import oracle
from tests import _golden as G

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def K():
    from quartz_b200 import kernels
    kernels.warmup()
    kernels.warmup_fused()
    return kernels


@pytest.fixture(scope="module", autouse=True)
def _clean_status():
    from quartz_b200 import device
    if torch.cuda.is_available():
        device.status(clear=True)
    yield
    if torch.cuda.is_available():
        device.check_status()


def _dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


@pytest.mark.parametrize("cid", G.ids("gemv"))
def test_gemv_golden(K, cid):
    c = G.case(cid)
    q, s, x = G.regen_gemv(c)
    y = np.empty(c["N"], np.float32)
    K.w8a32_gemv(q, s, x, y)
    ref, idx, inf = G.golden_out(c)
    G.assert_close(y if idx is None else y[idx], ref, inf, what=cid)
    if idx is not None:  # full vector against the oracle too
        yo = np.empty_like(y)
        oracle.w8a32_gemv(q, s, x, yo)
        G.assert_close(y, yo, what=cid + " vs oracle")


@pytest.mark.parametrize("cid", ["gemv_warmup", "gemv_edges"])
def test_gemv_explicit(K, cid):
    q, s, x, ref = (G.arr(cid, k) for k in ("q", "s", "x", "y"))
    y = np.empty(q.shape[0], np.float32)
    K.w8a32_gemv(q, s, x, y)
    G.assert_close(y, ref, what=cid)


@pytest.mark.parametrize("cid", G.ids("gemm"))
def test_gemm_golden(K, cid):
    c = G.case(cid)
    q, s, X = G.regen_gemv(c)
    Y = np.empty((c["M"], c["N"]), np.float32)
    K.w8a32_gemm(q, s, X, Y)
    ref, idx, inf = G.golden_out(c)
    G.assert_close(Y if idx is None else Y.ravel()[idx], ref, inf, what=cid)


@pytest.mark.parametrize("cid", G.ids("matmul"))
def test_matmul_dispatch_golden(K, cid):
    c = G.case(cid)
    q, s, x = G.regen_gemv(c)
    y = K.matmul_int8(q, s, x)
    ref = G.arr(cid, "y")
    assert y.shape == ref.shape
    G.assert_close(y, ref, what=cid)


@pytest.mark.parametrize("cid", G.ids("mlp"))
def test_mlp_golden(K, cid):
    from quartz_b200 import device
    c = G.case(cid)
    gu_q, gu_s, dq, ds, x = G.regen_mlp(c)
    ref = G.arr(cid, "y")
    if c["M"] == 1:
        abuf = np.empty(c["I"], np.float32)
        out = np.empty(c["H"], np.float32)
        K.fused_mlp_decode(gu_q, gu_s, np.ascontiguousarray(x[0]), dq, ds, abuf, out)
        G.assert_close(abuf, G.arr(cid, "abuf"), what=cid + " abuf")
        G.assert_close(out, ref, what=cid)
    else:
        # quartz/quantize.py:112-114: gate|up GEMM, clipped silu * up, down GEMM
        gu = device.gemm(_dev(gu_q), _dev(gu_s), _dev(x))
        a = device.silu_mul(gu)
        out = device.gemm(_dev(dq), _dev(ds), a).cpu().numpy()
        G.assert_close(out, ref, what=cid)


SHAPES = [(151936, 1024), (3072, 1024), (1024, 3072), (2048, 1024), (1024, 1024), (64, 32)]


@pytest.mark.parametrize("N,Kd", SHAPES)
@pytest.mark.parametrize("group_size", [None, 64])
def test_gemv_matches_fp32(K, N, Kd, group_size):
    """tests/test_kernels.py:21-33 of the reference: cos > 0.999 vs fp32 x @ W.T."""
    if group_size and Kd % group_size:
        pytest.skip("K not divisible by group_size")
    from quartz_b200.quantize import quantize_symmetric
    rng = np.random.default_rng(0)
    W = (rng.standard_normal((N, Kd)) * 0.05).astype(np.float32)
    x = rng.standard_normal(Kd).astype(np.float32)
    ref = (x.reshape(1, Kd) @ W.T).ravel()
    q, scale = quantize_symmetric(W, group_size)
    y = np.empty(N, np.float32)
    K.w8a32_gemv(q, scale, x, y)
    cos = float(y @ ref / (np.linalg.norm(y) * np.linalg.norm(ref) + 1e-12))
    assert cos > 0.999


def test_gemm_rows_match_gemv(K):
    """tests/test_kernels.py:36-47: GEMM rows equal GEMV rows (atol 1e-4)."""
    from quartz_b200.quantize import quantize_symmetric
    rng = np.random.default_rng(1)
    N, Kd, M = 128, 64, 5
    q, scale = quantize_symmetric((rng.standard_normal((N, Kd)) * 0.05).astype(np.float32), None)
    X = rng.standard_normal((M, Kd)).astype(np.float32)
    Y = np.empty((M, N), np.float32)
    K.w8a32_gemm(q, scale, X, Y)
    for m in range(M):
        y = np.empty(N, np.float32)
        K.w8a32_gemv(q, scale, np.ascontiguousarray(X[m]), y)
        assert np.allclose(Y[m], y, atol=1e-4)


def test_serial_bit_identical(K):
    """tests/test_fused.py:45-52: the serial twin is bit-identical."""
    from quartz_b200.workloads import gemv_case
    c = gemv_case(200, 128, seed=1, std=0.05, recipe="f64")
    yp, ys = np.empty(200, np.float32), np.empty(200, np.float32)
    K.w8a32_gemv(c.q, c.scale, c.x[0], yp)
    K.w8a32_gemv_serial(c.q, c.scale, c.x[0], ys)
    assert np.array_equal(yp, ys)


def test_gemv_deterministic(K):
    from quartz_b200.workloads import gemv_case
    c = gemv_case(50000, 1024, seed=3)
    y1, y2 = np.empty(50000, np.float32), np.empty(50000, np.float32)
    K.w8a32_gemv(c.q, c.scale, c.x[0], y1)
    K.w8a32_gemv(c.q, c.scale, c.x[0], y2)
    assert np.array_equal(y1, y2)


def test_residual_fused(K):
    from quartz_b200 import device
    from quartz_b200.workloads import gemv_case, mlp_case
    c = gemv_case(3000, 2048, seed=4)
    r = np.random.default_rng(5).standard_normal(3000).astype(np.float32)
    y = device.gemv(_dev(c.q), _dev(c.scale), _dev(c.x[0]), residual=_dev(r)).cpu().numpy()
    yo = np.empty(3000, np.float32)
    oracle.w8a32_gemv(c.q, c.scale, c.x[0], yo)
    G.assert_close(y, yo + r, what="gemv + residual")
    m = mlp_case(256, 1024, seed=6)
    rr = np.random.default_rng(7).standard_normal(256).astype(np.float32)
    out = device.fused_mlp(_dev(m.gu_q), _dev(m.gu_s), _dev(m.x[0]), _dev(m.down_q),
                           _dev(m.down_s), residual=_dev(rr)).cpu().numpy()
    o = np.empty(256, np.float32)
    oracle.fused_mlp_decode(m.gu_q, m.gu_s, m.x[0], m.down_q, m.down_s,
                            np.empty(1024, np.float32), o)
    G.assert_close(out, o + rr, what="mlp + residual")


@pytest.mark.parametrize("N,Kd,ng", [(1, 16, 1), (8, 16, 1), (9, 1040, 1), (77, 2064, 3),
                                     (300, 5120, 5), (17, 12288, 96), (1000, 48, 3)])
def test_gemv_odd_shapes_vs_oracle(K, N, Kd, ng):
    """Ragged row groups, K not a multiple of the 1 KB stage segment, many groups."""
    from quartz_b200.workloads import gemv_case
    c = gemv_case(N, Kd, seed=N + Kd, group_size=Kd // ng if ng > 1 else None)
    y = np.empty(N, np.float32)
    K.w8a32_gemv(c.q, c.scale, c.x[0], y)
    yo = np.empty(N, np.float32)
    oracle.w8a32_gemv(c.q, c.scale, c.x[0], yo)
    G.assert_close(y, yo, what=f"{N}x{Kd}/{ng}")


@pytest.mark.parametrize("H,I", [(1024, 3072), (16, 16), (64, 1040), (2048, 8192), (1040, 48)])
def test_fused_mlp_vs_oracle(K, H, I):
    from quartz_b200.workloads import mlp_case
    m = mlp_case(H, I, seed=H * 7 + I)
    abuf, out = np.empty(I, np.float32), np.empty(H, np.float32)
    K.fused_mlp_decode(m.gu_q, m.gu_s, m.x[0], m.down_q, m.down_s, abuf, out)
    ab, o = np.empty(I, np.float32), np.empty(H, np.float32)
    oracle.fused_mlp_decode(m.gu_q, m.gu_s, m.x[0], m.down_q, m.down_s, ab, o)
    G.assert_close(abuf, ab, what="abuf")
    G.assert_close(out, o, what="out")


def test_matmul_rejects_untiled_groups(K):
    with pytest.raises(ValueError, match="do not tile"):
        K.matmul_int8(np.zeros((4, 64), np.int8), np.ones((4, 3), np.float32),
                      np.zeros((1, 64), np.float32))


def test_device_api_rejects_bad_args(K):
    from quartz_b200 import device
    q = torch.zeros((4, 64), dtype=torch.int8, device="cuda")
    with pytest.raises(ValueError):
        device.gemv(q, torch.ones((4, 3), device="cuda"), torch.zeros(64, device="cuda"))
    with pytest.raises(TypeError):
        device.gemv(q.float(), torch.ones((4, 1), device="cuda"), torch.zeros(64, device="cuda"))


@pytest.mark.parametrize("N,Kd,group_size,res", [(151936, 1024, None, False),
                                                 (4096, 4096, 128, False),
                                                 (1000, 1056, None, True),
                                                 (3072, 2048, 32, False),
                                                 (77, 64, None, False),
                                                 (20000, 2048, 64, True)])
def test_w4a32_gemv_vs_oracle(K, N, Kd, group_size, res):
    """int4 weights (two per byte) through the numpy API and the torch API
    against the numpy oracle: eight-row groups (lm_head shape; 20000 rows with
    group scales and a residual), two-row groups with group scales, rows that
    are not a whole number of 512-byte segments (K = 1056, K = 64)."""
    from quartz_b200 import device
    from quartz_b200.quantize import quantize_symmetric_int4
    rng = np.random.default_rng(N + Kd)
    W = (rng.standard_normal((N, Kd)) * 0.02).astype(np.float32)
    q4, s = quantize_symmetric_int4(W, group_size)
    x = rng.standard_normal(Kd).astype(np.float32)
    r = rng.standard_normal(N).astype(np.float32) if res else None
    ref = np.empty(N, np.float32)
    oracle.w4a32_gemv(q4, s, x, ref)
    if res:
        ref = ref + r
    if not res:
        y = np.empty(N, np.float32)
        K.w4a32_gemv(q4, s, x, y)
        G.assert_close(y, ref, what=f"w4 numpy {N}x{Kd}")
    yd = device.gemv_w4(_dev(q4), _dev(s), _dev(x), residual=_dev(r) if res else None)
    G.assert_close(yd.cpu().numpy(), ref, what=f"w4 torch {N}x{Kd}")


def test_w4a32_gemv_rejects_bad_shapes(K):
    from quartz_b200 import device
    q4 = torch.zeros(8, 24, dtype=torch.uint8, device="cuda")      # K = 48
    with pytest.raises(Exception, match="multiples of 32"):
        device.gemv_w4(q4, torch.ones(8, 1, device="cuda"), torch.ones(48, device="cuda"))


def test_numpy_weight_cache_follows_the_arrays():
    """The numpy entry points keep a device copy of each weight array: the same
    object hits it without rebuilding its key, a view of the same buffer shares
    it, invalidate() after an in-place change re-uploads, and the copy is
    dropped when the array is freed."""
    import gc
    from quartz_b200 import _host
    from quartz_b200.kernels import w8a32_gemv
    from quartz_b200.workloads import gemv_case
    c = gemv_case(4096, 1024, seed=11)
    q, s = c.q.copy(), c.scale.copy()
    x = c.x[0].copy()

    def ref(qq):
        y = np.empty(qq.shape[0], np.float32)
        oracle.w8a32_gemv(qq, s, x, y)
        return y

    y = np.empty(4096, np.float32)
    w8a32_gemv(q, s, x, y)
    G.assert_close(y, ref(q), what="first call")
    d = torch.cuda.current_device()
    assert _host.resident(q, d) is _host.resident(q, d)
    v = q[:]                       # another object over the same buffer
    assert _host.resident(v, d) is _host.resident(q, d)
    y2 = np.empty_like(y)
    w8a32_gemv(v, s, x, y2)
    assert np.array_equal(y, y2)
    q[:100] = -q[:100]             # in-place change, announced
    _host.invalidate(q)
    w8a32_gemv(q, s, x, y)
    G.assert_close(y, ref(q), what="after invalidate")
    before = _host.cached_bytes()
    del q, v
    gc.collect()
    assert _host.cached_bytes() <= before - 4096 * 1024
