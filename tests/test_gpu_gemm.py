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
