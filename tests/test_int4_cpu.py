"""int4 weights on the host: the quantiser, the nibble packing and the numpy
oracle of the int4 GEMV (no GPU). quartz has no 4-bit path (a `bits` field kept
for future work, quartz/config.py:98), so these pin the format by its
definition: symmetric [-7, 7] per group, element 2i in the low nibble."""

import numpy as np
import pytest

import oracle
from quartz_b200.quantize import pack_int4, quantize_symmetric_int4, unpack_int4


@pytest.mark.parametrize("group_size", [None, 32, 128])
def test_quantize_int4_definition(group_size):
    rng = np.random.default_rng(5)
    W = (rng.standard_normal((37, 256)) * 0.02).astype(np.float32)
    W[3] = 0.0                                   # an all-zero row gets scale 1
    q4, s = quantize_symmetric_int4(W, group_size)
    G = group_size or 256
    assert q4.dtype == np.uint8 and q4.shape == (37, 128) and q4.flags.c_contiguous
    assert s.dtype == np.float32 and s.shape == (37, 256 // G)
    q = unpack_int4(q4)
    assert q.min() >= -7 and q.max() <= 7
    Wg = W.reshape(37, -1, G)
    want_s = (np.abs(Wg).max(axis=2) / 7.0).astype(np.float32)
    want_s[want_s == 0] = 1.0
    np.testing.assert_array_equal(s, want_s)
    want_q = np.clip(np.round(Wg / want_s[:, :, None]), -7, 7).astype(np.int8).reshape(37, 256)
    np.testing.assert_array_equal(q, want_q)
    assert (q[3] == 0).all() and (s[3] == 1.0).all()


def test_pack_layout_and_round_trip():
    q = np.array([[1, -1, 7, -8, 0, 3]], np.int8)
    q4 = pack_int4(q)
    # byte i = low nibble q[2i] | high nibble q[2i+1], two's complement
    assert q4.tolist() == [[0xF1, 0x87, 0x30]]
    rng = np.random.default_rng(1)
    r = rng.integers(-8, 8, (9, 64)).astype(np.int8)
    np.testing.assert_array_equal(unpack_int4(pack_int4(r)), r)
    with pytest.raises(ValueError):
        pack_int4(np.zeros((2, 3), np.int8))


@pytest.mark.parametrize("ng", [1, 4])
def test_int4_oracle_matches_dequantised_matmul(ng):
    rng = np.random.default_rng(2)
    N, K = 50, 512
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
    q4, s = quantize_symmetric_int4(W, None if ng == 1 else K // ng)
    x = rng.standard_normal(K).astype(np.float32)
    y = np.empty(N, np.float32)
    oracle.w4a32_gemv(q4, s, x, y)
    q = unpack_int4(q4).astype(np.float64).reshape(N, ng, K // ng)
    ref = ((q * s.astype(np.float64)[:, :, None]).reshape(N, K) @ x.astype(np.float64))
    np.testing.assert_allclose(y, ref.astype(np.float32), rtol=1e-6, atol=1e-6)


def test_w4a32_gemv_validates_before_touching_the_gpu():
    """The numpy entry point rejects bad operands on the host (no GPU needed)."""
    from quartz_b200.kernels import w4a32_gemv
    q4 = np.zeros((4, 32), np.uint8)          # K = 64
    s = np.ones((4, 1), np.float32)
    x = np.zeros(64, np.float32)
    y = np.zeros(4, np.float32)
    with pytest.raises(TypeError, match="uint8"):
        w4a32_gemv(q4.view(np.int8), s, x, y)
    with pytest.raises(ValueError, match="rows"):
        w4a32_gemv(q4, np.ones((3, 1), np.float32), x, y)
    with pytest.raises(ValueError, match="do not tile"):
        w4a32_gemv(q4, np.ones((4, 3), np.float32), x, y)
    with pytest.raises(ValueError, match="shape"):
        w4a32_gemv(q4, s, np.zeros(32, np.float32), y)
    with pytest.raises(TypeError, match="y must be"):
        w4a32_gemv(q4, s, x, np.zeros(4, np.float64))
    with pytest.raises(ValueError, match="writeable"):
        ro = np.zeros(4, np.float32)
        ro.setflags(write=False)
        w4a32_gemv(q4, s, x, ro)
