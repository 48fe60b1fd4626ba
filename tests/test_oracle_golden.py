"""Pin the CPU oracle (and our host quantiser) against outputs of the reference.

Every case regenerates its inputs from the stored seed, proves the int8 operands
are byte-identical to the reference quantiser's (SHA-256), runs the oracle, and
holds it to max|err| <= 1e-4 * ||y_ref||_inf.
"""

import numpy as np
import pytest

import oracle
from quartz_b200.quantize import quantize_symmetric, dequantize_symmetric
from tests import _golden as G


@pytest.mark.parametrize("cid", G.ids("gemv"))
def test_oracle_gemv(cid):
    c = G.case(cid)
    q, s, x = G.regen_gemv(c)
    y = np.empty(c["N"], np.float32)
    oracle.w8a32_gemv(q, s, x, y)
    ref, idx, inf = G.golden_out(c)
    G.assert_close(y if idx is None else y[idx], ref, inf, what=cid)


@pytest.mark.parametrize("cid", ["gemv_warmup", "gemv_edges"])
def test_oracle_gemv_explicit(cid):
    q, s, x, ref = (G.arr(cid, k) for k in ("q", "s", "x", "y"))
    y = np.empty(q.shape[0], np.float32)
    oracle.w8a32_gemv(q, s, x, y)
    G.assert_close(y, ref, what=cid)


@pytest.mark.parametrize("cid", G.ids("gemm"))
def test_oracle_gemm(cid):
    c = G.case(cid)
    q, s, X = G.regen_gemv(c)
    Y = np.empty((c["M"], c["N"]), np.float32)
    oracle.w8a32_gemm(q, s, X, Y)
    ref, idx, inf = G.golden_out(c)
    G.assert_close(Y if idx is None else Y.ravel()[idx], ref, inf, what=cid)


@pytest.mark.parametrize("cid", G.ids("matmul"))
def test_oracle_matmul_dispatch(cid):
    c = G.case(cid)
    q, s, x = G.regen_gemv(c)
    y = oracle.matmul_int8(q, s, x)
    ref = G.arr(cid, "y")
    assert y.shape == ref.shape == tuple(c["xshape"][:-1]) + (c["N"],)
    G.assert_close(y, ref, what=cid)


@pytest.mark.parametrize("cid", G.ids("mlp"))
def test_oracle_mlp(cid):
    c = G.case(cid)
    gu_q, gu_s, dq, ds, x = G.regen_mlp(c)
    ref = G.arr(cid, "y")
    if c["M"] == 1:
        abuf = np.empty(c["I"], np.float32)
        out = np.empty(c["H"], np.float32)
        oracle.fused_mlp_decode(gu_q, gu_s, np.ascontiguousarray(x[0]), dq, ds, abuf, out)
        G.assert_close(abuf, G.arr(cid, "abuf"), what=cid + " abuf")
        G.assert_close(out, ref, what=cid)
    else:
        out = oracle.mlp_per_op(gu_q, gu_s, dq, ds, x)
        G.assert_close(out, ref, what=cid)


def test_quantizer_matches_reference_bytes():
    W, q, s = (G.arr("quant0", k) for k in ("W", "q", "s"))
    q2, s2 = quantize_symmetric(W, 32)
    assert np.array_equal(q, q2) and np.array_equal(s, s2)
    assert q2.dtype == np.int8 and q2.flags["C_CONTIGUOUS"]
    # tests/test_kernels.py:62-69: round trip within half a step of the group absmax
    Wd = dequantize_symmetric(q2, s2, 32)
    assert np.abs(Wd - W).max() <= (np.abs(W).max() / 127.0) * 1.01


def test_quantizer_rejects_bad_group():
    with pytest.raises(ValueError):
        quantize_symmetric(np.zeros((4, 48), np.float32), 32)


def test_oracle_matmul_rejects_untiled_groups():
    q = np.zeros((4, 64), np.int8)
    s = np.ones((4, 3), np.float32)
    with pytest.raises(ValueError, match="do not tile"):
        oracle.matmul_int8(q, s, np.zeros((1, 64), np.float32))
