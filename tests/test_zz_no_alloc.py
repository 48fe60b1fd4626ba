"""The allocation-free fused MLP entry point, qz_fused_mlp_decode_noalloc.

It exists for callers that may not allocate device memory themselves -- a host
engine whose device memory belongs to another allocator, or a caller with no
allocation rights after start-up -- so it keeps its scratch in a fixed
device-side array inside the library instead of taking abuf / sync_ws.

Checked through the C ABI: two calls in a row give the same results as the
regular entry point (within the parity tolerance, 1e-4 * ||y||_inf), and an
intermediate size beyond the array's capacity is refused. This file sorts last
so that a run stopping at the first failure has run every other test first.
"""

import numpy as np
import pytest

from tests import _golden as G

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _ptr(t):
    return None if t is None else t.data_ptr()


def test_noalloc_matches_regular_entry_point_twice():
    from quartz_b200 import _lib, device
    from quartz_b200.workloads import mlp_case

    lib = _lib.load()
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    device.ensure_device(dev)
    device.status(clear=True)
    stream = torch.cuda.current_stream(dev).cuda_stream
    cases = [mlp_case(1024, 3072, seed=1000), mlp_case(2048, 8192, seed=1001)]
    for m in cases:
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
        gq, gs, dq, ds = t(m.gu_q), t(m.gu_s), t(m.down_q), t(m.down_s)
        H, I = m.down_q.shape
        xs = [t(m.x[0]), t(np.random.default_rng(7).standard_normal(H).astype(np.float32))]
        res = t(np.random.default_rng(8).standard_normal(H).astype(np.float32))
        for call, x in enumerate(xs):
            residual = res if call == 1 else None
            ref = device.fused_mlp(gq, gs, x, dq, ds, residual=residual)
            out = torch.full((H,), float("nan"), dtype=torch.float32, device=dev)
            rc = lib.qz_fused_mlp_decode_noalloc(
                gq.data_ptr(), gs.data_ptr(), gs.shape[1], x.data_ptr(), dq.data_ptr(),
                ds.data_ptr(), ds.shape[1], out.data_ptr(), _ptr(residual), H, I, stream)
            _lib.check(rc)
            torch.cuda.synchronize(dev)
            G.assert_close(out.cpu().numpy(), ref.cpu().numpy(),
                           what=f"no-alloc H={H} I={I} call {call}")
    device.check_status(dev)


def test_noalloc_refuses_oversized_intermediate():
    from quartz_b200 import _lib

    lib = _lib.load()
    rc = lib.qz_fused_mlp_decode_noalloc(None, None, 1, None, None, None, 1, None, None,
                                         1024, 32769, None)
    assert rc == _lib.QZ_ERR_INVALID
    assert "32768" in _lib.last_error()
