"""The allocation-free fused MLP entry point, qz_fused_mlp_decode_noalloc.

It exists for callers that may not allocate device memory themselves -- a host
engine whose device memory belongs to another allocator, or a caller with no
allocation rights after start-up -- so it keeps its scratch in a fixed
device-side array inside the library instead of taking abuf / sync_ws.

Checked through the C ABI: two calls in a row give the same results as the
regular entry point and as the CPU oracle (within the parity tolerance,
1e-4 * ||y||_inf), on the one-launch kernel's shapes, on a shape that takes
the two-launch fallback and at the array's capacity (I = 32768); the calls
leave the device's free memory unchanged; an intermediate size beyond the
array's capacity is refused. This file sorts last so that a run stopping at
the first failure has run every other test first.
"""

import numpy as np
import pytest

from tests import _golden as G

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")

NOALLOC_MAX_I = 32768


def _ptr(t):
    return None if t is None else t.data_ptr()


def _oracle_mlp(m, x, residual):
    import oracle
    H, I = m.down_q.shape
    out = np.empty(H, np.float32)
    oracle.fused_mlp_decode(m.gu_q, m.gu_s, np.ascontiguousarray(x), m.down_q, m.down_s,
                            np.empty(I, np.float32), out)
    return out if residual is None else out + residual


@pytest.mark.parametrize("H,I", [(1024, 3072), (2048, 8192),
                                 (1024, 1000),            # I % 16 != 0: two-launch fallback
                                 (64, NOALLOC_MAX_I)])    # the array's capacity
def test_noalloc_matches_regular_entry_point_twice(H, I):
    from quartz_b200 import _lib, device
    from quartz_b200.workloads import mlp_case

    lib = _lib.load()
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    device.ensure_device(dev)
    device.status(clear=True)
    stream = torch.cuda.current_stream(dev).cuda_stream
    m = mlp_case(H, I, seed=1000 + I)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
    gq, gs, dq, ds = t(m.gu_q), t(m.gu_s), t(m.down_q), t(m.down_s)
    x_np = [m.x[0], np.random.default_rng(7).standard_normal(H).astype(np.float32)]
    res_np = np.random.default_rng(8).standard_normal(H).astype(np.float32)
    xs = [t(x) for x in x_np]
    res = t(res_np)
    outs = [torch.full((H,), float("nan"), dtype=torch.float32, device=dev) for _ in xs]
    refs = [device.fused_mlp(gq, gs, x, dq, ds, residual=(res if call == 1 else None))
            for call, x in enumerate(xs)]
    torch.cuda.synchronize(dev)

    def noalloc(call):
        rc = lib.qz_fused_mlp_decode_noalloc(
            gq.data_ptr(), gs.data_ptr(), gs.shape[1], xs[call].data_ptr(), dq.data_ptr(),
            ds.data_ptr(), ds.shape[1], outs[call].data_ptr(),
            _ptr(res if call == 1 else None), H, I, stream)
        _lib.check(rc)

    noalloc(0)                         # the first call on the device sets the array up
    torch.cuda.synchronize(dev)
    free0 = torch.cuda.mem_get_info(dev)[0]
    for call in range(2):              # two calls in a row, the second with a residual
        noalloc(call)
    torch.cuda.synchronize(dev)
    free1 = torch.cuda.mem_get_info(dev)[0]
    assert free1 == free0, f"device free memory changed by {free0 - free1} bytes"
    for call in range(2):
        got = outs[call].cpu().numpy()
        G.assert_close(got, refs[call].cpu().numpy(),
                       what=f"no-alloc vs qz_fused_mlp_decode H={H} I={I} call {call}")
        G.assert_close(got, _oracle_mlp(m, x_np[call], res_np if call == 1 else None),
                       what=f"no-alloc vs oracle H={H} I={I} call {call}")
    device.check_status(dev)


def test_noalloc_refuses_oversized_intermediate():
    from quartz_b200 import _lib

    lib = _lib.load()
    rc = lib.qz_fused_mlp_decode_noalloc(None, None, 1, None, None, None, 1, None, None,
                                         1024, NOALLOC_MAX_I + 1, None)
    assert rc == _lib.QZ_ERR_INVALID
    assert str(NOALLOC_MAX_I) in _lib.last_error()
