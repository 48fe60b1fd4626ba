"""Vocab-parallel lm_head and tensor-parallel MLP on 2+ GPUs over NCCL, against
the CPU oracle. Skipped on a single-GPU host. NVLS is left off (NCCL_NVLS_ENABLE=0)."""

import datetime
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port):
    import sys
    sys.path.insert(0, REPO)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    torch.distributed.init_process_group(
        "nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
        timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    import oracle
    from quartz_b200 import device
    from quartz_b200.sharding import ShardedLMHead, ShardedMLP
    from quartz_b200.workloads import gemv_case, mlp_case
    try:
        dev = torch.device("cuda", rank)
        T = lambda a: torch.from_numpy(np.ascontiguousarray(a))  # noqa: E731
        for M in (1, 4):
            c = gemv_case(151936, 1024, M, seed=40 + M)
            head = ShardedLMHead(T(c.q), T(c.scale), device=dev)
            full = np.empty((M, 151936), np.float32)
            if M == 1:
                oracle.w8a32_gemv(c.q, c.scale, c.x[0], full[0])
            else:
                oracle.w8a32_gemm(c.q, c.scale, c.x, full)
            x = T(c.x).to(dev)
            lg = head.logits(x).cpu().numpy()
            assert np.abs(lg - full).max() <= 1e-4 * np.abs(full).max()
            tok = head.argmax(x).cpu().numpy()
            # the greedy choice must be a maximiser of the oracle's logits up to rounding
            for m in range(M):
                assert full[m, tok[m]] >= full[m].max() - 1e-4 * np.abs(full[m]).max()
        m = mlp_case(1024, 3072, 3, seed=77)
        I = 3072
        mlp = ShardedMLP(T(m.gu_q[:I]), T(m.gu_s[:I]), T(m.gu_q[I:]), T(m.gu_s[I:]),
                         T(m.down_q), T(m.down_s), device=dev)
        for M in (1, 3):
            x = m.x[:M]
            out = mlp(T(x).to(dev)).cpu().numpy()
            if M == 1:
                ref = np.empty(1024, np.float32)
                oracle.fused_mlp_decode(m.gu_q, m.gu_s, x[0], m.down_q, m.down_s,
                                        np.empty(I, np.float32), ref)
                ref = ref[None]
            else:
                ref = oracle.mlp_per_op(m.gu_q, m.gu_s, m.down_q, m.down_s, x)
            assert np.abs(out - ref).max() <= 1e-4 * np.abs(ref).max(), M
        device.check_status(dev)
    finally:
        torch.distributed.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_tensor_parallel_on_gpus():
    import torch.multiprocessing as mp
    world = min(torch.cuda.device_count(), 4)
    mp.spawn(_worker, args=(world, _free_port()), nprocs=world, join=True)
