"""Vocab-parallel lm_head and tensor-parallel MLP on CPU ranks (gloo).

The partition logic of quartz_b200.sharding runs on world_size 2 and 3 with
the local compute done by the CPU oracle, and is checked against the
unsharded oracle: greedy tokens equal np.argmax of the full logits (ties to
the lowest index), full logits within 1e-4 * ||y||_inf, and the MLP all-reduce
reproduces the unsharded MLP plus residual. A rank that dies before a
collective makes the others fail within the process-group timeout, not hang.
"""

import datetime
import os
import socket
import sys
import traceback

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class OracleOps:
    """CPU stand-ins for quartz_b200.device, computed by the oracle."""

    @staticmethod
    def gemv(q, s, x, y=None, residual=None):
        import oracle
        out = np.empty(q.shape[0], np.float32)
        oracle.w8a32_gemv(q.numpy(), s.numpy(), np.ascontiguousarray(x.numpy()), out)
        return torch.from_numpy(out)

    @staticmethod
    def gemm(q, s, X, Y=None, residual=None):
        import oracle
        out = np.empty((X.shape[0], q.shape[0]), np.float32)
        oracle.w8a32_gemm(q.numpy(), s.numpy(), np.ascontiguousarray(X.numpy()), out)
        return torch.from_numpy(out)

    @staticmethod
    def fused_mlp(gu_q, gu_s, x, dq, ds, abuf=None, out=None, residual=None):
        import oracle
        I = gu_q.shape[0] // 2
        o = np.empty(dq.shape[0], np.float32)
        oracle.fused_mlp_decode(gu_q.numpy(), gu_s.numpy(), np.ascontiguousarray(x.numpy()),
                                dq.numpy(), ds.numpy(), np.empty(I, np.float32), o)
        return torch.from_numpy(o)

    @staticmethod
    def silu_mul(gu, a=None):
        import oracle
        g = gu.numpy()
        I = g.shape[-1] // 2
        return torch.from_numpy(
            np.ascontiguousarray(oracle.silu_clipped(g[..., :I]) * g[..., I:]).astype(np.float32))


def _init(rank, world, port, seconds=30):
    sys.path.insert(0, REPO)
    torch.distributed.init_process_group(
        "gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
        timeout=datetime.timedelta(seconds=seconds))


def _lm_head_worker(rank, world, port):
    _init(rank, world, port)
    import oracle
    from quartz_b200.sharding import ShardedLMHead
    from quartz_b200.workloads import gemv_case
    try:
        for M in (1, 3):
            c = gemv_case(1001, 64, M, seed=5 + M)
            head = ShardedLMHead(torch.from_numpy(c.q), torch.from_numpy(c.scale), ops=OracleOps)
            x = torch.from_numpy(c.x)
            full = np.empty((M, 1001), np.float32)
            oracle.w8a32_gemm(c.q, c.scale, c.x, full) if M > 1 else oracle.w8a32_gemv(
                c.q, c.scale, c.x[0], full[0])
            tok = head.argmax(x).numpy()
            assert np.array_equal(tok, full.argmax(axis=1)), (tok, full.argmax(axis=1))
            lg = head.logits(x).numpy()
            assert lg.shape == (M, 1001)
            assert np.abs(lg - full).max() <= 1e-4 * np.abs(full).max()
        # exact ties across and within shards: lowest global index wins
        q = np.zeros((1001, 64), np.int8)
        s = np.ones((1001, 1), np.float32)
        q[[10, 900, 600, 700]] = 100
        q[[600, 700], 0] = 101            # 600 and 700 tie above 10 and 900
        x = np.ones((1, 64), np.float32)
        head = ShardedLMHead(torch.from_numpy(q), torch.from_numpy(s), ops=OracleOps)
        assert int(head.argmax(torch.from_numpy(x))[0]) == 600
        q[[600, 700], 0] = 100            # now all four tie: 10 wins
        head = ShardedLMHead(torch.from_numpy(q), torch.from_numpy(s), ops=OracleOps)
        assert int(head.argmax(torch.from_numpy(x))[0]) == 10
    finally:
        torch.distributed.destroy_process_group()


def _mlp_worker(rank, world, port):
    _init(rank, world, port)
    import oracle
    from quartz_b200.quantize import quantize_symmetric
    from quartz_b200.sharding import ShardedMLP
    from quartz_b200.workloads import draw_weight
    try:
        for gs in (None, 32):
            rng = np.random.default_rng(3)
            H, I = 64, 96
            gq, gsc = quantize_symmetric(draw_weight(rng, (I, H)), gs)
            uq, usc = quantize_symmetric(draw_weight(rng, (I, H)), gs)
            dq, dsc = quantize_symmetric(draw_weight(rng, (H, I)), gs)
            T = torch.from_numpy
            mlp = ShardedMLP(T(gq), T(gsc), T(uq), T(usc), T(dq), T(dsc), ops=OracleOps)
            align = 1 if gs is None else gs
            assert mlp.hi - mlp.lo >= (I // align) // world * align, (mlp.lo, mlp.hi)
            gu_q = np.concatenate([gq, uq]); gu_s = np.concatenate([gsc, usc])
            for M in (1, 4):
                x = rng.standard_normal((M, H)).astype(np.float32)
                r = rng.standard_normal((M, H)).astype(np.float32)
                out = mlp(T(x), residual=T(r)).numpy()
                if M == 1:
                    ref = np.empty(H, np.float32)
                    oracle.fused_mlp_decode(gu_q, gu_s, x[0], dq, dsc, np.empty(I, np.float32), ref)
                    ref = ref[None]
                else:
                    ref = oracle.mlp_per_op(gu_q, gu_s, dq, dsc, x)
                ref = ref + r
                assert np.abs(out - ref).max() <= 1e-4 * np.abs(ref).max(), (gs, M)
    finally:
        torch.distributed.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_lm_head_matches_unsharded(world):
    mp.spawn(_lm_head_worker, args=(world, _free_port()), nprocs=world, join=True)


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_mlp_matches_unsharded(world):
    mp.spawn(_mlp_worker, args=(world, _free_port()), nprocs=world, join=True)


def test_shard_range_covers_and_aligns():
    from quartz_b200.sharding import shard_range
    for n, w, a in [(151936, 8, 1), (12288, 8, 128), (96, 2, 32), (5, 8, 1)]:
        parts = [shard_range(n, w, r, a) for r in range(w)]
        assert parts[0][0] == 0 and parts[-1][1] == n
        assert all(parts[i][1] == parts[i + 1][0] for i in range(w - 1))
        assert all(lo % a == 0 for lo, _ in parts)
    with pytest.raises(ValueError):
        shard_range(100, 2, 0, align=32)


def _dying_rank_worker(rank, world, port, outdir):
    _init(rank, world, port, seconds=3)
    from quartz_b200.sharding import ShardedMLP
    status = "ok"
    try:
        if rank == 1:
            raise SystemExit(3)             # leaves before the collective
        t = torch.ones(8)
        torch.distributed.all_reduce(t)     # must fail, not hang
        status = "no error"
    except SystemExit:
        raise
    except Exception as e:  # noqa: BLE001
        status = "error: " + type(e).__name__
    finally:
        with open(os.path.join(outdir, f"rank{rank}.txt"), "w") as f:
            f.write(status)
    os._exit(0)


def test_rank_that_leaves_makes_peers_fail_not_hang(tmp_path):
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_dying_rank_worker, args=(r, 2, port, str(tmp_path)))
             for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    assert not alive, "a rank hung in the collective"
    assert (tmp_path / "rank0.txt").read_text().startswith("error"), (tmp_path / "rank0.txt").read_text()
