"""Tensor-parallel decode (head-sharded attention, unit-sharded MLP, vocab-sharded
lm_head, NCCL / peer-memory / in-kernel all-reduces) on 2, 4 and 8 GPUs: the
greedy tokens must equal quartz's own on the same synthetic checkpoints
(tests/golden/golden_model.npz), eager and CUDA-graph replay, prefill and
prefilled-cache starts. A rank count needs that many visible GPUs and is
skipped otherwise. NVLS is left off (NCCL_NVLS_ENABLE=0)."""

import datetime
import json
import os
import socket
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLD = Path(REPO) / "tests" / "golden"


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, cids, variants):
    import sys
    sys.path.insert(0, REPO)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    torch.distributed.init_process_group(
        "nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
        timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    from quartz_b200 import device
    from quartz_b200.model import ModelSpec, cached_int8_weights, norm_weights, seeded_kv
    from quartz_b200.tp_decode import TPDecodeEngine
    cases = {c["id"]: c for c in json.loads((GOLD / "cases_model.json").read_text())["cases"]}
    try:
        with np.load(GOLD / "golden_model.npz") as z:
            golds = {cid: z[f"{cid}__tokens"].tolist() for cid in cids}
        for cid in cids:
            case = cases[cid]
            spec = ModelSpec.from_hf(case["cfg"], case["arch"])
            start = case.get("kv_len") or len(case["prompt"])
            eng_kind = None
            for allreduce, graph in variants:
                if graph is False or allreduce != eng_kind:
                    eng_kind = allreduce
                    eng = TPDecodeEngine(spec, cached_int8_weights(spec), norm_weights(spec),
                                         max_ctx=start + case["steps"],
                                         max_prefill=max(2, len(case.get("prompt", [])) or 2),
                                         device=torch.device("cuda", rank), allreduce=allreduce)
                if case["start"] == "kv":
                    eng.load_kv(seeded_kv(spec, case["kv_len"]))
                    toks = eng.generate(case["first"], case["steps"], graph=graph, unroll=8)
                else:
                    eng.reset(0)
                    t0 = eng.prefill(case["prompt"])
                    toks = [t0] + eng.generate(t0, case["steps"] - 1, graph=graph, unroll=8)
                assert toks == golds[cid], (cid, allreduce, graph, rank)
                if graph:
                    eng.close()   # the graph (it holds collectives) and the peer buffers
                    del eng
                    torch.cuda.synchronize()
        device.check_status(torch.device("cuda", rank))
    finally:
        torch.distributed.destroy_process_group()


ALL_VARIANTS = (("nccl", False), ("nccl", True), ("peer", False), ("peer", True),
                ("fused", False), ("fused", True))
# Cases whose head and unit counts divide by the rank count: the small models
# have 2 kv heads; the Qwen3-0.6B (8 kv heads, MLP 3072) and Llama-3.2-1B (8 kv
# heads, MLP 8192) architectures split up to 8 ways.
TP_CASES = {
    2: (["qwen3_small_kv", "llama_small_prompt", "qwen3_0p6b_kv512"], ALL_VARIANTS),
    4: (["qwen3_0p6b_kv512"], ALL_VARIANTS),
    8: (["qwen3_0p6b_kv512", "llama_1b_prompt512"], (("nccl", True), ("fused", False),
                                                    ("fused", True))),
}


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_decode_tokens_match_reference(world):
    """NCCL, peer-memory and in-kernel (fused) all-reduces, eager and graph replay."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    cids, variants = TP_CASES[world]
    mp.spawn(_worker, args=(world, _free_port(), cids, variants), nprocs=world, join=True)


def _batch_worker(rank, world, port, cids, variants):
    import sys
    sys.path.insert(0, REPO)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    torch.distributed.init_process_group(
        "nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
        timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    from quartz_b200 import device
    from quartz_b200.model import ModelSpec, cached_int8_weights, norm_weights, seeded_kv
    from quartz_b200.tp_decode import TPDecodeEngine
    cases = {c["id"]: c for c in json.loads((GOLD / "cases_model.json").read_text())["cases"]}
    try:
        with np.load(GOLD / "golden_model.npz") as z:
            golds = {cid: z[f"{cid}__tokens"].tolist() for cid in cids}
        for cid in cids:
            case = cases[cid]
            spec = ModelSpec.from_hf(case["cfg"], case["arch"])
            B = case["batch"]
            for allreduce, graph in variants:
                eng = TPDecodeEngine(spec, cached_int8_weights(spec), norm_weights(spec),
                                     max_ctx=case["kv_len"] + case["steps"], max_prefill=1,
                                     device=torch.device("cuda", rank), allreduce=allreduce,
                                     batch=B)
                eng.load_kv(seeded_kv(spec, case["kv_len"], batch=B))
                toks = eng.generate_batch(case["firsts"], case["steps"], graph=graph, unroll=8)
                assert toks == golds[cid], (cid, allreduce, graph, rank)
                eng.close()
                del eng
                torch.cuda.synchronize()
        device.check_status(torch.device("cuda", rank))
    finally:
        torch.distributed.destroy_process_group()


TP_BATCH_CASES = {
    2: (["qwen3_0p6b_kv512_b4"], (("nccl", False), ("peer", True), ("fused", True))),
    4: (["qwen3_0p6b_kv512_b8"], (("peer", True),)),
    8: (["qwen3_0p6b_kv512_b16", "qwen3_0p6b_kv512_b2"], (("nccl", True), ("peer", True))),
}


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_batch_decode_tokens_match_reference(world):
    """B sequences in lockstep over the ranks ([B, H] all-reduces): every row's
    greedy tokens equal quartz's batched decode."""
    if not torch.cuda.is_available() or torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    cids, variants = TP_BATCH_CASES[world]
    mp.spawn(_batch_worker, args=(world, _free_port(), cids, variants), nprocs=world, join=True)


def _ar_worker(rank, world, port):
    import sys
    sys.path.insert(0, REPO)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    torch.distributed.init_process_group(
        "nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
        timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    from quartz_b200 import device
    from quartz_b200.comm import PeerAllReduce
    try:
        ar = PeerAllReduce(8192, device=torch.device("cuda", rank))
        g = torch.Generator().manual_seed(5)
        for n in (4, 1024, 4096, 8192, 4 * 777):
            xs = [torch.randn(n, generator=g) for _ in range(world)]
            ref = xs[0].clone()
            for x in xs[1:]:
                ref += x            # rank order, like the kernel
            for rep in range(3):    # both parities, repeated calls
                t = xs[rank].cuda()
                out = ar(t)
                assert torch.equal(out.cpu(), ref), (n, rep)
        # many back-to-back calls in one CUDA graph
        t = torch.full((4096,), float(rank + 1), device="cuda")
        graph = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(graph, stream=s):
                for _ in range(20):
                    ar(t)
                    t.mul_(1.0 / world)
        torch.cuda.current_stream().wait_stream(s)
        graph.replay()
        torch.cuda.synchronize()
        total = world * (world + 1) / 2 / world
        assert torch.allclose(t, torch.full_like(t, total)), float(t[0])
        del graph
        ar.close()
        device.check_status(torch.device("cuda", rank))
    finally:
        torch.distributed.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs 2 GPUs")
def test_peer_allreduce_exact():
    """The peer-memory sum equals the rank-order fp32 sum bit for bit, on both
    buffer parities and inside a CUDA graph."""
    import torch.multiprocessing as mp
    world = min(torch.cuda.device_count(), 4)
    mp.spawn(_ar_worker, args=(world, _free_port()), nprocs=world, join=True)
