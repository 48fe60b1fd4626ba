"""Seeded synthetic workloads for the int8 weight-only path.

Every input the tests and the benchmark use is drawn here from
``np.random.default_rng(seed)`` so that any run can be reproduced from its seed.
Two weight recipes exist because the reference uses two:

* ``"f32"`` (the benchmark recipe): ``rng.standard_normal(shape, dtype=float32)
  * float32(std)`` with std 0.02 -- the distribution of the lm_head / MLP
  workloads (Qwen3-0.6B lm_head [151936, 1024]; MLP H=1024, I=3072 per layer).
* ``"f64"`` (the recipe of quartz's own kernel tests, tests/test_kernels.py:25-26):
  ``(rng.standard_normal(shape) * std).astype(float32)`` with std 0.05.

Activations are N(0, 1) fp32 in both recipes.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from .quantize import quantize_symmetric, stack_gate_up

# Qwen3-0.6B shapes (hidden 1024, MLP 3072, 28 layers, tied vocab 151936).
LM_HEAD_N = 151936
LM_HEAD_K = 1024
MLP_H = 1024
MLP_I = 3072
MLP_LAYERS = 28
MLP_LAYER_SEED0 = 1000


def draw_weight(rng, shape, std=0.02, recipe="f32") -> np.ndarray:
    if recipe == "f32":
        return rng.standard_normal(shape, dtype=np.float32) * np.float32(std)
    if recipe == "f64":
        return (rng.standard_normal(shape) * std).astype(np.float32)
    raise ValueError(f"unknown weight recipe {recipe!r}")


def draw_act(rng, shape, recipe="f32") -> np.ndarray:
    if recipe == "f32":
        return rng.standard_normal(shape, dtype=np.float32)
    return rng.standard_normal(shape).astype(np.float32)


@dataclass
class GemvCase:
    q: np.ndarray       # int8 [N, K]
    scale: np.ndarray   # fp32 [N, ng]
    x: np.ndarray       # fp32 [M, K]


def gemv_case(N, K, M=1, *, seed=0, group_size=None, std=0.02, recipe="f32") -> GemvCase:
    """Weights first, then activations, from one rng (the lm_head recipe when
    N=151936, K=1024, seed 0)."""
    rng = np.random.default_rng(seed)
    W = draw_weight(rng, (N, K), std, recipe)
    q, s = quantize_symmetric(W, group_size)
    del W
    x = draw_act(rng, (M, K), recipe)
    return GemvCase(q, s, x)


@dataclass
class MlpCase:
    gu_q: np.ndarray    # int8 [2I, H]  (gate rows, then up rows)
    gu_s: np.ndarray    # fp32 [2I, ng]
    down_q: np.ndarray  # int8 [H, I]
    down_s: np.ndarray  # fp32 [H, ng_d]
    x: np.ndarray       # fp32 [M, H]


def mlp_case(H, I, M=1, *, seed=0, group_size=None, std=0.02, recipe="f32") -> MlpCase:
    """gate, up, down, then x from one rng. Layer l of the Qwen3-0.6B MLP body
    workload is ``mlp_case(1024, 3072, seed=1000 + l)``."""
    rng = np.random.default_rng(seed)
    gq, gs = quantize_symmetric(draw_weight(rng, (I, H), std, recipe), group_size)
    uq, us = quantize_symmetric(draw_weight(rng, (I, H), std, recipe), group_size)
    dq, ds = quantize_symmetric(draw_weight(rng, (H, I), std, recipe), group_size)
    x = draw_act(rng, (M, H), recipe)
    gu_q, gu_s = stack_gate_up(gq, gs, uq, us)
    return MlpCase(gu_q, gu_s, dq, ds, x)


def gemv_algorithmic_bytes(N, K, ng=1, M=1) -> int:
    """int8 weights + fp32 scales + fp32 activations in + fp32 outputs, each once."""
    return N * K + 4 * N * ng + 4 * M * K + 4 * M * N


def mlp_algorithmic_bytes(H, I, ng=1, ngd=1, M=1) -> int:
    """gate|up and down int8 + their scales + x in + out; the [I] intermediate
    stays on chip/L2 and is not counted."""
    return 2 * I * H + H * I + 4 * (2 * I * ng + H * ngd) + 4 * M * H * 2


# ---------------------------------------------------------------------------
# Command line: run ONE workload on cuda:0 and exit, so that a profiler can
# capture exactly its launches.
#
#   python -m quartz_b200.workloads gemm M N K      tensor-core GEMM, 3 calls
#   python -m quartz_b200.workloads mlp             28-layer fused MLP body, once
#   python -m quartz_b200.workloads lm4             lm_head GEMV, 3 int8 then 3 int4
#                                                   calls on one N(0, 0.02) draw
#   python -m quartz_b200.workloads decode [--persistent] [--tokens T]
#                                                   Qwen3-0.6B, 512 prefilled KV
#                                                   positions, T eager tokens
#   python -m quartz_b200.workloads decode8b [--tokens T]
#                                                   Qwen3-8B shapes, context 2048
#   python -m quartz_b200.workloads batch8b --batch B [--tokens T]
#                                                   Qwen3-8B shapes, B sequences
#                                                   in lockstep, context 2048
#   python -m quartz_b200.workloads mlp8b           one Qwen3-8B fused MLP layer
#                                                   (H 4096, I 12288), 3 calls
#   python -m quartz_b200.workloads attn8b [--batch B]
#                                                   decode attention, Qwen3-8B
#                                                   heads, context 2048, B
#                                                   sequences, 3 calls
#   python -m quartz_b200.workloads prefill         Llama-3.2-1B 512-token prefill
#
# --profile-last (decode, decode8b, batch8b, mlp8b, attn8b): the last token /
# call runs between cudaProfilerStart and cudaProfilerStop, for a profiler run
# with --profile-from-start off.
# ---------------------------------------------------------------------------
def _main(argv=None) -> None:
    import argparse

    import torch

    ap = argparse.ArgumentParser(prog="python -m quartz_b200.workloads")
    sub = ap.add_subparsers(dest="what", required=True)
    g = sub.add_parser("gemm")
    g.add_argument("M", type=int)
    g.add_argument("N", type=int)
    g.add_argument("K", type=int)
    sub.add_parser("mlp")
    sub.add_parser("lm4")
    d = sub.add_parser("decode")
    d.add_argument("--persistent", action="store_true")
    d.add_argument("--tokens", type=int, default=3)
    d8 = sub.add_parser("decode8b")
    d8.add_argument("--tokens", type=int, default=3)
    b8 = sub.add_parser("batch8b")
    b8.add_argument("--batch", type=int, default=16)
    b8.add_argument("--tokens", type=int, default=3)
    sub.add_parser("mlp8b")
    a8 = sub.add_parser("attn8b")
    a8.add_argument("--batch", type=int, default=1)
    sub.add_parser("prefill")
    for p_ in (d, d8, b8):
        p_.add_argument("--profile-last", action="store_true")
    a, rest = ap.parse_known_args(argv)
    a.profile_last = getattr(a, "profile_last", False) or "--profile-last" in rest
    dev = torch.device("cuda", 0)
    from . import device as qd
    qd.ensure_device(dev)

    def profiled(fn):
        """Run fn once more, inside the profiler range when asked."""
        torch.cuda.synchronize()
        if a.profile_last:
            torch.cuda.profiler.start()
        r = fn()
        torch.cuda.synchronize()
        if a.profile_last:
            torch.cuda.profiler.stop()
        return r
    if a.what == "gemm":
        c = gemv_case(a.N, a.K, M=a.M, seed=0)
        q, s = torch.from_numpy(c.q).to(dev), torch.from_numpy(c.scale).to(dev)
        X = torch.from_numpy(c.x).to(dev)
        for _ in range(3):
            Y = qd.gemm(q, s, X)
        torch.cuda.synchronize()
        print(f"gemm {a.M}x{a.N}x{a.K}: |Y|max {float(Y.abs().max()):.4g}")
    elif a.what == "lm4":
        from .quantize import quantize_symmetric, quantize_symmetric_int4
        rng = np.random.default_rng(0)
        W = rng.standard_normal((LM_HEAD_N, LM_HEAD_K), dtype=np.float32) * np.float32(0.02)
        (q8, s8), (q4, s4) = quantize_symmetric(W), quantize_symmetric_int4(W)
        x = torch.from_numpy(rng.standard_normal(LM_HEAD_K, dtype=np.float32)).to(dev)
        t = lambda v: torch.from_numpy(v).to(dev)  # noqa: E731
        q8d, s8d, q4d, s4d = t(q8), t(s8), t(q4), t(s4)
        for _ in range(3):
            y8 = qd.gemv(q8d, s8d, x)
        for _ in range(3):
            y4 = qd.gemv_w4(q4d, s4d, x)
        torch.cuda.synchronize()
        print(f"lm4: |y8|max {float(y8.abs().max()):.4g}, |y4|max {float(y4.abs().max()):.4g}")
    elif a.what == "mlp8b":
        gen = torch.Generator(device=dev)
        gen.manual_seed(5)
        H, I = 4096, 12288
        gq = torch.randint(-127, 128, (2 * I, H), dtype=torch.int8, device=dev, generator=gen)
        dq = torch.randint(-127, 128, (H, I), dtype=torch.int8, device=dev, generator=gen)
        gs = torch.rand(2 * I, 1, device=dev, generator=gen) * 1e-3
        ds = torch.rand(H, 1, device=dev, generator=gen) * 1e-3
        x = torch.randn(H, device=dev, generator=gen)
        for _ in range(2):
            out = qd.fused_mlp(gq, gs, x, dq, ds)
        out = profiled(lambda: qd.fused_mlp(gq, gs, x, dq, ds))
        print(f"mlp8b: |out|max {float(out.abs().max()):.4g}")
    elif a.what == "attn8b":
        import ctypes
        from . import _lib
        from .model import QWEN3_8B, rope_inv_freq
        S8, B, T, C = QWEN3_8B, a.batch, 2048, 2112
        gen = torch.Generator(device=dev)
        gen.manual_seed(6)
        kc = torch.randn(B, S8.n_kv, C, S8.head_dim, device=dev, generator=gen)
        vc = torch.randn(B, S8.n_kv, C, S8.head_dim, device=dev, generator=gen)
        qkv = torch.randn(B, S8.qkv_rows, device=dev, generator=gen)
        out = torch.empty(B, S8.n_heads * S8.head_dim, device=dev)
        inv = torch.from_numpy(rope_inv_freq(S8)).to(dev)
        qn = torch.ones(S8.head_dim, device=dev)
        pos = torch.tensor([T], dtype=torch.int64, device=dev)
        lib = _lib.load()
        nb = ctypes.c_int64(0)
        _lib.check(lib.qz_attention_decode_batch_workspace_bytes(
            B, S8.n_heads, S8.n_kv, S8.head_dim, C, ctypes.byref(nb)))
        ws = torch.zeros(nb.value, dtype=torch.uint8, device=dev)

        def attn():
            _lib.check(lib.qz_attention_decode_qkv_batch(
                qkv.data_ptr(), S8.qkv_rows, qn.data_ptr(), qn.data_ptr(), inv.data_ptr(),
                kc.data_ptr(), vc.data_ptr(), S8.n_kv * C * S8.head_dim, out.data_ptr(),
                S8.n_heads * S8.head_dim, B, S8.n_heads, S8.n_kv, S8.head_dim, C, 0,
                pos.data_ptr(), S8.eps, S8.head_dim ** -0.5, ws.data_ptr(), ws.numel(),
                torch.cuda.current_stream(dev).cuda_stream))
            return out
        for _ in range(2):
            attn()
        o = profiled(attn)
        print(f"attn8b (batch {B}): |out|max {float(o.abs().max()):.4g}")
    elif a.what == "mlp":
        for l in range(MLP_LAYERS):
            m = mlp_case(MLP_H, MLP_I, seed=MLP_LAYER_SEED0 + l)
            t = [torch.from_numpy(v).to(dev) for v in (m.gu_q, m.gu_s, m.x[0], m.down_q, m.down_s)]
            out = qd.fused_mlp(*t)
        torch.cuda.synchronize()
        print(f"mlp body: |out|max {float(out.abs().max()):.4g}")
    else:
        from .decode import DecodeEngine
        from .model import LLAMA_3P2_1B, QWEN3_0P6B, norm_weights, random_int8_weights, seeded_kv
        if a.what == "decode":
            spec = QWEN3_0P6B
            eng = DecodeEngine(spec, random_int8_weights(spec), norm_weights(spec), max_ctx=640,
                               max_prefill=1, device=dev, persistent=a.persistent)
            eng.load_kv(seeded_kv(spec, 512))
            toks = eng.generate(42, a.tokens - 1, graph=False)
            toks.append(profiled(lambda: eng.decode(toks[-1])))
            print(f"decode ({'persistent' if eng.persistent else 'per-op'}): {toks}")
        elif a.what in ("decode8b", "batch8b"):
            # Qwen3-8B shapes on one GPU, device-drawn weights and caches, context 2048
            from .model import QWEN3_8B
            from .tp_decode import random_tp_shard
            B = a.batch if a.what == "batch8b" else 1
            local, w, (lq, ls, _, _) = random_tp_shard(QWEN3_8B, 0, 1, dev)
            eng = DecodeEngine(local, w, norm_weights(QWEN3_8B), max_ctx=2048 + a.tokens,
                               max_prefill=1, device=dev, batch=B)
            del w
            eng.lm_q, eng.lm_s = lq, ls
            eng.k_cache.normal_()
            eng.v_cache.normal_()
            eng.reset(2048)
            if B == 1:
                toks = eng.generate(7, a.tokens - 1, graph=False)
                toks.append(profiled(lambda: eng.decode(toks[-1])))
            else:
                firsts = [(7 + 7919 * b) % QWEN3_8B.vocab for b in range(B)]
                toks = eng.generate_batch(firsts, a.tokens - 1, graph=False)

                def last_step():
                    eng._decode_ops_batch(eng._stream())
                    eng.pos += 1
                    return eng.tok.tolist()
                toks.append(profiled(last_step))
            print(f"{a.what}: {toks[-1]}")
        else:
            spec = LLAMA_3P2_1B
            eng = DecodeEngine(spec, random_int8_weights(spec), norm_weights(spec), max_ctx=600,
                               max_prefill=512, device=dev)
            ids = np.random.default_rng(7).integers(0, spec.vocab, 512).tolist()
            print(f"prefill: first token {eng.prefill(ids)}")
        torch.cuda.synchronize()
    qd.check_status(dev)


if __name__ == "__main__":
    _main()
