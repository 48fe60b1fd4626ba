"""Benchmark of the int8 weight-only path on B200.

Default workload (the one the headline metric is quoted on): the standalone
fused int8 GEMV at the Qwen3-0.6B lm_head shape -- q int8 [151936, 1024] from
per-row absmax quantisation of N(0, 0.02) fp32 draws (seed 0), x fp32 [1024]
~ N(0, 1), y = scale * (q . x) fp32 [151936].

A step is one GEMV over the whole lm_head. Steps rotate over several copies of
the weights (each 155.6 MB, larger than the 126 MB L2) so no step reads weights
the previous step left in L2.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Prints one JSON line. `value` is the device-timed whole-job HBM GB/s of
algorithmic bytes (int8 weights + fp32 scales + x + y, each once); `e2e` is the
same metric through the public numpy API (host x in, host y out, copies
included); `cpu_baseline` is the CPU oracle (a C/OpenMP restatement of the
reference's Numba kernel) on this host's cores.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

from quartz_b200.workloads import (LM_HEAD_K, LM_HEAD_N, MLP_H, MLP_I, MLP_LAYER_SEED0,  # noqa: E402
                                   MLP_LAYERS, gemv_algorithmic_bytes, gemv_case,
                                   mlp_algorithmic_bytes, mlp_case)

METRIC = "int8 GEMV achieved HBM GB/s (% of B200 peak); all-int8 decode tok/s"
UNIT = "GB/s"
WORKLOAD = "qwen3-0.6b lm_head int8 GEMV [151936x1024], M=1, per-row scale"


def bench_config(world: int, copies: int) -> dict:
    """The workload description both arms print (identical by construction)."""
    return {"workload": WORKLOAD, "seed": 0, "weight_copies": copies,
            "l2": f"inputs larger than L2: {copies} rotating weight copies of "
                  f"{LM_HEAD_N * LM_HEAD_K / 1e6:.1f} MB",
            "bytes_per_step_per_gpu": gemv_algorithmic_bytes(LM_HEAD_N, LM_HEAD_K),
            "parallelism": "replicas (one lm_head GEMV stream per GPU)" if world > 1
            else "single GPU"}


def _peaks():
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def _cpu_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# ---------------------------------------------------------------------------
# clocks sampled while the timed region runs
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int, period_ms: int = 20):
        self.gpu = gpu_index
        self.period = period_ms
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"qz_clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", f"-lms", str(self.period)],
                stdout=self.f, stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.1)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.f.close()

    def summary(self) -> dict:
        if self.proc is None or not self.path.exists():
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in self.path.read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append(dict(sm=float(parts[1]), smax=float(parts[2]),
                                 power=float(parts[3]) if parts[3] not in ("[N/A]", "") else None,
                                 hw=parts[5], hwt=parts[6], swt=parts[7], swp=parts[8]))
            except ValueError:
                continue
        try:
            self.path.unlink()
        except OSError:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        reasons = set()
        for r in rows:
            if r["hw"] == "Active":
                reasons.add("hw_slowdown")
            if r["hwt"] == "Active":
                reasons.add("hw_thermal_slowdown")
            if r["swt"] == "Active":
                reasons.add("sw_thermal_slowdown")
            if r["swp"] == "Active":
                reasons.add("sw_power_cap")
        powers = [r["power"] for r in rows if r["power"] is not None]
        return {"sm_mhz": statistics.median(r["sm"] for r in rows),
                "sm_max_mhz": max(r["smax"] for r in rows),
                "reasons": sorted(reasons),
                "samples": len(rows),
                "power_w_max": max(powers) if powers else None}


# ---------------------------------------------------------------------------
# CPU side (oracle = C/OpenMP restatement of quartz/kernels/int8.py:24-38)
# ---------------------------------------------------------------------------
def cpu_gemv_gbs(case, reps: int, threads: int | None = None):
    import oracle
    if threads:
        oracle.set_threads(threads)
    y = np.empty(case.q.shape[0], np.float32)
    x = np.ascontiguousarray(case.x[0])
    oracle.w8a32_gemv(case.q, case.scale, x, y)          # warm
    ts = []
    for _ in range(reps):
        t0 = time.perf_counter()
        oracle.w8a32_gemv(case.q, case.scale, x, y)
        ts.append(time.perf_counter() - t0)
    nbytes = gemv_algorithmic_bytes(*case.q.shape, case.scale.shape[1])
    med = statistics.median(ts)
    return nbytes / med / 1e9, med, oracle.threads(), oracle.load().isa


def run_reference(args) -> dict:
    """--impl reference: the CPU oracle on all host threads, K timed steps."""
    case = gemv_case(LM_HEAD_N, LM_HEAD_K, seed=0)
    import oracle
    oracle.set_threads(_cpu_cores())
    y = np.empty(LM_HEAD_N, np.float32)
    x = np.ascontiguousarray(case.x[0])
    for _ in range(args.warmup):
        oracle.w8a32_gemv(case.q, case.scale, x, y)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.w8a32_gemv(case.q, case.scale, x, y)
    dt = (time.perf_counter() - t0) / max(1, args.steps)
    nbytes = gemv_algorithmic_bytes(LM_HEAD_N, LM_HEAD_K)
    gbs = nbytes / dt / 1e9
    return {
        "metric": METRIC, "value": round(gbs, 3), "unit": UNIT, "impl": "reference",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt * 1e3, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "int8 weights, fp32 accumulate", "data": "synthetic",
        "config": bench_config(args.gpus, args.copies),
        "cpu_baseline": {"value": round(gbs, 3), "unit": UNIT, "cores": oracle.threads(),
                         "kind": "port",
                         "sample": f"full lm_head GEMV per step, {args.steps} steps "
                                   f"({oracle.load().isa})"},
        "e2e": {"value": round(gbs, 3), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


# ---------------------------------------------------------------------------
# GPU side
# ---------------------------------------------------------------------------
def run_gemv_int4(args, dev, world: int = 1) -> dict:
    """The lm_head GEMV on int4 weights (two per byte, per-row scale; quartz has
    no 4-bit kernel, so this line has no reference arm): the same Qwen3-0.6B
    lm_head shape and x as the headline, weights quantised from the same fp32
    draw, 3 rotating copies of 77.8 MB (> L2) in one CUDA graph."""
    import torch
    from quartz_b200 import device as qdev
    from quartz_b200.quantize import quantize_symmetric_int4
    import oracle

    N, K = LM_HEAD_N, LM_HEAD_K
    rng = np.random.default_rng(0)
    W = rng.standard_normal((N, K), dtype=np.float32) * np.float32(0.02)
    q4, s4 = quantize_symmetric_int4(W, None)
    del W
    x = rng.standard_normal(K, dtype=np.float32)
    copies = 3
    qs = [torch.from_numpy(q4).to(dev) for _ in range(copies)]
    sd = torch.from_numpy(s4).to(dev)
    xd = torch.from_numpy(x).to(dev)
    ys = [torch.empty(N, dtype=torch.float32, device=dev) for _ in range(copies)]
    qdev.gemv_w4(qs[0], sd, xd, ys[0])
    torch.cuda.synchronize()
    ref = np.empty(N, np.float32)
    oracle.w4a32_gemv(q4, s4, x, ref)
    rel = float(np.abs(ys[0].cpu().numpy() - ref).max() / np.abs(ref).max())
    if rel > 1e-4:
        raise SystemExit(f"int4 GEMV parity failed: rel err {rel:.3e}")
    chunk = 240
    stream = torch.cuda.current_stream()
    side = torch.cuda.Stream()
    side.wait_stream(stream)
    with torch.cuda.stream(side):
        qdev.gemv_w4(qs[1], sd, xd, ys[1])
    stream.wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for i in range(chunk):
            qdev.gemv_w4(qs[i % copies], sd, xd, ys[i % copies])
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    reps = max(2, args.steps // (chunk * 2))
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    _barrier(world)
    e0.record(stream)
    for _ in range(reps):
        g.replay()
    e1.record(stream)
    _barrier(world)
    qdev.check_status(dev)
    ms = _dist_max(e0.elapsed_time(e1) / (reps * chunk), world)
    nbytes = N * K // 2 + 4 * N + 4 * K + 4 * N
    peak, peak_kind = _peaks()
    achieved = nbytes / (ms * 1e-3) / 1e9
    del g
    return {"workload": "qwen3-0.6b lm_head GEMV [151936x1024] on int4 weights (packed two per "
                        "byte, per-row scale), M=1", "value": round(world * achieved, 1),
            "unit": UNIT, "us_per_gemv": round(ms * 1e3, 3), "steps": reps * chunk,
            "bytes_per_gemv": nbytes, "weights_per_s": round(N * K / (ms * 1e-3), 1),
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": UNIT, "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "per": "one GPU"},
            "gpu_launches": reps * chunk}


def run_mlp_body(args, dev, world: int = 1, do_cpu: bool = True) -> dict:
    """Fused int8 MLP body at Qwen3-0.6B shape, M = 1: one step runs the 28
    independently seeded layers (seed 1000 + l) back to back, each on its own
    x, as one CUDA graph. 28 x 9.47 MB of weights per step (> L2)."""
    import torch
    from quartz_b200 import device as qdev
    import oracle

    layers = [mlp_case(MLP_H, MLP_I, seed=MLP_LAYER_SEED0 + l) for l in range(MLP_LAYERS)]
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)  # noqa: E731
    W = [(t(m.gu_q), t(m.gu_s), t(m.down_q), t(m.down_s)) for m in layers]
    X = [t(m.x[0]) for m in layers]
    A = [torch.empty(MLP_I, dtype=torch.float32, device=dev) for _ in layers]
    O = [torch.empty(MLP_H, dtype=torch.float32, device=dev) for _ in layers]

    def step():
        for l in range(MLP_LAYERS):
            gq, gs, dq, ds = W[l]
            qdev.fused_mlp(gq, gs, X[l], dq, ds, A[l], O[l])

    # parity gate: layer 0 and 27 against the oracle
    step()
    torch.cuda.synchronize()
    for l in (0, MLP_LAYERS - 1):
        m = layers[l]
        ref = np.empty(MLP_H, np.float32)
        oracle.fused_mlp_decode(m.gu_q, m.gu_s, m.x[0], m.down_q, m.down_s,
                                np.empty(MLP_I, np.float32), ref)
        rel = float(np.abs(O[l].cpu().numpy() - ref).max() / np.abs(ref).max())
        if rel > 1e-4:
            raise SystemExit(f"mlp parity failed on layer {l}: rel err {rel:.3e}")
    stream = torch.cuda.current_stream()
    g = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(stream)
    with torch.cuda.stream(s):
        step()
    stream.wait_stream(s)
    torch.cuda.synchronize()
    with torch.cuda.graph(g):
        step()
    for _ in range(max(3, args.warmup // 10)):
        g.replay()
    torch.cuda.synchronize()
    steps = max(10, args.steps // 20)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    _barrier(world)
    e0.record(stream)
    for _ in range(steps):
        g.replay()
    e1.record(stream)
    _barrier(world)
    qdev.check_status(dev)
    ms = _dist_max(e0.elapsed_time(e1) / steps, world)
    per_layer = mlp_algorithmic_bytes(MLP_H, MLP_I)
    gbs = world * per_layer * MLP_LAYERS / (ms * 1e-3) / 1e9
    out = {"workload": "qwen3-0.6b MLP body, 28 fused int8 MLP layers (H=1024, I=3072), M=1",
           "value": round(gbs, 1), "unit": UNIT, "us_per_layer": round(ms * 1e3 / MLP_LAYERS, 3),
           "steps": steps, "bytes_per_layer": per_layer, "gpu_launches": steps * MLP_LAYERS}
    if do_cpu:
        oracle.set_threads(_cpu_cores())
        abuf = np.empty(MLP_I, np.float32)
        o = np.empty(MLP_H, np.float32)
        ts = []
        for _ in range(5):
            t0 = time.perf_counter()
            for m in layers:
                oracle.fused_mlp_decode(m.gu_q, m.gu_s, m.x[0], m.down_q, m.down_s, abuf, o)
            ts.append(time.perf_counter() - t0)
        cm = statistics.median(ts)
        out["cpu_baseline"] = {"value": round(per_layer * MLP_LAYERS / cm / 1e9, 2), "unit": UNIT,
                               "cores": oracle.threads(), "kind": "port",
                               "sample": f"28 layers, median of 5 passes "
                                         f"({cm / MLP_LAYERS * 1e6:.1f} us per layer)"}
    del g
    return out


DECODE_KV, DECODE_FIRST, DECODE_TOKENS, DECODE_UNROLL = 512, 42, 128, 16


def run_decode(args, dev, world: int = 1) -> dict:
    """All-int8 Qwen3-0.6B greedy decode on one GPU per rank (replicas): the
    KV cache prefilled with 512 seeded N(0, 1) positions, 128 greedy tokens
    from token 42, each token one pass of DecodeEngine's device step
    (embedding, 28 layers, lm_head, argmax) replayed from CUDA graphs of 16
    tokens. Weights are the seeded synthetic checkpoint (0.598 GB of int8
    weights and scales per token, > L2); the tokens must equal the ones quartz
    produced on the same checkpoint before anything is timed. Two device
    paths are timed: per-op launches (the engine's default, the headline) and
    the one-launch persistent decode-layers kernel."""
    import torch
    from quartz_b200 import device as qdev
    from quartz_b200.decode import DecodeEngine
    from quartz_b200.model import QWEN3_0P6B, norm_weights, random_int8_weights, seeded_kv

    spec = QWEN3_0P6B
    weights = list(random_int8_weights(spec))
    kv = list(seeded_kv(spec, DECODE_KV))
    with np.load(REPO / "tests" / "golden" / "golden_model.npz") as z:
        gold = z["qwen3_0p6b_kv512__tokens"].tolist()
    stream = torch.cuda.current_stream()
    nrep = DECODE_TOKENS // DECODE_UNROLL
    passes = max(3, min(20, args.steps // 200))

    def measure(persistent: bool):
        eng = DecodeEngine(spec, weights, norm_weights(spec), max_ctx=DECODE_KV + DECODE_TOKENS,
                           max_prefill=1, device=dev, persistent=persistent)
        eng.load_kv(kv)
        toks = eng.generate(DECODE_FIRST, DECODE_TOKENS, graph=True, unroll=DECODE_UNROLL)
        if toks != gold:
            bad = next(i for i, (x, y) in enumerate(zip(toks, gold)) if x != y)
            raise SystemExit(f"decode parity failed at token {bad}: {toks[bad]} != {gold[bad]}")

        def one_pass():
            eng.reset(DECODE_KV)
            eng.tok.fill_(DECODE_FIRST)
            for _ in range(nrep):
                eng.replay()

        for _ in range(2):
            one_pass()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        _barrier(world)
        e0.record(stream)
        for _ in range(passes):
            one_pass()
        e1.record(stream)
        _barrier(world)
        qdev.check_status(dev)
        ms_tok = _dist_max(e0.elapsed_time(e1) / (passes * DECODE_TOKENS), world)
        # e2e through generate(): first token in from the host, the token list out
        t0 = time.perf_counter()
        for _ in range(passes):
            eng.reset(DECODE_KV)
            eng.generate(DECODE_FIRST, DECODE_TOKENS, graph=True, unroll=DECODE_UNROLL)
        e2e_ms = _dist_max((time.perf_counter() - t0) * 1e3 / (passes * DECODE_TOKENS), world)
        launches = eng._launches_per_token()
        del eng
        torch.cuda.empty_cache()
        return ms_tok, e2e_ms, launches

    ms_tok, e2e_ms, launches = measure(False)
    ms_p, _, launches_p = measure(True)
    cpu = None
    if world == 1 and not args.no_cpu:
        # the oracle's CPU decode port (numpy glue + the C/OpenMP restatement of
        # quartz's int8 kernels) on a bounded sample: 8 tokens after the 512
        # prefilled positions, all host cores
        import oracle
        from oracle.decode_port import DecodePort
        cfg = dict(hidden_size=spec.hidden, num_hidden_layers=spec.layers,
                   num_attention_heads=spec.n_heads, num_key_value_heads=spec.n_kv,
                   head_dim=spec.head_dim, intermediate_size=spec.inter, vocab_size=spec.vocab,
                   rope_theta=spec.rope_theta, tie_word_embeddings=spec.tie, rms_norm_eps=spec.eps)
        oracle.set_threads(_cpu_cores())
        port = DecodePort(cfg, spec.arch, dict((n, (q, s_)) for n, q, s_ in weights),
                          norm_weights(spec), max_ctx=DECODE_KV + 8)
        port.load_kv(kv)
        tok = port.step(DECODE_FIRST)          # warm-up (first-touch of the weights)
        t0 = time.perf_counter()
        toks = []
        for _ in range(7):
            tok = port.step(tok)
            toks.append(tok)
        dt = (time.perf_counter() - t0) / 7
        if toks != gold[1:8]:
            raise SystemExit("CPU decode port disagrees with the reference tokens")
        cpu = {"value": round(1.0 / dt, 2), "unit": "tok/s", "cores": oracle.threads(),
               "kind": "port", "sample": "7 greedy tokens after the 512 prefilled positions "
                                        f"({dt * 1e3:.1f} ms per token)"}
    wbytes = spec.int8_bytes_per_token()
    ctx_mean = DECODE_KV + (DECODE_TOKENS + 1) / 2
    kvbytes = spec.kv_bytes_per_token(int(round(ctx_mean)))
    peak, peak_kind = _peaks()
    achieved = (wbytes + kvbytes) / (ms_tok * 1e-3) / 1e9
    return {"workload": "qwen3-0.6b all-int8 greedy decode, 512 prefilled KV positions, "
                        "128 tokens, CUDA-graph replay (16 tokens per graph)",
            "value": round(world / (ms_tok * 1e-3), 1), "unit": "tok/s",
            "us_per_token": round(ms_tok * 1e3, 2), "passes": passes,
            "tokens_match_reference": True,
            "bytes_per_token": {"int8_weights_and_scales": wbytes, "kv_cache_mean": kvbytes},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": UNIT, "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "per": "one GPU"},
            "e2e": {"value": round(world / (e2e_ms * 1e-3), 1), "unit": "tok/s",
                    "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 8 * DECODE_TOKENS,
                    "note": "DecodeEngine.generate per 128-token pass (first token in, "
                            "token list out)"},
            "cpu_baseline": cpu,
            "persistent_kernel": {"value": round(world / (ms_p * 1e-3), 1), "unit": "tok/s",
                                  "us_per_token": round(ms_p * 1e3, 2),
                                  "launches_per_token": launches_p},
            "gpu_launches": passes * DECODE_TOKENS * launches,
            "parallelism": "replicas (one sequence per GPU)" if world > 1 else "single GPU"}


LLAMA_PROMPT, LLAMA_TOKENS = 512, 256


def run_llama_prefill_decode(args, dev) -> dict:
    """Llama-3.2-1B architecture (16 layers, hidden 2048, 32 query / 8 kv heads,
    head_dim 64, MLP 8192, tied vocab 128256, llama3 RoPE), all-int8 synthetic
    checkpoint: a 512-token prefill (seeded prompt ids, default_rng(7)), then
    256 greedy tokens -- the reference's time_decode recipe (bench/decode.py:
    26-40) on the device engine. The 256 tokens must equal quartz's own before
    anything is timed. Prefill: CUDA-event time of one prefill pass (tensor-core
    int8 GEMMs at M = 512, causal attention); decode: the 256 tokens from CUDA
    graphs of 16. CPU: the oracle's decode port at context 512 and the oracle's
    int8 GEMM on one layer's prefill shapes (M = 512), all host cores."""
    import torch
    import oracle
    from oracle.decode_port import DecodePort
    from quartz_b200 import device as qdev
    from quartz_b200.decode import DecodeEngine
    from quartz_b200.model import LLAMA_3P2_1B, cached_int8_weights, norm_weights, seeded_kv
    spec = LLAMA_3P2_1B
    with np.load(REPO / "tests" / "golden" / "golden_model.npz") as z:
        gold = z["llama_1b_prompt512__tokens"].tolist()
    if len(gold) < LLAMA_TOKENS:
        raise SystemExit("the Llama-1B golden fixture holds fewer than 256 tokens")
    prompt = np.random.default_rng(7).integers(0, spec.vocab, LLAMA_PROMPT).tolist()
    weights = cached_int8_weights(spec)
    eng = DecodeEngine(spec, weights, norm_weights(spec), max_ctx=LLAMA_PROMPT + LLAMA_TOKENS,
                       max_prefill=LLAMA_PROMPT, device=dev)
    stream = torch.cuda.current_stream()

    def run_once():
        eng.reset(0)
        t0 = eng.prefill(prompt)
        return [t0] + eng.generate(t0, LLAMA_TOKENS - 1, graph=True, unroll=16)

    toks = run_once()
    if toks != gold[:LLAMA_TOKENS]:
        bad = next(i for i, (x, y) in enumerate(zip(toks, gold)) if x != y)
        raise SystemExit(f"Llama-1B parity failed at token {bad}: {toks[bad]} != {gold[bad]}")
    reps = 3
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    pre = []
    for _ in range(reps):                        # prefill alone, device time
        eng.reset(0)
        torch.cuda.synchronize()
        e0.record(stream)
        eng.prefill(prompt)
        e1.record(stream)
        torch.cuda.synchronize()
        pre.append(e0.elapsed_time(e1))
    pre_ms = statistics.median(pre)
    dec = []
    for _ in range(reps):                        # the 255 graph-replayed tokens after it
        eng.reset(0)
        t0 = eng.prefill(prompt)
        torch.cuda.synchronize()
        e0.record(stream)
        eng.tok.fill_(t0)
        eng.pos_dev.fill_(eng.pos)
        n = 0
        while n + 16 <= LLAMA_TOKENS - 1:
            eng.replay()
            n += 16
        e1.record(stream)
        torch.cuda.synchronize()
        dec.append(e0.elapsed_time(e1) / n)
    ms_tok = statistics.median(dec)
    # end to end through the public calls: prompt ids in, the token list out
    t0 = time.perf_counter()
    for _ in range(reps):
        run_once()
    e2e_s = (time.perf_counter() - t0) / reps
    qdev.check_status(dev)
    launches = eng._launches_per_token()
    del eng
    torch.cuda.empty_cache()
    # prefill FLOPs: the int8 linears at M = 512 (2 flops per MAC) + causal attention
    H, I, hd = spec.hidden, spec.inter, spec.head_dim
    lin = 2 * LLAMA_PROMPT * spec.layers * (spec.qkv_rows * H + H * spec.n_heads * hd
                                            + 2 * I * H + H * I)
    att = 2 * 2 * spec.layers * spec.n_heads * hd * LLAMA_PROMPT * (LLAMA_PROMPT + 1) // 2
    peak_int8 = 2 * _bf16_peak()            # int8 dense = 2x the measured bf16 GEMM rate
    # each fp32 activation is three int8 limbs on the tensor cores: 3 int8 MACs per MAC
    int8_tops = 3 * lin / (pre_ms * 1e-3) / 1e12
    wbytes = spec.int8_bytes_per_token()
    kv_mean = spec.kv_bytes_per_token(LLAMA_PROMPT + LLAMA_TOKENS // 2)
    peak, peak_kind = _peaks()
    achieved = (wbytes + kv_mean) / (ms_tok * 1e-3) / 1e9
    cpu = None
    if not args.no_cpu:
        oracle.set_threads(_cpu_cores())
        cfg = dict(hidden_size=H, num_hidden_layers=spec.layers, num_attention_heads=spec.n_heads,
                   num_key_value_heads=spec.n_kv, head_dim=hd, intermediate_size=I,
                   vocab_size=spec.vocab, rope_theta=spec.rope_theta,
                   rope_scaling=spec.rope_scaling, tie_word_embeddings=spec.tie,
                   rms_norm_eps=spec.eps)
        port = DecodePort(cfg, spec.arch, {n: (q, s_) for n, q, s_ in weights},
                          norm_weights(spec), max_ctx=LLAMA_PROMPT + 8)
        port.load_kv(seeded_kv(spec, LLAMA_PROMPT))
        tok = port.step(gold[0])                 # warm-up (first touch of the weights)
        t0 = time.perf_counter()
        for _ in range(4):
            tok = port.step(tok)
        cdt = (time.perf_counter() - t0) / 4
        # prefill: the oracle's int8 GEMM on layer 0's four matmuls at M = 512
        w = {n: (q, s_) for n, q, s_ in weights[:8]}
        X = np.random.default_rng(3).standard_normal((LLAMA_PROMPT, H), dtype=np.float32)
        A = np.random.default_rng(4).standard_normal((LLAMA_PROMPT, I), dtype=np.float32)
        p0 = "model.layers.0."
        qkv_q = np.concatenate([w[p0 + "self_attn." + n][0] for n in ("q_proj", "k_proj", "v_proj")])
        qkv_s = np.concatenate([w[p0 + "self_attn." + n][1] for n in ("q_proj", "k_proj", "v_proj")])
        gu_q = np.concatenate([w[p0 + "mlp.gate_proj"][0], w[p0 + "mlp.up_proj"][0]])
        gu_s = np.concatenate([w[p0 + "mlp.gate_proj"][1], w[p0 + "mlp.up_proj"][1]])
        t0 = time.perf_counter()
        oracle.matmul_int8(qkv_q, qkv_s, X)
        oracle.matmul_int8(*w[p0 + "self_attn.o_proj"], X[:, :spec.n_heads * hd])
        oracle.matmul_int8(gu_q, gu_s, X)
        oracle.matmul_int8(*w[p0 + "mlp.down_proj"], A)
        layer_s = time.perf_counter() - t0
        cpu = {"decode": {"value": round(1.0 / cdt, 2), "unit": "tok/s", "cores": oracle.threads(),
                          "kind": "port", "sample": f"4 greedy tokens at context 512 "
                                                    f"({cdt * 1e3:.1f} ms per token)"},
               "prefill": {"value": round(layer_s * spec.layers * 1e3, 1), "unit": "ms",
                           "cores": oracle.threads(), "kind": "port",
                           "sample": "the int8 GEMMs of 1 of 16 layers at M = 512 "
                                     f"({layer_s * 1e3:.0f} ms), times 16; attention "
                                     "not included"}}
    return {"workload": "llama-3.2-1b all-int8: 512-token prefill then 256 greedy tokens "
                        "(CUDA-graph replay, 16 tokens per graph)",
            "tokens_match_reference": True,
            "prefill": {"ms": round(pre_ms, 3), "tokens": LLAMA_PROMPT,
                        "tok_per_s": round(LLAMA_PROMPT / (pre_ms * 1e-3), 1),
                        "linear_flops": lin, "attention_flops": att,
                        "roofline": {"bound": "tensor",
                                     "achieved": round(int8_tops, 1), "unit": "int8 TOP/s",
                                     "peak": round(peak_int8, 1),
                                     "frac": round(int8_tops / peak_int8, 4),
                                     "peak_kind": "2x measured bf16 GEMM (dense int8 rate)",
                                     "note": "whole prefill time incl. attention, norms and "
                                             "limb splits; 3 int8 MACs per fp32 MAC"}},
            "decode": {"value": round(1.0 / (ms_tok * 1e-3), 1), "unit": "tok/s",
                       "us_per_token": round(ms_tok * 1e3, 2),
                       "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                                    "unit": UNIT, "frac": round(achieved / peak, 4),
                                    "peak_kind": peak_kind,
                                    "bytes_per_token": wbytes + kv_mean}},
            "e2e": {"value": round(LLAMA_TOKENS / e2e_s, 1), "unit": "tok/s",
                    "s_per_request": round(e2e_s, 4), "h2d_bytes_per_step": 8 * LLAMA_PROMPT,
                    "d2h_bytes_per_step": 8 * LLAMA_TOKENS,
                    "note": "prefill(prompt ids) + generate(255): one request, prompt in, "
                            "token list out"},
            "cpu_baseline": cpu,
            "gpu_launches": reps * (launches * (LLAMA_TOKENS - 1))}


BATCH_SIZES = (2, 4, 8, 16)
BATCH_CTX, BATCH_STEPS = 2048, 16


def batch_parity_gate(rank: int, world: int, dev, batch: int) -> dict:
    """The batched tensor-parallel engine at this rank count and batch
    reproduces quartz's batched decode: the Qwen3-0.6B architecture, `batch`
    sequences from seeded [batch, 8, 512, 128] caches, 32 greedy tokens per
    sequence (the reference's tokens); every rank checks, the verdict is
    all-reduced."""
    import torch
    from quartz_b200.model import QWEN3_0P6B, cached_int8_weights, norm_weights, seeded_kv
    from quartz_b200.tp_decode import TPDecodeEngine
    cid = f"qwen3_0p6b_kv512_b{batch}"
    cases = {c["id"]: c for c in json.loads(
        (REPO / "tests" / "golden" / "cases_model.json").read_text())["cases"]}
    case = cases[cid]
    with np.load(REPO / "tests" / "golden" / "golden_model.npz") as z:
        gold = z[f"{cid}__tokens"].tolist()
    spec = QWEN3_0P6B
    eng = TPDecodeEngine(spec, cached_int8_weights(spec), norm_weights(spec),
                         max_ctx=case["kv_len"] + case["steps"], max_prefill=1, device=dev,
                         allreduce="peer", batch=batch)
    eng.load_kv(seeded_kv(spec, case["kv_len"], batch=batch))
    toks = eng.generate_batch(case["firsts"], case["steps"], graph=True, unroll=8)
    eng.close()
    del eng
    torch.cuda.empty_cache()
    if not _all_ranks_ok(toks == gold, world):
        raise SystemExit(f"batched decode parity failed (batch {batch}, {world} ranks, rank {rank})")
    return {"case": cid, "ranks": world, "batch": batch, "tokens_match_reference": True}


def run_batch_decode(args, rank: int, world: int, dev) -> dict:
    """Qwen3-8B all-int8 decode of M sequences in lockstep (M in {2, 4, 8, 16};
    M = 1 is the tensor-parallel decode line), split over the ranks like the
    single-sequence engine (heads, units, vocab rows) with the [M, H] partial
    sums summed by the peer all-reduce kernel: every linear is the int8 GEMM on
    M rows (tensor cores, weights read once per step), attention runs all M
    caches in one launch. Caches hold 2048 random positions per sequence;
    16 steps per CUDA graph. Weights are drawn on the device per shard (timing
    does not depend on the values); each M is first gated on the reference's
    batched tokens at the same rank count (batch_parity_gate). Strong scaling
    over the ranks; per-GPU roofline over the rank's weight share plus its
    share of the M caches."""
    import torch
    from quartz_b200.model import QWEN3_8B, norm_weights
    from quartz_b200.tp_decode import TPDecodeEngine, random_tp_shard
    spec = QWEN3_8B
    stream = torch.cuda.current_stream()
    peak, peak_kind = _peaks()
    out = {"workload": "qwen3-8b all-int8 batched greedy decode, M sequences at context "
                       f"{BATCH_CTX}..{BATCH_CTX + 2 * BATCH_STEPS}, CUDA-graph replay",
           "n_gpus": world, "scaling": "strong", "rows": {}}
    shard = random_tp_shard(spec, rank, world, dev)
    for M in BATCH_SIZES:
        gate = batch_parity_gate(rank, world, dev, M)
        eng = TPDecodeEngine(spec, None, norm_weights(spec),
                             max_ctx=BATCH_CTX + 2 * BATCH_STEPS + 8, max_prefill=1, device=dev,
                             presharded=shard, allreduce="peer", batch=M)
        gen = torch.Generator(device=dev)
        gen.manual_seed(99 + rank)
        for t in (eng.k_cache, eng.v_cache):
            t.normal_(generator=gen)
        eng.reset(BATCH_CTX)
        eng.tok.copy_(torch.arange(M, device=dev) * 7919 % spec.vocab)
        eng.capture(BATCH_STEPS)

        def one_pass():
            eng.reset(BATCH_CTX)
            eng.replay()

        for _ in range(2):
            one_pass()
        torch.cuda.synchronize()
        passes = 3
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        _barrier(world)
        e0.record(stream)
        for _ in range(passes):
            one_pass()
        e1.record(stream)
        _barrier(world)
        ms_step = _dist_max(e0.elapsed_time(e1) / (passes * BATCH_STEPS), world)
        launches = eng._launches_per_token()
        eng.close()
        del eng
        torch.cuda.empty_cache()
        wbytes = spec.int8_bytes_per_token()
        kv = M * spec.kv_bytes_per_token(BATCH_CTX + BATCH_STEPS // 2)
        per_gpu = (wbytes + kv) / world
        achieved = per_gpu / (ms_step * 1e-3) / 1e9
        out["rows"][f"M{M}"] = {
            "value": round(M / (ms_step * 1e-3), 1), "unit": "tok/s",
            "ms_per_step": round(ms_step, 4), "tokens_match_reference": True,
            "parity_gate": gate,
            "bytes_per_step": {"int8_weights_and_scales": wbytes, "kv_cache": kv},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": UNIT, "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "per": "one GPU (its 1/N of the bytes)"},
            "gpu_launches": passes * BATCH_STEPS * launches}
    del shard
    torch.cuda.empty_cache()
    return out


def _bf16_peak() -> float:
    p = REPO / "MEASURED_PEAKS.json"
    if p.exists():
        return float(json.loads(p.read_text())["bf16_tflops"])
    return 1590.0


def _log(rank: int, msg: str) -> None:
    if rank == 0:
        print(f"[bench] {msg}", file=sys.stderr, flush=True)


def _dist_max(value: float, world: int) -> float:
    """Max of a per-rank float over all ranks (identity on one rank)."""
    if world == 1:
        return value
    import torch
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device=torch.device("cuda", torch.cuda.current_device()))
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(world: int) -> None:
    import torch
    if world > 1:
        import torch.distributed as dist
        dist.barrier(device_ids=[torch.cuda.current_device()])
    torch.cuda.synchronize()


def tp_layers_parity(rank: int, world: int, dev, case) -> dict:
    """The sharded MLP and lm_head at this rank count against the oracle
    before the tensor-parallel step is timed: the Qwen3-0.6B MLP layer (H 1024,
    I 3072, seed 1000) at M = 1 (fused kernel, quartz/kernels/fused.py:27-65)
    and M = 16 (per-op path, quartz/quantize.py:112-114), max |err| <= 1e-4 *
    ||y||_inf; the lm_head workload's greedy token at M = 1 and 16 rows, equal
    to the oracle's argmax unless the oracle's top two logits are closer than
    that tolerance. Every rank checks, then the verdict is all-reduced."""
    import torch
    import oracle
    from quartz_b200.sharding import ShardedLMHead, ShardedMLP
    m = mlp_case(MLP_H, MLP_I, M=16, seed=MLP_LAYER_SEED0)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a))  # noqa: E731
    I = MLP_I
    mlp = ShardedMLP(t(m.gu_q[:I]), t(m.gu_s[:I]), t(m.gu_q[I:]), t(m.gu_s[I:]), t(m.down_q),
                     t(m.down_s), device=dev)
    errs = {}
    ref1 = np.empty(MLP_H, np.float32)
    oracle.fused_mlp_decode(m.gu_q, m.gu_s, m.x[0], m.down_q, m.down_s,
                            np.empty(I, np.float32), ref1)
    got1 = mlp(t(m.x[:1]).to(dev)).cpu().numpy()[0]
    errs["mlp_M1"] = float(np.abs(got1 - ref1).max() / np.abs(ref1).max())
    ref16 = oracle.mlp_per_op(m.gu_q, m.gu_s, m.down_q, m.down_s, m.x)
    got16 = mlp(t(m.x).to(dev)).cpu().numpy()
    errs["mlp_M16"] = float(np.abs(got16 - ref16).max() / np.abs(ref16).max())
    head = ShardedLMHead(t(case.q), t(case.scale), device=dev)
    X = np.concatenate([case.x, np.random.default_rng(5).standard_normal(
        (15, case.q.shape[1]), dtype=np.float32)])
    Y = np.empty((16, case.q.shape[0]), np.float32)
    oracle.w8a32_gemm(case.q, case.scale, X, Y)
    toks = head.argmax(t(X).to(dev)).cpu().numpy()
    tol = 1e-4 * np.abs(Y).max(axis=1)
    near = Y[np.arange(16), toks] >= Y.max(axis=1) - tol
    ok = max(errs.values()) <= 1e-4 and bool(near.all())
    del mlp, head
    torch.cuda.empty_cache()
    if not _all_ranks_ok(ok, world):
        raise SystemExit(f"sharded MLP / lm_head parity failed on {world} ranks (rank {rank}): "
                         f"{errs}, argmax within tolerance {near.tolist()}")
    return {"ranks": world, "rel_err": {k: float(f"{v:.3e}") for k, v in errs.items()},
            "argmax_rows_equal": int((toks == Y.argmax(axis=1)).sum()), "argmax_rows": 16,
            "match_oracle": True}


def run_tp(args, rank: int, world: int, dev, case) -> dict:
    """Tensor-parallel Qwen3-8B shapes (hidden 4096, MLP 12288, vocab 151936,
    36 layers): per step, the 36 MLP layers (gate/up column-parallel, down
    row-parallel, all-reduce of the partials) and the vocab-parallel lm_head
    with the greedy (max, index) all-gather. Strong scaling: the whole model's
    int8 weights are split over the ranks. Weights are drawn on the device
    (int8 uniform, fp32 scales): timing does not depend on their values;
    the sharded layers are checked against the oracle first (tp_layers_parity)."""
    import torch
    from quartz_b200.sharding import ShardedLMHead, ShardedMLP, shard_range
    H, I, V, L = 4096, 12288, 151936, 36
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)

    def q_(shape):
        return torch.randint(-127, 128, shape, dtype=torch.int8, device=dev, generator=gen)

    def s_(n):
        return torch.rand((n, 1), device=dev, generator=gen) * 2e-4 + 1e-4

    parity = tp_layers_parity(rank, world, dev, case)
    lo, hi = shard_range(V, world, rank)
    head = ShardedLMHead.from_local(q_((hi - lo, H)), s_(hi - lo), V)
    ulo, uhi = shard_range(I, world, rank)
    layers = [ShardedMLP.from_local(q_((2 * (uhi - ulo), H)), s_(2 * (uhi - ulo)),
                                    q_((H, uhi - ulo)), s_(H), I) for _ in range(L)]
    weight_bytes = V * H + L * 3 * I * H
    out = {"workload": "qwen3-8b shapes: 36 TP MLP layers + vocab-parallel lm_head argmax",
           "n_gpus": world, "scaling": "strong", "weight_bytes": weight_bytes,
           "layers_parity": parity}
    for M in (1, 16):
        x = torch.randn((M, H), device=dev, generator=gen)

        def step():
            for mlp in layers:
                mlp(x)
            return head.argmax(x)

        for _ in range(3):
            step()
        _barrier(world)
        # The whole step -- kernels and NCCL collectives -- as one CUDA graph.
        graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            step()
        torch.cuda.current_stream().wait_stream(side)
        _barrier(world)
        with torch.cuda.graph(graph):
            step()
        _barrier(world)
        for _ in range(3):
            graph.replay()
        _barrier(world)
        steps = 20
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(steps):
            graph.replay()
        t1.record()
        _barrier(world)
        ms = _dist_max(t0.elapsed_time(t1) / steps, world)
        out[f"M{M}"] = {"ms_per_step": round(ms, 4), "tok_per_s": round(M / (ms * 1e-3), 1),
                        "weight_GBs": round(weight_bytes / (ms * 1e-3) / 1e9, 1)}
        del graph      # a graph holding NCCL calls must go before the process group
        torch.cuda.synchronize()
    del layers, head
    torch.cuda.empty_cache()
    out["decode"] = run_tp_decode(args, rank, world, dev)
    return out


TP_CTX, TP_TOKENS, TP_UNROLL = 2048, 64, 16


def _all_ranks_ok(ok: bool, world: int) -> bool:
    """True when every rank passed (one all-reduce, taken by every rank)."""
    if world == 1:
        return ok
    import torch
    import torch.distributed as dist
    t = torch.tensor([1 if ok else 0], dtype=torch.int32,
                     device=torch.device("cuda", torch.cuda.current_device()))
    dist.all_reduce(t, op=dist.ReduceOp.MIN)
    return bool(t.item())


def tp_parity_gate(rank: int, world: int, dev, allreduce: str) -> dict:
    """Greedy tokens of the N-rank TPDecodeEngine against the reference's own
    tokens before anything is timed: the Qwen3-0.6B architecture (16 query / 8
    kv heads, MLP 3072 -- every split up to 8 ranks is whole), the seeded
    synthetic checkpoint, 512 prefilled KV positions, 128 greedy tokens from
    token 42, replayed from CUDA graphs of 16 tokens. Any rank's mismatch
    stops every rank (SystemExit) after a common all-reduce of the verdict."""
    import torch
    from quartz_b200.model import QWEN3_0P6B, cached_int8_weights, norm_weights, seeded_kv
    from quartz_b200.tp_decode import TPDecodeEngine
    spec = QWEN3_0P6B
    with np.load(REPO / "tests" / "golden" / "golden_model.npz") as z:
        gold = z["qwen3_0p6b_kv512__tokens"].tolist()
    eng = TPDecodeEngine(spec, cached_int8_weights(spec), norm_weights(spec),
                         max_ctx=DECODE_KV + DECODE_TOKENS, max_prefill=1, device=dev,
                         allreduce=allreduce)
    eng.load_kv(seeded_kv(spec, DECODE_KV))
    toks = eng.generate(DECODE_FIRST, DECODE_TOKENS, graph=True, unroll=DECODE_UNROLL)
    eng.close()
    del eng
    torch.cuda.empty_cache()
    ok = toks == gold
    if not _all_ranks_ok(ok, world):
        bad = next((i for i, (x, y) in enumerate(zip(toks, gold)) if x != y), None)
        raise SystemExit(f"tensor-parallel decode parity failed ({allreduce}, {world} ranks, "
                         f"rank {rank}): first differing token {bad}")
    return {"case": "qwen3-0.6b architecture, 512 prefilled KV positions, 128 greedy tokens "
                    "from token 42 (the reference's tokens)", "allreduce": allreduce,
            "ranks": world, "tokens_match_reference": True}


def run_tp_decode(args, rank: int, world: int, dev) -> dict:
    """Greedy decode of one Qwen3-8B sequence split over the ranks
    (TPDecodeEngine: head-sharded attention, unit-sharded MLP, vocab-sharded
    lm_head, two all-reduces per layer), at context 2048..2112, 64 tokens per
    pass replayed from CUDA graphs of 16. Weights are drawn on the device per
    shard (timing does not depend on the values). Before each all-reduce form
    is timed, the same engine at the same rank count must reproduce the
    reference's greedy tokens on the Qwen3-0.6B workload (tp_parity_gate)."""
    import torch
    from quartz_b200.model import QWEN3_8B, norm_weights
    from quartz_b200.tp_decode import TPDecodeEngine, random_tp_shard
    spec = QWEN3_8B
    stream = torch.cuda.current_stream()

    gates = []

    def measure(allreduce: str) -> float:
        gates.append(tp_parity_gate(rank, world, dev, allreduce))
        shard = random_tp_shard(spec, rank, world, dev)
        eng = TPDecodeEngine(spec, None, norm_weights(spec), max_ctx=TP_CTX + TP_TOKENS,
                             max_prefill=1, device=dev, presharded=shard, allreduce=allreduce)
        del shard

        def one_pass():
            eng.reset(TP_CTX)
            eng.tok.fill_(7)
            for _ in range(TP_TOKENS // TP_UNROLL):
                eng.replay()

        eng.reset(TP_CTX)
        eng.capture(TP_UNROLL)
        for _ in range(2):
            one_pass()
        torch.cuda.synchronize()
        passes = 3
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        _barrier(world)
        e0.record(stream)
        for _ in range(passes):
            one_pass()
        e1.record(stream)
        _barrier(world)
        ms = _dist_max(e0.elapsed_time(e1) / (passes * TP_TOKENS), world)
        eng.close()          # the graph (it holds collectives) and the peer buffers
        del eng
        torch.cuda.empty_cache()
        return ms

    ms_tok = measure("fused")
    ms_peer = measure("peer") if world > 1 else ms_tok
    ms_nccl = measure("nccl") if world > 1 else ms_tok
    ar_us = allreduce_latency(world, dev, spec.hidden) if world > 1 else None
    wbytes = spec.int8_bytes_per_token()
    kvbytes = spec.kv_bytes_per_token(TP_CTX + TP_TOKENS // 2)
    peak, peak_kind = _peaks()
    per_gpu = (wbytes + kvbytes) / world
    achieved = per_gpu / (ms_tok * 1e-3) / 1e9
    return {"workload": "qwen3-8b all-int8 greedy decode, one sequence over the ranks, context "
                        f"{TP_CTX}..{TP_CTX + TP_TOKENS}, CUDA-graph replay",
            "value": round(1.0 / (ms_tok * 1e-3), 1), "unit": "tok/s",
            "us_per_token": round(ms_tok * 1e3, 1), "n_gpus": world, "scaling": "strong",
            "bytes_per_token": {"int8_weights_and_scales": wbytes, "kv_cache": kvbytes},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "unit": UNIT, "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                         "per": "one GPU (its 1/N of the bytes)"},
            "collectives_per_token": 2 * spec.layers + 1,
            "allreduce": ("in the kernels: GEMV / MLP epilogues push to peer memory, the next "
                          "RMSNorm sums") if world > 1 else "none",
            "with_peer_allreduce_kernel": {"us_per_token": round(ms_peer * 1e3, 1),
                                           "value": round(1.0 / (ms_peer * 1e-3), 1)},
            "with_nccl_allreduce": {"us_per_token": round(ms_nccl * 1e3, 1),
                                    "value": round(1.0 / (ms_nccl * 1e-3), 1)},
            "allreduce_us_per_call": ar_us,
            "tokens_match_reference": all(g["tokens_match_reference"] for g in gates),
            "parity_gates": gates}


def allreduce_latency(world: int, dev, n: int) -> dict:
    """Device time per all-reduce of n fp32 (one decode step's [H] partial):
    200 back-to-back calls in one CUDA graph, max over ranks, for the
    peer-memory kernel and for NCCL."""
    import torch
    import torch.distributed as dist
    from quartz_b200.comm import PeerAllReduce
    ar = PeerAllReduce(n, device=dev)
    t = torch.randn(n, device=dev)
    out = {}
    for name, fn in (("peer_kernel", lambda: ar(t)), ("nccl", lambda: dist.all_reduce(t))):
        for _ in range(5):
            fn()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            with torch.cuda.graph(g, stream=side):
                for _ in range(200):
                    fn()
        torch.cuda.current_stream().wait_stream(side)
        g.replay()
        torch.cuda.synchronize()
        _barrier(world)
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        out[name] = round(_dist_max(e0.elapsed_time(e1) * 1e3 / 200, world), 2)
        del g              # a graph holding NCCL calls goes before the process group
    ar.close()
    return out


def run_ours(args, rank: int, world: int, local: int) -> dict | None:
    import torch
    from quartz_b200 import device as qdev
    from quartz_b200 import kernels as qk

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    qdev.ensure_device(dev)
    qdev.status(clear=True)

    case = gemv_case(LM_HEAD_N, LM_HEAD_K, seed=0)
    N, K = case.q.shape
    nbytes = gemv_algorithmic_bytes(N, K)
    copies = args.copies
    qs = [torch.from_numpy(case.q).to(dev) for _ in range(copies)]
    ss = [torch.from_numpy(case.scale).to(dev) for _ in range(copies)]
    x = torch.from_numpy(case.x[0]).to(dev)
    ys = [torch.empty(N, dtype=torch.float32, device=dev) for _ in range(copies)]

    def step(i):
        j = i % copies
        qdev.gemv(qs[j], ss[j], x, ys[j])

    # correctness gate before timing: copy 0 against the CPU oracle
    import oracle
    y_ref = np.empty(N, np.float32)
    oracle.w8a32_gemv(case.q, case.scale, case.x[0], y_ref)
    step(0)
    torch.cuda.synchronize()
    rel = float(np.abs(ys[0].cpu().numpy() - y_ref).max() / np.abs(y_ref).max())
    if rel > 1e-4:
        raise SystemExit(f"parity check failed before timing on rank {rank}: rel err {rel:.3e}")

    stream = torch.cuda.current_stream()
    use_graph = not args.no_graph
    graphs = []          # (graph, steps it holds); the timed region replays each once per pass
    if use_graph:
        # The K timed steps are whole graph replays: `chunk` steps per graph,
        # the largest divisor of K up to 256, plus one graph for a remainder
        # when K has no divisor of useful size.
        chunk = max(d for d in range(1, min(args.steps, 256) + 1) if args.steps % d == 0)
        if chunk < 32:
            chunk = min(args.steps, 256)
        full, rem = divmod(args.steps, chunk)
        s = torch.cuda.Stream()
        s.wait_stream(stream)
        with torch.cuda.stream(s):
            step(0)
        stream.wait_stream(s)
        torch.cuda.synchronize()
        def copy_of(i, n):
            # weight copy of step i of an n-step graph: round robin, except that
            # a graph never ends on copy 0, which the next replay starts with
            if i == n - 1 and n > 1 and i % copies == 0:
                return 1
            return i % copies

        for n in ([chunk] * (1 if full else 0)) + ([rem] if rem else []):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                for i in range(n):
                    step(copy_of(i, n))
            graphs.append((g, n))
        torch.cuda.synchronize()

    def run(n):
        """n steps exactly as the timed region runs them."""
        if use_graph:
            main_reps, tail = divmod(n, chunk)
            for _ in range(main_reps):
                graphs[0][0].replay()
            if tail:
                graphs[-1][0].replay()
        else:
            for i in range(n):
                step(i)

    # Warm-up runs the timed path itself: every graph the timed region replays
    # is replayed (and so uploaded) at least once, W steps or more in all.
    if use_graph:
        warm_done = 0
        while warm_done < args.warmup:
            run(args.steps)
            warm_done += args.steps
    else:
        run(args.warmup)
        warm_done = args.warmup
    torch.cuda.synchronize()
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    clk = ClockSampler(torch.cuda.current_device()) if rank == 0 else None
    if clk:
        clk.__enter__()
    _barrier(world)
    # a short device-side delay ahead of the start event lets the host enqueue
    # the timed launches before the GPU reaches them (no host gaps are timed)
    torch.cuda._sleep(200_000)
    start.record(stream)
    run(args.steps)
    end.record(stream)
    _barrier(world)
    if clk:
        clk.__exit__(None, None, None)
    ms = _dist_max(start.elapsed_time(end) / args.steps, world)
    qdev.check_status(dev)
    gbs = world * nbytes / (ms * 1e-3) / 1e9
    peak, peak_kind = _peaks()

    # e2e: public numpy API, host x in and host y out every step
    e2e = None
    if not args.no_e2e:
        qnp = [case.q.copy() for _ in range(copies)]
        snp = [case.scale.copy() for _ in range(copies)]
        xh = np.ascontiguousarray(case.x[0])
        yh = np.empty(N, np.float32)
        for j in range(copies):
            qk.w8a32_gemv(qnp[j], snp[j], xh, yh)          # first use uploads the weights
        for i in range(args.warmup):
            qk.w8a32_gemv(qnp[i % copies], snp[i % copies], xh, yh)
        esteps = max(1, min(args.steps, args.e2e_steps))
        _barrier(world)
        t0 = time.perf_counter()
        for i in range(esteps):
            qk.w8a32_gemv(qnp[i % copies], snp[i % copies], xh, yh)
        et = _dist_max((time.perf_counter() - t0) / esteps, world)
        rel_e = float(np.abs(yh - y_ref).max() / np.abs(y_ref).max())
        if rel_e > 1e-4:
            raise SystemExit(f"e2e parity failed: rel err {rel_e:.3e}")
        e2e = {"value": round(world * nbytes / et / 1e9, 2), "unit": UNIT,
               "h2d_bytes_per_step": int(xh.nbytes), "d2h_bytes_per_step": int(yh.nbytes),
               "ms_per_step": round(et * 1e3, 4), "steps": esteps,
               "note": "numpy w8a32_gemv per rank; int8 weights resident after first use"}

    cpu = None
    if not args.no_cpu and world == 1:
        cgbs, cmed, cthreads, isa = cpu_gemv_gbs(case, reps=args.cpu_reps, threads=_cpu_cores())
        cpu = {"value": round(cgbs, 3), "unit": UNIT, "cores": cthreads, "kind": "port",
               "sample": f"full lm_head GEMV, median of {args.cpu_reps} calls "
                         f"({cmed * 1e3:.3f} ms each, {isa})"}

    _log(rank, f"lm_head GEMV {ms * 1e3:.2f} us/step; e2e and cpu done")
    mlp = None
    if not args.no_mlp:
        mlp = run_mlp_body(args, dev, world=world, do_cpu=(world == 1 and not args.no_cpu))
    _log(rank, "mlp body done")
    w4 = None if args.no_int4 else run_gemv_int4(args, dev, world=world)
    _log(rank, "int4 GEMV done")
    dec = None if args.no_decode else run_decode(args, dev, world=world)
    _log(rank, "decode done")
    tp = None if args.no_tp else run_tp(args, rank, world, dev, case)
    _log(rank, "tensor-parallel block done")
    batch = None if args.no_batch else run_batch_decode(args, rank, world, dev)
    _log(rank, "batched decode done")
    llama = None
    if not args.no_llama and world == 1:
        llama = run_llama_prefill_decode(args, dev)
        _log(rank, "llama prefill + decode done")
    del graphs

    if rank != 0:
        return None
    traffic = None
    tpath = REPO / "profiles" / "gemv_lm_head_traffic.json"
    if tpath.exists():
        traffic = json.loads(tpath.read_text()).get("dram_bytes_per_launch")
    achieved = nbytes / (ms * 1e-3) / 1e9
    return {
        "metric": METRIC, "value": round(gbs, 2), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8 weights, fp32 accumulate", "data": "synthetic",
        "config": bench_config(world, copies),
        "timing": {"graph": use_graph, "graph_steps": chunk if use_graph else None,
                   "warmup_steps_run": warm_done,
                   "note": "warm-up replays the same CUDA graph(s) the timed region replays"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": UNIT,
                     "frac": round(achieved / peak, 4), "peak_kind": peak_kind,
                     "traffic": traffic, "per": "one GPU"},
        "e2e": e2e,
        "cpu_baseline": cpu,
        "clocks": clk.summary() if clk else None,
        "gpu_launches": args.steps,
        "secondary": {"mlp_body": mlp, "gemv_int4": w4, "decode": dec, "tensor_parallel": tp,
                      "batched_decode": batch, "llama_prefill_decode": llama},
    }


def main():
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=4000)
    ap.add_argument("--warmup", type=int, default=100)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--copies", type=int, default=3)
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-mlp", action="store_true")
    ap.add_argument("--no-tp", action="store_true")
    ap.add_argument("--no-decode", action="store_true")
    ap.add_argument("--no-int4", action="store_true")
    ap.add_argument("--no-batch", action="store_true")
    ap.add_argument("--no-llama", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=500)
    ap.add_argument("--cpu-reps", type=int, default=30)
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank != 0:
            return
        print(json.dumps(run_reference(args)), flush=True)
        return
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}: launch N>1 with torchrun")
    # stdout carries exactly one JSON line: anything a library prints to fd 1
    # (NCCL's version banner, for one) goes to stderr while we run
    real_stdout = os.dup(1)
    os.dup2(2, 1)
    import datetime
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(local)
    if world > 1:
        init = "env://"
    else:
        import socket
        with socket.socket() as sk:
            sk.bind(("127.0.0.1", 0))
            init = f"tcp://127.0.0.1:{sk.getsockname()[1]}"
    dist.init_process_group("nccl", init_method=init, rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=300),
                            device_id=torch.device("cuda", local))
    try:
        result = run_ours(args, rank, world, local)
        if rank == 0:
            sys.stdout.flush()
            os.write(real_stdout, (json.dumps(result) + "\n").encode())
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
