"""Generate the golden fixtures by running the reference itself (quartz, Numba).

Run in a container where the reference source is present:

    NUMBA_CACHE_DIR=/tmp/numba_cache PYTHONDONTWRITEBYTECODE=1 \
        python tests/golden/make_golden.py /root/reference

For every case the script draws fp32 weights and activations with the recipes of
``quartz_b200.workloads`` (the RNG recipe only), quantises them with the
reference's own ``quantize_symmetric`` (quartz/quantize.py:26-38), runs the
reference kernel, and stores:

* the case parameters (seed, shapes, group size, recipe) in ``cases.json``;
* SHA-256 digests of the reference's q and scale bytes, so a test can prove that
  regenerating the inputs on our side gives the same int8 operands;
* the reference's fp32 outputs (all of them, or a fixed index subset for the
  large shapes) in ``golden.npz``.

The tests never import the reference: they regenerate inputs from the
parameters and compare against the stored outputs.
"""

from __future__ import annotations

import hashlib
import json
import os
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from quartz_b200.workloads import draw_weight, draw_act  # noqa: E402  (RNG recipe only)


def _digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _subset(n: int, stride: int) -> np.ndarray:
    """Every `stride`-th index plus the last 64 (the ragged tail of any tiling)."""
    idx = np.arange(0, n, stride, dtype=np.int64)
    tail = np.arange(max(0, n - 64), n, dtype=np.int64)
    return np.unique(np.concatenate([idx, tail]))


def main(ref_root: str) -> None:
    os.environ.setdefault("NUMBA_CACHE_DIR", "/tmp/numba_cache")
    sys.path.insert(0, ref_root)
    from quartz.quantize import quantize_symmetric, FusedMLP, QuantizedLinear
    from quartz.kernels.int8 import (w8a32_gemv, w8a32_gemv_serial, w8a32_gemm,
                                     matmul_int8, warmup)
    from quartz.kernels.fused import fused_mlp_decode, warmup_fused

    warmup()
    warmup_fused()
    cases: list[dict] = []
    arrays: dict[str, np.ndarray] = {}

    def put(cid, name, arr):
        arrays[f"{cid}__{name}"] = np.ascontiguousarray(arr)

    # ---------------- GEMV (int8.py:24-38) ----------------
    gemv_specs = []
    for (N, K) in [(3072, 1024), (1024, 3072), (2048, 1024), (1024, 1024), (64, 32),
                   (151936, 1024)]:
        for g in (None, 64):
            if g and K % g:
                continue
            gemv_specs.append(dict(N=N, K=K, group_size=g, seed=0, std=0.05, recipe="f64"))
    gemv_specs += [
        dict(N=151936, K=1024, group_size=None, seed=0, std=0.02, recipe="f32"),  # lm_head workload
        dict(N=4096, K=4096, group_size=None, seed=5, std=0.02, recipe="f32"),
        dict(N=256, K=12288, group_size=None, seed=6, std=0.02, recipe="f32"),
        dict(N=2048, K=8192, group_size=None, seed=7, std=0.02, recipe="f32"),
        dict(N=1000, K=2048, group_size=128, seed=8, std=0.02, recipe="f32"),
        dict(N=777, K=512, group_size=32, seed=9, std=0.02, recipe="f32"),
        dict(N=1, K=16, group_size=None, seed=10, std=0.02, recipe="f32"),
        dict(N=7, K=48, group_size=16, seed=11, std=0.02, recipe="f32"),
        dict(N=5, K=40, group_size=8, seed=12, std=0.02, recipe="f32"),
        dict(N=33, K=1000, group_size=None, seed=13, std=0.02, recipe="f32"),
        dict(N=129, K=24, group_size=None, seed=14, std=0.02, recipe="f32"),
    ]
    for i, sp in enumerate(gemv_specs):
        cid = f"gemv{i}"
        rng = np.random.default_rng(sp["seed"])
        W = draw_weight(rng, (sp["N"], sp["K"]), sp["std"], sp["recipe"])
        q, s = quantize_symmetric(W, sp["group_size"])
        del W
        x = draw_act(rng, (1, sp["K"]), sp["recipe"])[0]
        y = np.empty(sp["N"], np.float32)
        w8a32_gemv(q, s, x, y)
        ys = np.empty(sp["N"], np.float32)
        w8a32_gemv_serial(q, s, x, ys)
        assert np.array_equal(y, ys)
        rec = dict(id=cid, kind="gemv", **sp, q_sha=_digest(q), s_sha=_digest(s))
        if sp["N"] > 8192:
            idx = _subset(sp["N"], 64)
            put(cid, "idx", idx)
            put(cid, "y", y[idx])
            rec["y_inf"] = float(np.abs(y).max())
        else:
            put(cid, "y", y)
        cases.append(rec)

    # Hand-built edge cases: the warmup shapes (int8.py:111-117), zero rows
    # (scale replaced by 1, quantize.py:36) and +-127 extremes.
    cid = "gemv_warmup"
    q = np.ones((2, 4), np.int8); s = np.ones((2, 1), np.float32)
    y = np.zeros(2, np.float32)
    w8a32_gemv(q, s, np.ones(4, np.float32), y)
    put(cid, "q", q); put(cid, "s", s); put(cid, "x", np.ones(4, np.float32)); put(cid, "y", y)
    cases.append(dict(id=cid, kind="gemv_explicit"))

    cid = "gemv_edges"
    rng = np.random.default_rng(21)
    W = draw_weight(rng, (40, 96), 0.02, "f32")
    W[3] = 0.0                        # all-zero row -> scale 1.0, q 0
    W[7, :32] = 0.0                   # all-zero group (group_size 32)
    W[11] = np.float32(0.5) * np.sign(rng.standard_normal(96)).astype(np.float32)  # +-127 everywhere
    W[12, 5] = np.float32(3.0)        # one outlier: most of the row rounds to 0
    q, s = quantize_symmetric(W, 32)
    x = draw_act(rng, (1, 96), "f32")[0]
    y = np.empty(40, np.float32)
    w8a32_gemv(q, s, x, y)
    put(cid, "q", q); put(cid, "s", s); put(cid, "x", x); put(cid, "y", y)
    cases.append(dict(id=cid, kind="gemv_explicit"))

    # ---------------- quantiser (quantize.py:26-38) ----------------
    cid = "quant0"
    rng = np.random.default_rng(3)
    W = draw_weight(rng, (40, 64), 0.05, "f64")
    q, s = quantize_symmetric(W, 32)
    put(cid, "W", W); put(cid, "q", q); put(cid, "s", s)
    cases.append(dict(id=cid, kind="quant", group_size=32))

    # ---------------- GEMM (int8.py:66-87) ----------------
    gemm_specs = [
        dict(N=128, K=64, M=5, group_size=None, seed=1, std=0.05, recipe="f64"),
        dict(N=1024, K=1024, M=16, group_size=None, seed=31, std=0.02, recipe="f32"),
        dict(N=2048, K=1024, M=2, group_size=None, seed=32, std=0.02, recipe="f32"),
        dict(N=1024, K=4096, M=8, group_size=None, seed=33, std=0.02, recipe="f32"),
        dict(N=256, K=2048, M=64, group_size=None, seed=34, std=0.02, recipe="f32"),
        dict(N=512, K=1024, M=128, group_size=None, seed=35, std=0.02, recipe="f32"),
        dict(N=256, K=512, M=4, group_size=64, seed=36, std=0.02, recipe="f32"),
        dict(N=128, K=256, M=70, group_size=32, seed=37, std=0.02, recipe="f32"),
        dict(N=100, K=40, M=3, group_size=8, seed=38, std=0.02, recipe="f32"),
    ]
    for i, sp in enumerate(gemm_specs):
        cid = f"gemm{i}"
        rng = np.random.default_rng(sp["seed"])
        W = draw_weight(rng, (sp["N"], sp["K"]), sp["std"], sp["recipe"])
        q, s = quantize_symmetric(W, sp["group_size"])
        X = draw_act(rng, (sp["M"], sp["K"]), sp["recipe"])
        Y = np.empty((sp["M"], sp["N"]), np.float32)
        w8a32_gemm(q, s, X, Y)
        rec = dict(id=cid, kind="gemm", **sp, q_sha=_digest(q), s_sha=_digest(s))
        if Y.size > 16384:
            idx = _subset(Y.size, 7)
            put(cid, "idx", idx); put(cid, "y", Y.ravel()[idx])
            rec["y_inf"] = float(np.abs(Y).max())
        else:
            put(cid, "y", Y)
        cases.append(rec)

    # ---------------- matmul_int8 dispatcher (int8.py:90-108) ----------------
    for i, xshape in enumerate([(1, 3, 64), (1, 1, 64), (64,), (2, 2, 64), (4, 1, 1, 64)]):
        cid = f"matmul{i}"
        rng = np.random.default_rng(2)
        W = draw_weight(rng, (100, 64), 0.05, "f64")
        q, s = quantize_symmetric(W, None)
        x = draw_act(rng, xshape, "f64")
        out = matmul_int8(q, s, x)
        put(cid, "y", out)
        cases.append(dict(id=cid, kind="matmul", N=100, K=64, group_size=None, seed=2,
                          std=0.05, recipe="f64", xshape=list(xshape),
                          q_sha=_digest(q), s_sha=_digest(s)))

    # ---------------- fused MLP (fused.py:27-65; FusedMLP quantize.py:86-114) ----------------
    mlp_specs = [
        dict(H=128, I=256, M=1, group_size=None, seed=0, std=0.05, recipe="f64"),
        dict(H=128, I=256, M=1, group_size=64, seed=0, std=0.05, recipe="f64"),
        dict(H=1024, I=3072, M=1, group_size=None, seed=1000, std=0.02, recipe="f32"),
        dict(H=1024, I=3072, M=1, group_size=None, seed=1001, std=0.02, recipe="f32"),
        dict(H=1024, I=3072, M=1, group_size=None, seed=1027, std=0.02, recipe="f32"),
        dict(H=2048, I=8192, M=1, group_size=None, seed=3000, std=0.02, recipe="f32"),
        dict(H=4096, I=12288, M=1, group_size=None, seed=2000, std=0.02, recipe="f32"),
        dict(H=256, I=512, M=1, group_size=32, seed=41, std=0.02, recipe="f32"),
        dict(H=128, I=256, M=5, group_size=None, seed=0, std=0.05, recipe="f64"),
        dict(H=128, I=256, M=5, group_size=64, seed=0, std=0.05, recipe="f64"),
    ]
    for i, sp in enumerate(mlp_specs):
        cid = f"mlp{i}"
        rng = np.random.default_rng(sp["seed"])
        H, I, gs = sp["H"], sp["I"], sp["group_size"]
        gq, gsc = quantize_symmetric(draw_weight(rng, (I, H), sp["std"], sp["recipe"]), gs)
        uq, usc = quantize_symmetric(draw_weight(rng, (I, H), sp["std"], sp["recipe"]), gs)
        dq, dsc = quantize_symmetric(draw_weight(rng, (H, I), sp["std"], sp["recipe"]), gs)
        x = draw_act(rng, (sp["M"], H), sp["recipe"])
        mlp = FusedMLP(QuantizedLinear(gq, gsc, gs, I, H), QuantizedLinear(uq, usc, gs, I, H),
                       QuantizedLinear(dq, dsc, gs, H, I))
        if sp["M"] == 1:
            abuf = np.empty(I, np.float32)
            out = np.empty(H, np.float32)
            fused_mlp_decode(mlp.gu_q, mlp.gu_s, np.ascontiguousarray(x[0]), mlp.down_q,
                             mlp.down_s, abuf, out)
            put(cid, "abuf", abuf)
        else:
            out = mlp(x.reshape(1, sp["M"], H)).reshape(sp["M"], H)
        put(cid, "y", out)
        cases.append(dict(id=cid, kind="mlp", **sp,
                          gu_q_sha=_digest(mlp.gu_q), gu_s_sha=_digest(mlp.gu_s),
                          d_q_sha=_digest(dq), d_s_sha=_digest(dsc)))

    np.savez_compressed(HERE / "golden.npz", **arrays)
    with open(HERE / "cases.json", "w") as f:
        json.dump(dict(
            generator="tests/golden/make_golden.py",
            reference="mlelarge/quartz (quartz/kernels/int8.py, quartz/kernels/fused.py, "
                      "quartz/quantize.py)",
            numpy=np.__version__,
            numba=__import__("numba").__version__,
            cases=cases), f, indent=1)
    print(f"wrote {len(cases)} cases, {sum(a.nbytes for a in arrays.values())} bytes raw")


if __name__ == "__main__":
    if len(sys.argv) < 2:
        raise SystemExit("usage: make_golden.py <path of the quartz source tree>")
    main(sys.argv[1])
