"""Golden fixtures produced by the reference (tests/golden/make_golden.py):
loading, input regeneration with the hash pin, and the parity tolerance."""

from __future__ import annotations

import hashlib
import json
from functools import lru_cache
from pathlib import Path

import numpy as np

from quartz_b200.quantize import quantize_symmetric, stack_gate_up
from quartz_b200.workloads import draw_act, draw_weight

GOLDEN = Path(__file__).resolve().parent / "golden"

# Parity bar for fp32 outputs: max |err| <= REL_TOL * ||y||_inf.
REL_TOL = 1e-4


@lru_cache(maxsize=1)
def cases() -> list[dict]:
    with open(GOLDEN / "cases.json") as f:
        return json.load(f)["cases"]


@lru_cache(maxsize=1)
def arrays():
    return dict(np.load(GOLDEN / "golden.npz"))


def case(cid: str) -> dict:
    for c in cases():
        if c["id"] == cid:
            return c
    raise KeyError(cid)


def ids(kind: str) -> list[str]:
    return [c["id"] for c in cases() if c["kind"] == kind]


def arr(cid: str, name: str) -> np.ndarray:
    return arrays()[f"{cid}__{name}"]


def digest(a) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def regen_gemv(c: dict):
    """(q, scale, x) for a gemv/gemm/matmul case; asserts the int8 operands are
    byte-identical to what the reference's quantiser produced."""
    rng = np.random.default_rng(c["seed"])
    W = draw_weight(rng, (c["N"], c["K"]), c["std"], c["recipe"])
    q, s = quantize_symmetric(W, c["group_size"])
    del W
    assert digest(q) == c["q_sha"], f"{c['id']}: q differs from the reference quantiser"
    assert digest(s) == c["s_sha"], f"{c['id']}: scale differs from the reference quantiser"
    if c["kind"] == "gemv":
        x = draw_act(rng, (1, c["K"]), c["recipe"])[0]
    elif c["kind"] == "gemm":
        x = draw_act(rng, (c["M"], c["K"]), c["recipe"])
    else:
        x = draw_act(rng, tuple(c["xshape"]), c["recipe"])
    return q, s, x


def regen_mlp(c: dict):
    rng = np.random.default_rng(c["seed"])
    H, I, gs = c["H"], c["I"], c["group_size"]
    gq, gsc = quantize_symmetric(draw_weight(rng, (I, H), c["std"], c["recipe"]), gs)
    uq, usc = quantize_symmetric(draw_weight(rng, (I, H), c["std"], c["recipe"]), gs)
    dq, dsc = quantize_symmetric(draw_weight(rng, (H, I), c["std"], c["recipe"]), gs)
    x = draw_act(rng, (c["M"], H), c["recipe"])
    gu_q, gu_s = stack_gate_up(gq, gsc, uq, usc)
    assert digest(gu_q) == c["gu_q_sha"] and digest(gu_s) == c["gu_s_sha"]
    assert digest(dq) == c["d_q_sha"] and digest(dsc) == c["d_s_sha"]
    return gu_q, gu_s, dq, dsc, x


def golden_out(c: dict):
    """(reference output, index subset or None, ||y||_inf of the full output)."""
    y = arr(c["id"], "y")
    key = f"{c['id']}__idx"
    if key in arrays():
        return y, arrays()[key], c["y_inf"]
    return y, None, float(np.abs(y).max())


def assert_close(got, ref, inf=None, tol=REL_TOL, what=""):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    if inf is None:
        inf = float(np.abs(ref).max()) if ref.size else 0.0
    err = float(np.abs(got - ref).max()) if ref.size else 0.0
    assert err <= tol * inf + 1e-30, f"{what}: max|err| {err:.3e} > {tol:g} * {inf:.3e}"
    return err / inf if inf else 0.0
