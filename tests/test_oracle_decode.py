"""The oracle's CPU decode port against quartz's own greedy decoding on the same
synthetic checkpoints (tests/golden/golden_model.npz): tokens identical, every
step's top-8 logits within 1e-4 of the largest. This pins the port that checks
the device engine and serves as bench.py's CPU decode baseline."""

import json
from pathlib import Path

import numpy as np
import pytest

from oracle.decode_port import DecodePort, rope_inv_freq
from quartz_b200.model import ModelSpec, norm_weights, random_int8_weights, seeded_kv

HERE = Path(__file__).resolve().parent
CASES = {c["id"]: c for c in json.loads((HERE / "golden" / "cases_model.json").read_text())["cases"]}


def _golden(cid, key):
    with np.load(HERE / "golden" / "golden_model.npz") as z:
        return z[f"{cid}__{key}"]


@pytest.mark.parametrize("cid,steps", [("qwen3_tiny_kv", None), ("qwen3_small_kv", None),
                                       ("qwen3_0p6b_kv512", 12)])
def test_port_matches_reference(cid, steps):
    c = CASES[cid]
    spec = ModelSpec.from_hf(c["cfg"], c["arch"])
    steps = steps or c["steps"]
    w = {n: (q, s) for n, q, s in random_int8_weights(spec)}
    port = DecodePort(c["cfg"], c["arch"], w, norm_weights(spec), max_ctx=c["kv_len"] + steps)
    port.load_kv(seeded_kv(spec, c["kv_len"]))
    gold = _golden(cid, "tokens")[:steps].tolist()
    top_ids, top_vals = _golden(cid, "top_ids"), _golden(cid, "top_vals")
    tok, toks = c["first"], []
    for s in range(steps):
        tok = port.step(tok)
        toks.append(tok)
        got = port.logits[top_ids[s]]
        assert np.abs(got - top_vals[s]).max() <= 1e-4 * np.abs(top_vals[s]).max(), (cid, s)
    assert toks == gold


@pytest.mark.parametrize("cid", sorted(CASES))
def test_port_rope_frequencies(cid):
    c = CASES[cid]["cfg"]
    hd = c.get("head_dim") or c["hidden_size"] // c["num_attention_heads"]
    got = rope_inv_freq(hd, c["rope_theta"], c.get("rope_scaling"))
    assert np.array_equal(got, _golden(cid, "inv_freq"))
