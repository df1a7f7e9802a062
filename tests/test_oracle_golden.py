"""The oracle against fixtures the reference itself produced (tests/golden/make_golden.py).

These run without the reference sources: inputs are regenerated from their
seeds (pinned by SHA-256) and the oracle must reproduce the reference's
outputs bit for bit, in the evaluation order of the kernel table the reference
selected when the fixtures were made (meta.json "isa").
"""
import hashlib
import json
import os

import numpy as np
import pytest

from oracle.oracle import ORDER_AVX2, ORDER_VNNI, q8k_fields

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
META = json.load(open(os.path.join(GOLD, "meta.json")))
ORDER = ORDER_VNNI if "VNNI" in META["isa"] else ORDER_AVX2


def load(name):
    return np.load(os.path.join(GOLD, name + ".npz"))


def test_router_known_answer(oracle):
    """Reference test 3 (tests/test_moe_checkpoint.c:138-218): experts 9 and 25
    must win, weights sum to 1 within 1e-6, ratios equal the unbiased sigmoid
    ratios within 1e-5; and the exact ids/weights the reference produced."""
    g = load("router_kat")
    xb, w, b = oracle.kat_router_inputs(2048, 32)
    idx, wt, logits, _ = oracle.route(w, b, xb, 4)
    assert np.array_equal(idx, g["idx"]) and np.array_equal(wt, g["w"])
    assert 9 in idx and 25 in idx
    assert abs(float(wt.sum()) - 1.0) < 1e-6
    sig = 1.0 / (1.0 + np.exp(-logits.astype(np.float64)))
    np.testing.assert_allclose(wt / wt[0], sig[idx] / sig[idx[0]], atol=1e-5)


def test_q8k_known_answer(oracle):
    """Reference Q8_K test input (tests/test_cpuid_quants.c:69-111) and the all-zero edge case."""
    g = load("q8k_kat")
    x = oracle.kat_q8k_inputs(2048)
    q = oracle.quantize_q8k(x)
    assert np.array_equal(q, g["q8"])
    qz = oracle.quantize_q8k(np.zeros(512, np.float32))
    assert np.array_equal(qz, g["q8_zero"])
    d, qs, bs = q8k_fields(qz, 2)
    assert np.all(d == 0) and np.all(qs == 0) and np.all(bs == 0)


@pytest.mark.parametrize("name", sorted(META["cases"]["moe"]))
def test_moe_layer_golden(oracle, name):
    from laii_b200 import synth
    c = META["cases"]["moe"][name]
    L = synth.make_moe_layer(c["D"], c["E"], c["K"], c["I"], layer=c["layer"], down_type=c.get("down_type", 12))
    x = synth.make_hidden(c["T"], c["D"], seed_offset=c["seed_offset"])
    assert L.digest() == META["digests"][name]["layer"], "synthetic generator changed"
    assert hashlib.sha256(x.tobytes()).hexdigest() == META["digests"][name]["x"]
    g = load(name)
    xo, idx, w, xq, _ = oracle.moe_forward(L, x, order=ORDER)
    assert np.array_equal(idx, g["idx"])
    assert np.array_equal(w, g["w"])
    assert np.array_equal(xq, g["xq"])
    assert np.array_equal(xo, g["x_out"])


def test_dense_layer_golden(oracle):
    from laii_b200 import synth
    c = META["cases"]["dense"]
    L = synth.make_dense_layer(c["D"], c["I"], layer=c["layer"])
    x = synth.make_hidden(c["T"], c["D"], seed_offset=c["seed_offset"])
    assert np.array_equal(oracle.dense_forward(L, x, order=ORDER), load("dense_small")["x_out"])
