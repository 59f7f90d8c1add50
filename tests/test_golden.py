"""The oracle against the committed golden fixtures (tests/golden/, made by
tests/golden/make_golden.py). Guards the checker itself: if the oracle drifts,
the GPU parity tests would compare against the wrong numbers."""
import os

import numpy as np
import pytest

import synth

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load(name):
    return np.load(os.path.join(GOLD, name))


@pytest.mark.parametrize("fmt", ["q4k", "q6k", "q80"])
def test_ref_patterns(oracle, fmt):
    """fused.rs property-test block patterns: bit-exact dequant, fused GEMV within
    the reference's own bound (rel < 1e-4)."""
    O = oracle
    g = _load("ref_patterns.npz")
    dt = {"q4k": O.Q4K, "q6k": O.Q6K, "q80": O.Q80}[fmt]
    b, x, w, y = g[f"{fmt}_blocks"], g[f"{fmt}_x"], g[f"{fmt}_w"], g[f"{fmt}_y"]
    k = x.size
    assert np.array_equal(O.dequant(dt, b).reshape(2, k).view(np.uint32), w.view(np.uint32))
    rc, got = O.fused_matmul(dt, b, x[None], 1, 2, k)
    assert rc == 2
    assert np.all(np.abs(got[0] - y) <= 1e-4 * np.maximum(np.abs(y), 1e-6))


def test_tinyllama_prefix(oracle):
    """Config 1: the oracle regenerates the first greedy tokens and their top logits."""
    O = oracle
    g = _load("tinyllama_c1.npz")
    cfg = synth.TINYLLAMA
    om = O.Model(dict(cfg, kv_fp16=0), synth.make_weights(cfg, seed=0))
    n = 4
    toks, logits = om.generate(g["prompt"], n)
    assert np.array_equal(toks, g["tokens"][:n])
    got = np.take_along_axis(logits, g["top_idx"][:n].astype(np.int64), axis=1)
    assert np.abs(got - g["top_val"][:n]).max() < 1e-4
    assert np.abs(logits[0] - g["full_logits"][0]).max() < 1e-4
