"""GPU parity against the committed golden fixtures (tests/golden/).

ref_patterns: the reference's fused-kernel property-test blocks
(crates/realm-compute-cpu/src/fused.rs:2840-2915, 3483-3573, 3648-3726):
dequant bit-exact; GEMV within the GEMV tolerance (relative to sum |w x|:
1e-5 for every format).

tinyllama_c1: configuration 1 (TinyLlama-1.1B, Q4_K_M, 40-token prompt, 64
greedy tokens, fp32 KV), teacher-forced with the fixture's tokens: logits
|err| <= 2e-3 + 1e-3 |ref| on the stored full-logit steps and on every step's
top-8 logits; greedy argmax agreement >= 99 %.
"""
import os

import numpy as np
import pytest

import synth

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
ATOL, RTOL = 2e-3, 1e-3


@pytest.mark.parametrize("fmt", ["q4k", "q6k", "q80"])
def test_ref_patterns_gpu(ctx, fmt):
    import realm_b200 as rb
    g = np.load(os.path.join(GOLD, "ref_patterns.npz"))
    dt = {"q4k": rb.Q4_K, "q6k": rb.Q6_K, "q80": rb.Q8_0}[fmt]
    b, x, w, y = g[f"{fmt}_blocks"], g[f"{fmt}_x"], g[f"{fmt}_w"], g[f"{fmt}_y"]
    k = x.size
    got_w = ctx.dequantize(dt, b).reshape(2, k)
    assert np.array_equal(got_w.view(np.uint32), w.view(np.uint32))
    got = ctx.fused_dequant_matmul(dt, b, x[None], 1, 2, k)[0]
    scale = np.abs(w.astype(np.float64)) @ np.abs(x.astype(np.float64))
    tol = 1e-5
    assert np.all(np.abs(got.astype(np.float64) - y) / scale < tol)


def test_tinyllama_config1_teacher_forced(ctx):
    import realm_b200 as rb
    g = np.load(os.path.join(GOLD, "tinyllama_c1.npz"))
    cfg = synth.TINYLLAMA
    m = rb.Model(ctx, dict(cfg, kv_dtype=rb.F32, max_tenants=1))
    m.set_weights(synth.make_weights(cfg, seed=0))
    m.tenant_create(0)
    prompt, toks = g["prompt"], g["tokens"]
    for cs in range(0, len(prompt), 8):       # prefill in chunks of 8 (model.rs:784-792)
        lg, am = m.forward_rows([0] * len(prompt[cs:cs + 8]), prompt[cs:cs + 8])
    full = {int(s): i for i, s in enumerate(g["full_steps"])}
    agree = 0
    for step in range(len(toks)):
        if step > 0:
            lg, am = m.forward_rows([0], [toks[step - 1]])
        row = lg[-1]
        if step in full:
            ref = g["full_logits"][full[step]]
            err = np.abs(row - ref)
            assert np.all(err <= ATOL + RTOL * np.abs(ref)), (step, err.max())
        ref_top = g["top_val"][step]
        got_top = row[g["top_idx"][step]]
        assert np.all(np.abs(got_top - ref_top) <= ATOL + RTOL * np.abs(ref_top)), step
        agree += int(am[-1] == toks[step])
    assert agree / len(toks) >= 0.99, agree
    m.close()
