"""Failure detection on the GPU without a GPU fault.

A grid barrier of the multi-phase GEMV launch is made to run out on purpose
(rb_test_fail_next_grid_barrier: its target is moved out of reach and every
barrier wait gives up after a few polls). The bounded waits record the
failure in the device error word and the kernel finishes; the host turns it
into RB_ERR_TIMEOUT (-25), the reference's convention of a negative status
from the host functions (crates/realm-runtime/src/host_functions.rs:145-155).
The context must then run the same step again and match the oracle.
"""
import numpy as np
import pytest

import synth

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-3


def test_grid_barrier_timeout_reports_and_context_recovers(ctx, oracle):
    import realm_b200 as rb
    O = oracle
    cfg = synth.SMALL
    W = synth.make_weights(cfg, seed=0)
    prompt = np.random.default_rng(8).integers(0, cfg["vocab"], 11).astype(np.uint32)
    om = O.Model(dict(cfg, kv_fp16=1), W)
    toks, ref_logits = om.generate(prompt, 4)
    m = rb.Model(ctx, dict(cfg, kv_dtype=rb.F16, max_tenants=2))
    m.set_weights(W)
    m.tenant_create(0)
    lg, am = m.forward_rows([0] * len(prompt), prompt)
    assert int(am[-1]) == toks[0]
    # step 1 fails on purpose: one barrier wait runs out
    assert rb.lib().rb_test_fail_next_grid_barrier(ctx.handle, 256) == 0
    with pytest.raises(rb.RealmError) as e:
        m.forward_rows([0], [toks[0]])
    assert e.value.code == -25, e.value
    assert "grid barrier" in str(e.value)
    assert m.kv.len(0) == len(prompt)  # the failed step did not advance the cache
    # the same step, then one more, run correctly on the same context
    for g in (1, 2):
        lg, am = m.forward_rows([0], [toks[g - 1]])
        err = np.abs(lg[-1] - ref_logits[g])
        assert np.all(err <= ATOL + RTOL * np.abs(ref_logits[g])), (g, err.max())
        assert int(am[-1]) == toks[g]
    m.close()
