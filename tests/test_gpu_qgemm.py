"""GPU parity of the tcgen05 dequant-GEMM (batches of 16..64 rows).

With RB_QGEMM=1 (read when a context is created), rb_weight_matmul,
rb_fused_dequant_matmul and rb_forward route 16+ rows of every format to the
tcgen05 kernels (by default only Q4_K batches of 33+ rows take them: the
exact-weight GEMM, faster than the mma.sync GEMV there on B200). Q4_K runs
the exact-weight GEMM (A = sc * q in fp16, exact; d and dmin applied per
super-block when tensor memory is drained); Q6_K / Q8_0 the hi/lo-weight GEMM
(weights dequantised as dequantize_q6_k / q8_0 do, crates/realm-core/src/quant.rs,
scaled by a per-row power of two and split into fp16 hi + lo, three MMAs per
k-step). Activations fp16 hi + lo, fp32 accumulation in tensor memory.
Compared with the oracle's dequant + GEMM in double, relative to
sum_k |W[n,k] x[k]|: 3e-5 for Q4_K, 1e-5 for Q6_K / Q8_0. Also against the
mma.sync GEMV (a context with RB_QGEMM=0), NaN scale guards, ragged shapes, determinism, and a model forward
whose prefill chunks run on the GEMM, against the oracle's Model::forward.
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def qctx():
    import realm_b200 as rb
    os.environ["RB_QGEMM"] = "1"
    try:
        c = rb.Context(0)
    finally:
        del os.environ["RB_QGEMM"]
    yield c
    c.close()


@pytest.fixture(scope="module")
def gemv_ctx():
    """A context that keeps every batch on the mma.sync GEMV."""
    import realm_b200 as rb
    os.environ["RB_QGEMM"] = "0"
    try:
        c = rb.Context(0)
    finally:
        del os.environ["RB_QGEMM"]
    yield c
    c.close()


def _dt(O, name):
    return {"q4k": O.Q4K, "q6k": O.Q6K, "q80": O.Q80}[name]


def _err(O, dt, blocks, x, got, m, n, k):
    ref = O.dequant_matmul(dt, blocks, x, m, n, k, f64=True)
    w = O.dequant(dt, blocks).reshape(n, k).astype(np.float64)
    scale = np.abs(x.astype(np.float64)) @ np.abs(w).T + 1e-30
    return (np.abs(got.astype(np.float64) - ref) / scale).max()


@pytest.mark.parametrize("fmt", ["q4k", "q6k", "q80"])
@pytest.mark.parametrize("m", [16, 17, 24, 33, 48, 64])
def test_qgemm_vs_oracle(qctx, oracle, fmt, m):
    O = oracle
    dt = _dt(O, fmt)
    rng = np.random.default_rng(1000 + m)
    n, k = 640, 1536
    blocks = O.quantize(dt, rng.normal(0, 0.02, size=(n, k)).astype(np.float32))
    x = rng.normal(0, 1, size=(m, k)).astype(np.float32)
    got = qctx.fused_dequant_matmul(dt, blocks, x, m, n, k)
    assert np.all(np.isfinite(got))
    assert _err(O, dt, blocks, x, got, m, n, k) < (3e-5 if dt == O.Q4K else 1e-5)


@pytest.mark.parametrize("fmt,n,k,m", [
    ("q4k", 22016, 4096, 64),   # Llama-2-7B gate|up
    ("q4k", 4096, 11008, 40),   # down projection
    ("q6k", 32000, 4096, 16),   # LM head
    ("q4k", 300, 512, 20),      # ragged rows, one super-block pair
    ("q80", 40, 64, 16),        # Q8_0 K padded to 256
    ("q6k", 17, 256, 33),       # a single 128-row tile, one super-block
])
def test_qgemm_shapes(qctx, oracle, fmt, n, k, m):
    O = oracle
    dt = _dt(O, fmt)
    rng = np.random.default_rng(n + k + m)
    blocks = O.quantize(dt, rng.normal(0, 0.02, size=(n, k)).astype(np.float32))
    x = rng.normal(0, 1, size=(m, k)).astype(np.float32)
    got = qctx.fused_dequant_matmul(dt, blocks, x, m, n, k)
    assert _err(O, dt, blocks, x, got, m, n, k) < (3e-5 if dt == O.Q4K else 1e-5)


def test_qgemm_scale_extremes_and_nan_guard(qctx, oracle):
    """Rows of very different magnitudes (the per-row exponent keeps each in fp16
    range) and NaN / Inf scales (replaced by 6e-8 / 2.4e-7 as the fused kernels do)."""
    O = oracle
    rng = np.random.default_rng(8)
    n, k, m = 256, 1024, 32
    W = rng.normal(0, 1, size=(n, k)).astype(np.float32)
    W *= (10.0 ** rng.uniform(-6, 3, size=(n, 1))).astype(np.float32)
    blocks = O.quantize(O.Q4K, W).reshape(-1, 144).copy()
    blocks[5, 0:2] = np.frombuffer(np.uint16(0x7E00).tobytes(), np.uint8)
    blocks[11, 2:4] = np.frombuffer(np.uint16(0x7C00).tobytes(), np.uint8)
    blocks = blocks.ravel()
    x = rng.normal(0, 1, size=(m, k)).astype(np.float32)
    rc, ref = O.fused_matmul(O.Q4K, blocks, x, m, n, k)
    got = qctx.fused_dequant_matmul(O.Q4K, blocks, x, m, n, k)
    assert np.all(np.isfinite(got))
    wdq = np.nan_to_num(O.dequant(O.Q4K, blocks).reshape(n, k).astype(np.float64), nan=0.0, posinf=0.0, neginf=0.0)
    scale = np.abs(x.astype(np.float64)) @ np.abs(wdq).T
    bad = np.zeros(n, bool)
    bad[5 // 4] = bad[11 // 4] = True   # rows whose blocks carry the replaced scales
    err = np.abs(got - ref) / (scale + 1e-30)
    assert err[:, ~bad].max() < 3e-5
    # the replaced scales: the same bound (a wrong replacement value would miss by
    # the super-block's whole contribution); the exact-weight GEMM folds d and
    # dmin in per super-block, so its rounding follows sum |W x|, not |y|
    assert err[:, bad].max() < 3e-5


def test_qgemm_matches_gemv_and_is_deterministic(gemv_ctx, qctx, oracle):
    import realm_b200 as rb
    O = oracle
    rng = np.random.default_rng(9)
    n, k, m = 4096, 4096, 48
    blocks = O.quantize(O.Q4K, rng.normal(0, 0.02, size=(n, k)).astype(np.float32))
    x = rng.normal(0, 1, size=(m, k)).astype(np.float32)
    w = rb.Weight(qctx, rb.Q4_K, n, k, blocks)
    a, b = w.matmul(x, m), w.matmul(x, m)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
    w.free()
    g = gemv_ctx.fused_dequant_matmul(rb.Q4_K, blocks, x, m, n, k)
    wd = O.dequant(O.Q4K, blocks).reshape(n, k).astype(np.float64)
    scale = np.abs(x.astype(np.float64)) @ np.abs(wd).T
    assert (np.abs(a.astype(np.float64) - g) / scale).max() < 6e-5


def test_forward_prefill_on_qgemm_matches_oracle(qctx, oracle):
    """A 40-row prefill chunk and a 24-row mixed batch run every projection on the
    GEMM (fused epilogues: RoPE + KV append, residual, SwiGLU, logits)."""
    import realm_b200 as rb
    import synth
    O = oracle
    cfg = synth.SMALL
    W = synth.make_weights(cfg, seed=0)
    m = rb.Model(qctx, dict(cfg, kv_dtype=rb.F16, max_tenants=4))
    m.set_weights(W)
    rng = np.random.default_rng(12)
    prompts = [rng.integers(0, cfg["vocab"], 40).astype(np.uint32), rng.integers(0, cfg["vocab"], 23).astype(np.uint32)]
    m.tenant_create(0)
    m.tenant_create(1)
    lg0, am0 = m.forward_rows([0] * 40, prompts[0])
    lg1, am1 = m.forward_rows([1] * 23 + [0], np.concatenate([prompts[1], [am0[-1]]]).astype(np.uint32))
    for t, (lg, toks) in enumerate([(lg1[22], prompts[1]), (lg0[39], prompts[0])]):
        om = O.Model(dict(cfg, kv_fp16=1), W)
        ref = om.forward(toks, 0)
        assert np.all(np.abs(lg - ref) <= 2e-3 + 1e-3 * np.abs(ref)), (t, np.abs(lg - ref).max())
    om = O.Model(dict(cfg, kv_fp16=1), W)
    om.forward(prompts[0], 0)
    ref = om.forward(np.array([am0[-1]], np.uint32), 40)
    assert np.all(np.abs(lg1[23] - ref) <= 2e-3 + 1e-3 * np.abs(ref))
    m.close()
