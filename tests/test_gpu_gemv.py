"""GPU parity: block dequant, quantiser, tile repack and the fused dequant GEMV.

Oracle: oracle/oracle.cpp (restatement of crates/realm-core/src/quant.rs and
crates/realm-compute-cpu/src/fused.rs). Dequant, quantise and repack are
bit-exact; GEMV outputs are compared with the oracle's dequant+GEMM accumulated
in double. Tolerance, relative to sum_k |W[n,k] x[k]|: 1e-5 (exact integer
tensor-core weights; fp16 hi/lo activations, ~22 bits, for Q6_K / Q8_0; int8
three-limb activations, per-element error <= 2^-24 of the 64-column group
maximum, for Q4_K). The absolute logits bound (2e-3 + 1e-3 |y|) is checked on
outlier-bearing rows in test_gpu_configs and end to end in test_gpu_model.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

FMTS = ["q4k", "q6k", "q80"]


def _dt(O, name):
    return {"q4k": O.Q4K, "q6k": O.Q6K, "q80": O.Q80}[name]


def _rand_blocks(O, dt, n, rng):
    """Random block bytes with sane fp16 scales (every bit pattern of the quants)."""
    bb = O.BLOCK_BYTES[dt]
    raw = rng.integers(0, 256, size=(n, bb), dtype=np.uint8)
    def f16(vals):
        return np.array([O.f32_to_f16_bits(float(v)) for v in vals], np.uint16).view(np.uint8).reshape(-1, 2)
    if dt == O.Q4K:
        raw[:, 0:2] = f16(rng.uniform(1e-4, 2e-3, n))
        raw[:, 2:4] = f16(rng.uniform(1e-4, 2e-3, n))
    elif dt == O.Q6K:
        raw[:, 208:210] = f16(rng.uniform(1e-5, 1e-3, n))
    else:
        raw[:, 0:2] = f16(rng.uniform(1e-4, 1e-2, n))
    return raw.ravel()


@pytest.mark.parametrize("fmt", FMTS)
def test_dequant_bit_exact(ctx, oracle, fmt):
    O = oracle
    dt = _dt(O, fmt)
    rng = np.random.default_rng(11)
    blocks = _rand_blocks(O, dt, 777, rng)
    ref = O.dequant(dt, blocks)
    got = ctx.dequantize(dt, blocks)
    assert np.array_equal(ref.view(np.uint32), got.view(np.uint32))


@pytest.mark.parametrize("fmt", FMTS)
def test_quantize_bit_exact(ctx, oracle, fmt):
    O = oracle
    dt = _dt(O, fmt)
    rng = np.random.default_rng(12)
    x = rng.normal(0, 0.02, size=256 * 300).astype(np.float32)
    x[:256] = 0.0                     # all-zero block
    x[256:512] = np.abs(x[256:512])   # min > 0 branch
    assert np.array_equal(O.quantize(dt, x), ctx.quantize(dt, x))


def test_repack_round_trip(ctx, oracle):
    O = oracle
    rng = np.random.default_rng(13)
    n, k = 300, 1024  # n not a multiple of the 128-row group: exercises padding
    blocks = _rand_blocks(O, O.Q4K, n * k // 256, rng)
    import realm_b200 as rb
    w = rb.Weight(ctx, rb.Q4_K, n, k, blocks)
    assert np.array_equal(w.export(), blocks)
    w.free()


def _check_gemv(O, dt, blocks, x, got, m, n, k, tol=None):
    if tol is None:
        tol = 1e-5
    ref = O.dequant_matmul(dt, blocks, x, m, n, k, f64=True)
    w = O.dequant(dt, blocks).reshape(n, k).astype(np.float64)
    scale = np.abs(x.astype(np.float64)) @ np.abs(w).T + 1e-30
    err = np.abs(got.astype(np.float64) - ref) / scale
    assert err.max() < tol, (err.max(), np.unravel_index(err.argmax(), err.shape))


@pytest.mark.parametrize("fmt", FMTS)
@pytest.mark.parametrize("m", [1, 3, 8, 9, 16, 33, 64])
def test_gemv_vs_oracle(ctx, oracle, fmt, m):
    O = oracle
    dt = _dt(O, fmt)
    rng = np.random.default_rng(100 + m)
    n, k = 384, 1024
    W = rng.normal(0, 0.02, size=(n, k)).astype(np.float32)
    blocks = O.quantize(dt, W)
    x = rng.normal(0, 1, size=(m, k)).astype(np.float32)
    got = ctx.fused_dequant_matmul(dt, blocks, x, m, n, k)
    _check_gemv(O, dt, blocks, x, got, m, n, k)


@pytest.mark.parametrize("n,k", [(4096, 4096), (11008, 4096), (4096, 11008), (300, 512), (16, 256)])
def test_gemv_shapes_q4k(ctx, oracle, n, k):
    O = oracle
    rng = np.random.default_rng(n + k)
    blocks = O.quantize(O.Q4K, rng.normal(0, 0.02, size=(n, k)).astype(np.float32))
    for m in (1, 8):
        x = rng.normal(0, 1, size=(m, k)).astype(np.float32)
        got = ctx.fused_dequant_matmul(O.Q4K, blocks, x, m, n, k)
        _check_gemv(O, O.Q4K, blocks, x, got, m, n, k)


@pytest.mark.parametrize("n,k", [(40, 64), (300, 544), (17, 32)])
def test_gemv_q80_k_not_multiple_of_256(ctx, oracle, n, k):
    """Q8_0 takes any K that is a multiple of 32 (fused.rs:2451-2554); rows are
    zero-padded to the next 256 columns inside the library."""
    O = oracle
    import realm_b200 as rb
    rng = np.random.default_rng(n * k)
    blocks = O.quantize(O.Q80, rng.normal(0, 0.02, size=(n, k)).astype(np.float32))
    for m in (1, 5):
        x = rng.normal(0, 1, size=(m, k)).astype(np.float32)
        _check_gemv(O, O.Q80, blocks, x, ctx.fused_dequant_matmul(O.Q80, blocks, x, m, n, k), m, n, k)
        w = rb.Weight(ctx, rb.Q8_0, n, k, blocks)
        _check_gemv(O, O.Q80, blocks, x, w.matmul(x, m), m, n, k)
        w.free()


def test_gemv_q6k_lm_head_shape(ctx, oracle):
    O = oracle
    rng = np.random.default_rng(7)
    n, k = 32000, 4096
    blocks = O.quantize(O.Q6K, rng.normal(0, 0.02, size=(n, k)).astype(np.float32))
    x = rng.normal(0, 1, size=(16, k)).astype(np.float32)
    got = ctx.fused_dequant_matmul(O.Q6K, blocks, x, 16, n, k)
    _check_gemv(O, O.Q6K, blocks, x, got, 16, n, k)


def test_gemv_matches_reference_fused_kernel(ctx, oracle):
    """Reference property test pattern (fused.rs:2840-2915) through the GPU."""
    O = oracle
    import struct
    blocks = bytearray()
    for i in range(2):
        for j in range(2):
            sv = 16 + i + j
            blocks += struct.pack("<HH", O.f32_to_f16_bits(0.5 + i * 0.1), O.f32_to_f16_bits(0.1))
            blocks += bytes([sv] * 12) + bytes([(i * 17 + j * 13) % 256] * 128)
    blocks = np.frombuffer(bytes(blocks), np.uint8)
    x = np.array([((i % 7) - 3.0) * 0.5 for i in range(512)], np.float32)[None]
    rc, ref = O.fused_matmul(O.Q4K, blocks, x, 1, 2, 512)
    got = ctx.fused_dequant_matmul(O.Q4K, blocks, x, 1, 2, 512)
    assert np.allclose(got, ref, rtol=1e-4, atol=0)


def test_gemv_nan_scale_guard(ctx, oracle):
    """fused.rs:276-285: NaN/Inf d -> 6e-8, dmin -> 2.4e-7 in the fused kernels."""
    O = oracle
    rng = np.random.default_rng(5)
    n, k = 128, 512
    blocks = O.quantize(O.Q4K, rng.normal(0, 0.02, size=(n, k)).astype(np.float32)).reshape(-1, 144).copy()
    blocks[3, 0:2] = np.frombuffer(np.uint16(0x7E00).tobytes(), np.uint8)  # NaN d
    blocks[9, 2:4] = np.frombuffer(np.uint16(0x7C00).tobytes(), np.uint8)  # Inf dmin
    blocks = blocks.ravel()
    x = rng.normal(0, 1, size=(2, k)).astype(np.float32)
    rc, ref = O.fused_matmul(O.Q4K, blocks, x, 2, n, k)
    got = ctx.fused_dequant_matmul(O.Q4K, blocks, x, 2, n, k)
    assert np.all(np.isfinite(got))
    assert np.allclose(got, ref, rtol=1e-4, atol=1e-4)


def test_gemv_validation_errors(ctx, oracle):
    import realm_b200 as rb
    blocks = np.zeros(144, np.uint8)
    with pytest.raises(rb.RealmError) as e:
        ctx.fused_dequant_matmul(rb.Q4_K, blocks, np.zeros(256, np.float32), 1, 1, 100)
    assert e.value.code == -23
    with pytest.raises(rb.RealmError) as e:
        ctx.fused_dequant_matmul(rb.Q4_K, blocks, np.zeros(256, np.float32), 1, 2, 256)
    assert e.value.code == -3
    with pytest.raises(rb.RealmError) as e:
        ctx.fused_dequant_matmul(rb.Q8_0, np.zeros(34, np.uint8), np.zeros(32, np.float32), 1, 2, 32)
    assert e.value.code == -3


def test_weight_resident_matmul_batches_over_64(ctx, oracle):
    O = oracle
    import realm_b200 as rb
    rng = np.random.default_rng(21)
    n, k = 256, 512
    blocks = O.quantize(O.Q4K, rng.normal(0, 0.02, size=(n, k)).astype(np.float32))
    w = rb.Weight(ctx, rb.Q4_K, n, k, blocks)
    x = rng.normal(0, 1, size=(100, k)).astype(np.float32)
    got = w.matmul(x, 100)
    _check_gemv(O, O.Q4K, blocks, x, got, 100, n, k)
    w.free()


def test_candle_matmul(ctx):
    rng = np.random.default_rng(3)
    a = rng.normal(size=(37, 70)).astype(np.float32)
    b = rng.normal(size=(70, 45)).astype(np.float32)
    c = ctx.candle_matmul(a, b, 37, 70, 45)
    assert np.allclose(c, a @ b, rtol=1e-4, atol=1e-4)
    ct = ctx.candle_matmul(a, np.ascontiguousarray(b.T), 37, 70, 45, transposed=True)
    assert np.allclose(ct, a @ b, rtol=1e-4, atol=1e-4)
