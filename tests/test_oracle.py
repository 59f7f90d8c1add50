"""CPU tests of the oracle (the parity checker) against the reference's own
known-answer and property tests, hand-derived KATs and an independent NumPy
restatement. No GPU needed.

Reference tests pinned here (paths relative to the reference project root):
  crates/realm-core/src/quant.rs:963-973      Q8_0 KAT (10 * 0.25 = 2.5)
  crates/realm-core/src/quant.rs:976-1032     Q4_K / Q6_K dequant patterns (exact values derived by hand)
  crates/realm-compute-cpu/src/fused.rs:2840-2915, 3483-3573, 3648-3726  fused vs dequant+matmul, rel < 1e-4
  crates/realm-compute-cpu/src/fused.rs:2978-3000, 3623-3646, 3924-3950  validation errors
  crates/realm-models/src/kv_cache.rs:44-70   append / overflow / current_data
  crates/realm-models/src/sampling.rs:141-148 argmax ties -> last index
"""
import struct

import numpy as np
import pytest


def f16(O, v):
    return O.f32_to_f16_bits(float(v))


def q4k_block(O, d, dmin, scales, qs):
    return np.frombuffer(struct.pack("<HH", f16(O, d), f16(O, dmin)) + bytes(scales) + bytes(qs), np.uint8)


def test_q8_0_kat(oracle):
    O = oracle
    b = np.frombuffer(struct.pack("<H", f16(O, 0.25)) + bytes([10] * 32), np.uint8)
    assert np.all(O.dequant(O.Q80, b) == 2.5)


def test_q4_k_kat(oracle):
    """quant.rs:976-999 pattern; exact values from get_scale_min_k4 by hand."""
    O = oracle
    y = O.dequant(O.Q4K, q4k_block(O, 1.0, 0.5, [0x11] * 12, [0x50] * 128))
    exp = np.concatenate([np.full(32, v, np.float32) for v in (-8.5, 76.5, -8.5, 76.5, -0.5, 4.5, -0.5, 4.5)])
    assert np.array_equal(y, exp)


def test_q6_k_kat(oracle):
    """quant.rs:1001-1032 pattern: everything -32 except element 64 (ql[0] >> 4 = 1) -> -31."""
    O = oracle
    ql = [0] * 128
    ql[0] = 0x10
    b = np.frombuffer(bytes(ql) + bytes(64) + bytes([1] * 16) + struct.pack("<H", f16(O, 1.0)), np.uint8)
    y = O.dequant(O.Q6K, b)
    exp = np.full(256, -32.0, np.float32)
    exp[64] = -31.0
    assert np.array_equal(y, exp)


def test_scale_min_k4_high_bits(oracle):
    """Sub-blocks 4..7 take their top two bits from bytes 0..7 (quant.rs:108-122)."""
    O = oracle
    scales = [0xC0 | 5, 0x40 | 6, 0x80 | 7, 0x00 | 8, 0xC0 | 9, 0x40 | 10, 0x80 | 11, 0x00 | 12,
              0x21, 0x43, 0x65, 0x87]
    y = O.dequant(O.Q4K, q4k_block(O, 1.0, 1.0, scales, [0x11] * 128)).reshape(8, 32)
    # element value with q = 1: sc - m
    sc = [5, 6, 7, 8, (0x21 & 0xF) | (3 << 4), (0x43 & 0xF) | (1 << 4), (0x65 & 0xF) | (2 << 4), (0x87 & 0xF) | 0]
    mn = [9, 10, 11, 12, (0x21 >> 4) | (3 << 4), (0x43 >> 4) | (1 << 4), (0x65 >> 4) | (2 << 4), (0x87 >> 4) | 0]
    order = [0, 1, 2, 3, 4, 5, 6, 7]
    for j in order:
        assert np.all(y[j] == np.float32(sc[j]) - np.float32(mn[j])), j


def test_f16_conversions_exact(oracle):
    O = oracle
    import ctypes as C
    L = O.lib()
    bits = np.arange(0, 65536, 97, dtype=np.uint16)
    for b in bits:
        ref = np.array([b], np.uint16).view(np.float16).astype(np.float32)[0]
        got = L.or_f16_to_f32(int(b))
        assert (np.isnan(ref) and np.isnan(got)) or ref == got
    rng = np.random.default_rng(0)
    xs = np.concatenate([rng.normal(0, 1, 2000), rng.normal(0, 1e-5, 2000), rng.normal(0, 1e4, 500),
                         [65504, 65520, 1e-8, 6e-8, 3e-8, -0.0]]).astype(np.float32)
    for x in xs:
        assert L.or_f32_to_f16(float(x)) == np.array([x], np.float32).astype(np.float16).view(np.uint16)[0], x


def _np_dequant(O, dt, blocks):
    """Independent NumPy restatement of the three block formats."""
    bb = O.BLOCK_BYTES[dt]
    B = blocks.reshape(-1, bb)
    h2f = lambda u8: u8.copy().view(np.uint16).view(np.float16).astype(np.float32)
    if dt == O.Q80:
        d = h2f(B[:, 0:2])
        return (B[:, 2:].view(np.int8).astype(np.float32) * d).ravel()
    if dt == O.Q4K:
        d, dmin = h2f(B[:, 0:2]), h2f(B[:, 2:4])
        s = B[:, 4:16].astype(np.int32)
        sc = np.zeros((len(B), 8), np.int32)
        mn = np.zeros((len(B), 8), np.int32)
        for j in range(8):
            if j < 4:
                sc[:, j], mn[:, j] = s[:, j] & 63, s[:, j + 4] & 63
            else:
                sc[:, j] = (s[:, j + 4] & 0xF) | ((s[:, j - 4] >> 6) << 4)
                mn[:, j] = (s[:, j + 4] >> 4) | ((s[:, j] >> 6) << 4)
        qs = B[:, 16:].astype(np.int32).reshape(-1, 4, 32)
        q = np.stack([qs & 0xF, qs >> 4], axis=2).reshape(-1, 256)  # [grp][lo|hi][32]
        d1 = (d * sc.astype(np.float32)).astype(np.float32)
        m1 = (dmin * mn.astype(np.float32)).astype(np.float32)
        d1 = np.repeat(d1, 32, axis=1)
        m1 = np.repeat(m1, 32, axis=1)
        return (d1 * q.astype(np.float32) - m1).astype(np.float32).ravel()
    # Q6_K
    ql, qh = B[:, :128].astype(np.int32), B[:, 128:192].astype(np.int32)
    sc = B[:, 192:208].view(np.int8).astype(np.float32)
    d = h2f(B[:, 208:210])
    out = np.zeros((len(B), 256), np.float32)
    for h in range(2):
        for t in range(4):
            l = np.arange(32)
            lo = ql[:, 64 * h + l + (32 if t & 1 else 0)]
            nib = (lo >> 4) if t & 2 else (lo & 0xF)
            hb = (qh[:, 32 * h + l] >> (2 * t)) & 3
            q = (nib | (hb << 4)) - 32
            e = 128 * h + 32 * t + l
            out[:, e] = (d * sc[:, e // 16]).astype(np.float32) * q.astype(np.float32)
    return out.ravel()


@pytest.mark.parametrize("name", ["q4k", "q6k", "q80"])
def test_dequant_matches_numpy_restatement(oracle, name):
    O = oracle
    dt = {"q4k": O.Q4K, "q6k": O.Q6K, "q80": O.Q80}[name]
    rng = np.random.default_rng(4)
    blocks = rng.integers(0, 256, 200 * O.BLOCK_BYTES[dt]).astype(np.uint8).reshape(200, -1)
    # finite scales
    if dt == O.Q4K:
        blocks[:, 0:4] = np.array([f16(O, 0.01), f16(O, 0.003)], np.uint16).view(np.uint8)
    elif dt == O.Q6K:
        blocks[:, 208:210] = np.array([f16(O, 0.002)], np.uint16).view(np.uint8)
    else:
        blocks[:, 0:2] = np.array([f16(O, 0.05)], np.uint16).view(np.uint8)
    blocks = blocks.ravel()
    assert np.array_equal(O.dequant(dt, blocks), _np_dequant(O, dt, blocks))


def test_fused_property_q4k(oracle):
    """fused.rs:2840-2915."""
    O = oracle
    blocks = b""
    for i in range(2):
        for j in range(2):
            blocks += q4k_block(O, 0.5 + i * 0.1, 0.1, [16 + i + j] * 12, [(i * 17 + j * 13) % 256] * 128).tobytes()
    blocks = np.frombuffer(blocks, np.uint8)
    x = np.array([((i % 7) - 3.0) * 0.5 for i in range(512)], np.float32)[None]
    rc, y = O.fused_matmul(O.Q4K, blocks, x, 1, 2, 512)
    ref = O.dequant(O.Q4K, blocks).reshape(2, 512) @ x[0]
    assert rc == 2 and np.all(np.abs(y[0] - ref) / np.abs(ref) < 1e-4)


def test_fused_property_q6k(oracle):
    """fused.rs:3483-3573."""
    O = oracle
    blocks = b""
    for i in range(2):
        for j in range(2):
            ql = bytes((i * 15 + j * 9 + idx) % 255 for idx in range(128))
            qh = bytes((i * 13 + j * 7 + idx) % 255 for idx in range(64))
            sc = np.array([((i * 9 + j * 5 + idx) % 127) - 64 for idx in range(16)], np.int8).tobytes()
            blocks += ql + qh + sc + struct.pack("<H", f16(O, 0.5 + i * 0.1))
    blocks = np.frombuffer(blocks, np.uint8)
    x = np.array([((i % 7) - 3.0) * 0.5 for i in range(512)], np.float32)[None]
    rc, y = O.fused_matmul(O.Q6K, blocks, x, 1, 2, 512)
    ref = O.dequant(O.Q6K, blocks).reshape(2, 512).astype(np.float64) @ x[0]
    assert rc == 2 and np.all(np.abs(y[0] - ref) / np.maximum(np.abs(ref), 1e-6) < 1e-4)


def test_fused_property_q80(oracle):
    """fused.rs:3648-3726."""
    O = oracle
    blocks = b""
    for i in range(2):
        for j in range(2):
            q = np.array([((i * 13 + j * 7 + idx) % 127) - 64 for idx in range(32)], np.int8).tobytes()
            blocks += struct.pack("<H", f16(O, 0.5 + i * 0.1)) + q
    blocks = np.frombuffer(blocks, np.uint8)
    x = np.array([((i % 7) - 3.0) * 0.5 for i in range(64)], np.float32)[None]
    rc, y = O.fused_matmul(O.Q80, blocks, x, 1, 2, 64)
    ref = O.dequant(O.Q80, blocks).reshape(2, 64).astype(np.float64) @ x[0]
    assert rc == 2 and np.all(np.abs(y[0] - ref) / np.maximum(np.abs(ref), 1e-6) < 1e-4)


def test_fused_validation(oracle):
    """fused.rs:2978-3000, 3623-3646, 3924-3950."""
    O = oracle
    x = np.zeros(256, np.float32)
    for dt in (O.Q4K, O.Q6K):
        one = np.zeros(O.BLOCK_BYTES[dt], np.uint8)
        assert O.fused_matmul(dt, one, x, 1, 1, 100)[0] < 0   # K not a multiple of 256
        assert O.fused_matmul(dt, one, x, 1, 2, 256)[0] < 0   # wrong block count
    one = np.zeros(34, np.uint8)
    assert O.fused_matmul(O.Q80, one, np.zeros(32, np.float32), 1, 2, 32)[0] < 0


@pytest.mark.parametrize("name", ["q4k", "q6k", "q80"])
def test_fused_matches_dequant_matmul(oracle, name):
    O = oracle
    dt = {"q4k": O.Q4K, "q6k": O.Q6K, "q80": O.Q80}[name]
    rng = np.random.default_rng(9)
    W = rng.normal(0, 0.02, (48, 768)).astype(np.float32)
    blocks = O.quantize(dt, W)
    x = rng.normal(0, 1, (3, 768)).astype(np.float32)
    rc1, y1 = O.fused_matmul(dt, blocks, x, 3, 48, 768, threads=1)
    rc2, y2 = O.fused_matmul(dt, blocks, x, 3, 48, 768, threads=4)
    assert np.array_equal(y1, y2)  # threading does not change the per-element order
    y3 = O.dequant_matmul(dt, blocks, x, 3, 48, 768, f64=True)
    assert np.abs(y1 - y3).max() < 1e-4 * np.abs(y3).max()


@pytest.mark.parametrize("name", ["q4k", "q6k", "q80"])
def test_quantizer_round_trip(oracle, name):
    O = oracle
    dt = {"q4k": O.Q4K, "q6k": O.Q6K, "q80": O.Q80}[name]
    rng = np.random.default_rng(10)
    W = rng.normal(0, 0.02, 256 * 64).astype(np.float32)
    err = np.abs(O.dequant(dt, O.quantize(dt, W)) - W).max()
    bound = {"q4k": 6e-3, "q6k": 2e-3, "q80": 5e-4}[name]
    assert err < bound, err


def test_kv_cache_semantics(oracle):
    O = oracle
    kv = O.KVCache(10, 2, 4)
    a = np.arange(3 * 8, dtype=np.float32)
    assert kv.append(a, -a) == 3
    assert kv.current_seq_len == 3
    assert kv.append(np.zeros(8 * 8, np.float32), np.zeros(8 * 8, np.float32)) == -22  # overflow
    k, v = kv.current_data()
    assert np.array_equal(k, a) and np.array_equal(v, -a)
    kv.clear()
    assert kv.current_seq_len == 0


def test_argmax_ties_last(oracle):
    assert oracle.argmax(np.array([1.0, 3.0, 2.0, 3.0, 0.5], np.float32)) == 3


def _np_attention(q, k, v, S, Lk, pos, nh, nkv, hd):
    q = q.reshape(S, nh, hd).astype(np.float64)
    k = k.reshape(Lk, nkv, hd).astype(np.float64)
    v = v.reshape(Lk, nkv, hd).astype(np.float64)
    rep = nh // nkv
    out = np.zeros((S, nh, hd))
    for h in range(nh):
        for i in range(S):
            s = k[:, h // rep] @ q[i, h] / np.sqrt(hd)
            s[np.arange(Lk) > pos + i] = -np.inf
            p = np.exp(s - s.max())
            out[i, h] = (p / p.sum()) @ v[:, h // rep]
    return out.ravel()


def test_attention_matches_numpy(oracle):
    O = oracle
    rng = np.random.default_rng(3)
    S, Lk, nh, nkv, hd, pos = 3, 20, 8, 2, 16, 17
    q = rng.normal(size=S * nh * hd).astype(np.float32)
    k = rng.normal(size=Lk * nkv * hd).astype(np.float32)
    v = rng.normal(size=Lk * nkv * hd).astype(np.float32)
    got = O.attention(q, k, v, S, Lk, pos, nh, nkv, hd)
    assert np.abs(got - _np_attention(q, k, v, S, Lk, pos, nh, nkv, hd)).max() < 1e-5


def test_rope_matches_numpy(oracle):
    O = oracle
    rng = np.random.default_rng(4)
    S, nh, hd, theta, p0 = 3, 2, 8, 10000.0, 5
    t = rng.normal(size=S * nh * hd).astype(np.float32)
    got = O.rope(t, p0, S, nh, hd, theta).reshape(S, nh, hd)
    ref = t.reshape(S, nh, hd).astype(np.float64).copy()
    for s in range(S):
        for i in range(0, hd, 2):
            ang = (p0 + s) / theta ** (i / hd)
            x0, x1 = ref[s, :, i].copy(), ref[s, :, i + 1].copy()
            ref[s, :, i] = x0 * np.cos(ang) - x1 * np.sin(ang)
            ref[s, :, i + 1] = x0 * np.sin(ang) + x1 * np.cos(ang)
    assert np.abs(got - ref).max() < 1e-5


def test_model_forward_consistency(oracle):
    """Chunked prefill + decode equals a single full forward (persistent KV)."""
    import synth
    O = oracle
    cfg = dict(synth.SMALL, n_layers=1)
    W = synth.make_weights(cfg, seed=1)
    ids = np.array([5, 9, 100, 7, 3], np.uint32)
    a = O.Model(cfg, W)
    full = a.forward(ids, 0)
    b = O.Model(cfg, W)
    b.forward(ids[:3], 0)
    step = b.forward(ids[3:], 3)
    assert np.abs(full - step).max() < 1e-5
    assert a.kv_len() == b.kv_len() == 5
