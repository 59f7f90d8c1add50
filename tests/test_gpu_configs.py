"""GPU parity at the benchmarked configurations' own shapes.

Each case here runs a geometry that the bench times (or that config 5 needs)
against the oracle, on the same seeded inputs as the bench:

- configs[3] (Llama-2-7B Q4_K_M, 8 tenants, fp16 paged KV, prompts U[128, 512]
  from seed 4): the full-width model (hidden 4096, 32 MHA heads x 128, FFN 11008,
  vocab 32000) with 2 of its 32 layers, so the oracle (model.rs:572-625 restated)
  finishes in well under a minute. Prompts are prefilled in 64-row steps, then
  16 batched decode steps of all 8 tenants are teacher-forced on the oracle's
  greedy tokens.
- configs[1] (paged attention microbench): exactly the bench's inputs, 16
  tenants, 32 q / 8 kv heads, hd 128, contexts U[512, 8192] from seed 2,
  permuted pages, one appended token each. Pairs of up to 513 pages take the
  stream-K split and the cross-CTA merge.
- configs[4]'s attention geometry: 64 q / 8 kv heads (GQA 8) at hd 128, fp16.
- Attention steps with more (row group, kv head) pairs than CTAs, where one CTA
  takes several whole pairs (decode rows and prompt-chunk groups mixed).
- Activations with outlier channels 100-1000x the median (as real Llama hidden
  states carry), in the Q4_K GEMV and through a model whose norm weights make
  them, at the absolute logits bound.

Bounds (north star): logits and attention |err| <= 2e-3 + 1e-3 |ref|
elementwise; greedy-argmax agreement >= 99 %.
"""
import os

import numpy as np
import pytest

import synth

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-3


def _assert_close(got, ref, what):
    assert np.all(np.isfinite(got)) and np.all(np.isfinite(ref)), (what, "non-finite values")
    err = np.abs(np.asarray(got, np.float64) - np.asarray(ref, np.float64))
    bound = ATOL + RTOL * np.abs(np.asarray(ref, np.float64))
    bad = err > bound
    assert not bad.any(), (what, float(err.max()), int(bad.sum()), np.unravel_index(np.argmax(err - bound), err.shape))


# ---------------------------------------------------------------------------
# Llama-2-7B geometry, 8 tenants
# ---------------------------------------------------------------------------
def test_config4_geometry_teacher_forced(ctx, oracle):
    import realm_b200 as rb
    O = oracle
    cfg = dict(synth.LLAMA7B, n_layers=2, max_seq=1024)
    W = synth.make_weights(cfg, seed=4)
    rng = np.random.default_rng(4)
    lens = rng.integers(128, 513, 8)
    prompts = [rng.integers(0, cfg["vocab"], int(n)).astype(np.uint32) for n in lens]
    n_dec = 16
    # oracle: each tenant alone (the reference serves one tenant per model instance)
    ref_tok, ref_lg, ref_prompt_lg = [], [], []
    for p in prompts:
        om = O.Model(dict(cfg, kv_fp16=1), W)
        for cs in range(0, len(p), 64):
            lg = om.forward(p[cs:cs + 64], cs)
        ref_prompt_lg.append(lg.copy())
        toks, lgs = [O.argmax(lg)], [lg.copy()]
        pos = len(p)
        for _ in range(n_dec - 1):
            lg = om.forward([toks[-1]], pos)
            pos += 1
            toks.append(O.argmax(lg))
            lgs.append(lg.copy())
        ref_tok.append(toks)
        ref_lg.append(np.stack(lgs))
        del om
    m = rb.Model(ctx, dict(cfg, kv_dtype=rb.F16, max_tenants=8))
    m.set_weights(W)
    for t, p in enumerate(prompts):
        m.tenant_create(t)
        for cs in range(0, len(p), 64):
            lg, am = m.forward_rows([t] * len(p[cs:cs + 64]), p[cs:cs + 64])
        _assert_close(lg[-1], ref_prompt_lg[t], ("prompt", t))
        assert int(am[-1]) == ref_tok[t][0]
    agree, total = 0, 0
    for g in range(1, n_dec):
        lg, am = m.forward_rows(list(range(8)), [ref_tok[t][g - 1] for t in range(8)])
        for t in range(8):
            _assert_close(lg[t], ref_lg[t][g], ("decode", g, t))
            agree += int(am[t] == ref_tok[t][g])
            total += 1
    assert agree / total >= 0.99, (agree, total)
    m.close()


# ---------------------------------------------------------------------------
# attention
# ---------------------------------------------------------------------------
def _fill_pool(rb, O, ctx, lens, n_kv, hd, rng, shuffle_seed, max_seq, extra_pages=16):
    pool = ctx.kv_pool(1, n_kv, hd, rb.F16, n_pages=int(sum((L + 17) // 16 for L in lens)) + extra_pages,
                       max_tenants=len(lens), max_seq=max_seq)
    pool.shuffle(shuffle_seed)
    refs = []
    for t, L in enumerate(lens):
        pool.create(t)
        k = rng.normal(size=(int(L), n_kv * hd)).astype(np.float32)
        v = rng.normal(size=(int(L), n_kv * hd)).astype(np.float32)
        pool.append(t, 0, k, v)
        r = O.KVCache(max_seq, n_kv, hd, kv_fp16=True)
        r.append(k, v)
        refs.append(r)
    return pool, refs


def test_config2_attention_exact(ctx, oracle):
    """configs[1] as the bench runs it: append one token per tenant, attend over
    the whole context (stream-K split and merge at up to 513 pages per pair)."""
    import realm_b200 as rb
    O = oracle
    rng = np.random.default_rng(2)
    n_t, hq, hkv, hd = 16, 32, 8, 128
    ctxs = rng.integers(512, 8193, n_t)
    assert ctxs.max() > 4096
    pool, refs = _fill_pool(rb, O, ctx, ctxs, hkv, hd, rng, 2, 8208)
    q = rng.normal(size=(n_t, hq * hd)).astype(np.float32)
    kn = rng.normal(size=(n_t, hkv * hd)).astype(np.float32)
    vn = rng.normal(size=(n_t, hkv * hd)).astype(np.float32)
    scale = 1.0 / np.sqrt(hd)
    out = pool.attention_forward(0, list(range(n_t)), q, hq, scale, positions=[int(c) for c in ctxs],
                                 k_new=kn, v_new=vn)
    for t in range(n_t):
        refs[t].append(kn[t], vn[t])
        rk, rv = refs[t].current_data()
        exp = O.attention(q[t], rk, rv, 1, int(ctxs[t]) + 1, int(ctxs[t]), hq, hkv, hd)
        _assert_close(out[t], exp, ("tenant", t, int(ctxs[t])))
    # the appended rows are bit-exact in the pool
    for t in (0, n_t - 1):
        gk, gv = pool.gather(t, 0)
        rk, rv = refs[t].current_data()
        assert np.array_equal(gk.view(np.uint32), rk.view(np.uint32))


def test_config5_attention_gqa8_hd128(ctx, oracle):
    """configs[4]'s attention geometry: 64 q / 8 kv heads (n_rep 8), hd 128, fp16 K/V,
    contexts around 4096 (3840-token prompt plus decode) and page edges."""
    import realm_b200 as rb
    O = oracle
    rng = np.random.default_rng(5)
    hq, hkv, hd = 64, 8, 128
    lens = [1, 16, 17, 3840, 3841, 4095, 4096, 2000]
    pool, refs = _fill_pool(rb, O, ctx, lens, hkv, hd, rng, 5, 4112)
    q = rng.normal(size=(len(lens), hq * hd)).astype(np.float32)
    scale = 1.0 / np.sqrt(hd)
    out = pool.attention_forward(0, list(range(len(lens))), q, hq, scale, positions=[L - 1 for L in lens])
    for t, L in enumerate(lens):
        rk, rv = refs[t].current_data()
        exp = O.attention(q[t], rk, rv, 1, L, L - 1, hq, hkv, hd)
        _assert_close(out[t], exp, ("tenant", t, L))


def _many_pairs_case(rb, O, ctx, hq, hkv, hd, seed):
    rng = np.random.default_rng(seed)
    n_t = 44  # + 18 prompt-chunk rows = 62 rows (the step limit is 64)
    lens = rng.integers(20, 700, n_t)
    pool, refs = _fill_pool(rb, O, ctx, lens, hkv, hd, rng, seed, 1024)
    # one decode row per tenant at its last position, plus prompt-chunk groups:
    # tenant 3 rows at 10..22, tenant 40 rows at its last 5 positions
    tenants = list(range(n_t)) + [3] * 13 + [40] * 5
    positions = [int(L) - 1 for L in lens] + list(range(10, 23)) + list(range(int(lens[40]) - 5, int(lens[40])))
    q = rng.normal(size=(len(tenants), hq * hd)).astype(np.float32)
    return pool, refs, tenants, positions, q


@pytest.mark.parametrize("hq,hkv", [(32, 8), (32, 32)])
def test_attention_more_pairs_than_ctas(ctx, oracle, hq, hkv):
    """More (row group, kv head) pairs than CTAs: whole pairs, several per CTA, in
    floor-split ranges that differ in length. Checked against the oracle, and
    against even page splitting (RB_ATTN_WHOLE=0) on a second context."""
    import realm_b200 as rb
    O = oracle
    hd = 128
    pool, refs, tenants, positions, q = _many_pairs_case(rb, O, ctx, hq, hkv, hd, 31 + hkv)
    assert len(tenants) * hkv > 2 * ctx.num_sms  # pairs > CTAs (decode rows alone)
    scale = 1.0 / np.sqrt(hd)
    out = pool.attention_forward(0, tenants, q, hq, scale, positions=positions)
    for i, (t, p) in enumerate(zip(tenants, positions)):
        rk, rv = refs[t].current_data()
        n = (p + 1) * hkv * hd
        exp = O.attention(q[i], rk[:n], rv[:n], 1, p + 1, p, hq, hkv, hd)
        _assert_close(out[i], exp, ("row", i, t, p))
    os.environ["RB_ATTN_WHOLE"] = "0"
    try:
        c2 = rb.Context(0)
    finally:
        del os.environ["RB_ATTN_WHOLE"]
    try:
        pool2, _, tenants2, positions2, q2 = _many_pairs_case(rb, O, c2, hq, hkv, hd, 31 + hkv)
        out2 = pool2.attention_forward(0, tenants2, q2, hq, scale, positions=positions2)
        err = np.abs(out2 - out)
        assert err.max() < 1e-5, err.max()
    finally:
        c2.close()


# ---------------------------------------------------------------------------
# outlier channels
# ---------------------------------------------------------------------------
def _outlier_rows(rng, m, k, n_out=4):
    x = rng.normal(0, 1, size=(m, k)).astype(np.float32)
    for r in range(m):
        ch = rng.choice(k, n_out, replace=False)
        x[r, ch] = (rng.uniform(100, 1000, n_out) * rng.choice([-1, 1], n_out)).astype(np.float32)
    return x


@pytest.mark.parametrize("fmt", ["q4k", "q6k", "q80"])
@pytest.mark.parametrize("m", [1, 8, 16, 64])
def test_gemv_outlier_activations_absolute_bound(ctx, oracle, fmt, m):
    """Rows with a few channels 100-1000x the median: the int8 three-limb (Q4_K)
    and fp16 hi/lo (Q6_K, Q8_0) activations still meet the absolute bound
    2e-3 + 1e-3 |y| against the oracle's dequant + GEMM in double."""
    O = oracle
    dt = {"q4k": O.Q4K, "q6k": O.Q6K, "q80": O.Q80}[fmt]
    rng = np.random.default_rng(77 + m)
    n, k = 4096, 4096
    blocks = O.quantize(dt, rng.normal(0, 0.02, size=(n, k)).astype(np.float32))
    x = _outlier_rows(rng, m, k)
    got = ctx.fused_dequant_matmul(dt, blocks, x, m, n, k)
    ref = O.dequant_matmul(dt, blocks, x, m, n, k, f64=True)
    _assert_close(got, ref, (fmt, m))


def test_model_outlier_channels_teacher_forced(ctx, oracle):
    """A model whose norm weights carry a few channels at 100-1000x (so every
    GEMV input has outlier channels, as real Llama hidden states do), decoded
    against the oracle at the logits bound."""
    import realm_b200 as rb
    O = oracle
    cfg = dict(synth.TINYLLAMA, n_layers=2, max_seq=256)
    W = synth.make_weights(cfg, seed=9)
    rng = np.random.default_rng(9)
    H = cfg["hidden"]
    for l in range(cfg["n_layers"]):
        for which in (O.W_ATTN_NORM, O.W_FFN_NORM):
            w = np.ones(H, np.float32)
            ch = rng.choice(H, 6, replace=False)
            w[ch] = rng.uniform(100, 1000, 6).astype(np.float32)
            W[(which, l)] = (O.F32, w)
    prompt = rng.integers(0, cfg["vocab"], 37).astype(np.uint32)
    om = O.Model(dict(cfg, kv_fp16=1), W)
    toks, ref_logits = om.generate(prompt, 12)
    m = rb.Model(ctx, dict(cfg, kv_dtype=rb.F16, max_tenants=1))
    m.set_weights(W)
    m.tenant_create(0)
    for cs in range(0, len(prompt), 8):
        lg, am = m.forward_rows([0] * len(prompt[cs:cs + 8]), prompt[cs:cs + 8])
    agree = 0
    for g in range(len(toks)):
        if g > 0:
            lg, am = m.forward_rows([0], [toks[g - 1]])
        _assert_close(lg[-1], ref_logits[g], ("step", g))
        agree += int(am[-1] == toks[g])
    assert agree / len(toks) >= 0.99
    m.close()


# ---------------------------------------------------------------------------
# Llama-2-70B geometry
# ---------------------------------------------------------------------------
LLAMA70B = dict(n_layers=80, hidden=8192, n_heads=64, n_kv_heads=8, head_dim=128, ffn=28672, vocab=32000,
                max_seq=4096, rms_eps=1e-5, layer_eps=1e-5, rope_theta=10000.0)


def test_config5_geometry_one_layer_teacher_forced(ctx, oracle):
    """The 70B layer geometry (hidden 8192, 64 q / 8 kv heads of 128, FFN 28672 =
    112 super-blocks, GQA 8 in the model path, fp16 KV) with 1 of its 80 layers:
    4 tenants with prompts prefilled in 64-row steps, then 8 batched decode
    steps teacher-forced on the oracle's greedy tokens."""
    import realm_b200 as rb
    O = oracle
    cfg = dict(LLAMA70B, n_layers=1, max_seq=512)
    W = synth.make_weights(cfg, seed=5)
    rng = np.random.default_rng(5)
    lens = rng.integers(60, 200, 4)
    prompts = [rng.integers(0, cfg["vocab"], int(n)).astype(np.uint32) for n in lens]
    n_dec = 8
    ref_tok, ref_lg = [], []
    for p in prompts:
        om = O.Model(dict(cfg, kv_fp16=1), W)
        for cs in range(0, len(p), 64):
            lg = om.forward(p[cs:cs + 64], cs)
        toks, lgs = [O.argmax(lg)], [lg.copy()]
        pos = len(p)
        for _ in range(n_dec - 1):
            lg = om.forward([toks[-1]], pos)
            pos += 1
            toks.append(O.argmax(lg))
            lgs.append(lg.copy())
        ref_tok.append(toks)
        ref_lg.append(np.stack(lgs))
        del om
    m = rb.Model(ctx, dict(cfg, kv_dtype=rb.F16, max_tenants=4))
    m.set_weights(W)
    del W
    for t, p in enumerate(prompts):
        m.tenant_create(t)
        for cs in range(0, len(p), 64):
            lg, am = m.forward_rows([t] * len(p[cs:cs + 64]), p[cs:cs + 64])
        _assert_close(lg[-1], ref_lg[t][0], ("prompt", t))
    agree, total = 0, 0
    for g in range(1, n_dec):
        lg, am = m.forward_rows(list(range(4)), [ref_tok[t][g - 1] for t in range(4)])
        for t in range(4):
            _assert_close(lg[t], ref_lg[t][g], ("decode", g, t))
            agree += int(am[t] == ref_tok[t][g])
            total += 1
    assert agree / total >= 0.99, (agree, total)
    m.close()
