"""GPU parity: paged KV append/gather (bit-exact) and paged GQA decode attention.

Oracle: KVCache (crates/realm-models/src/kv_cache.rs:7-80) and compute_attention /
StandardAttention (attention.rs:310-380, attention_stub/mod.rs:42-158) restated in
oracle/oracle.cpp. Attention tolerance: max-abs 2e-3 and relative 1e-3 (the
north star's bound); observed errors are ~1e-6.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kv_dtype", ["f32", "f16"])
def test_kv_append_gather_bit_exact(ctx, oracle, kv_dtype):
    import realm_b200 as rb
    O = oracle
    n_kv, hd, max_seq = 4, 64, 100
    f16 = kv_dtype == "f16"
    cache = rb.KVCache(ctx, max_seq, n_kv, hd, rb.F16 if f16 else rb.F32)
    ref = O.KVCache(max_seq, n_kv, hd, kv_fp16=f16)
    rng = np.random.default_rng(1)
    for s in (1, 7, 16, 9, 33):  # ragged appends crossing page boundaries
        k = rng.normal(size=s * n_kv * hd).astype(np.float32)
        v = rng.normal(size=s * n_kv * hd).astype(np.float32)
        gk, gv = cache.append(k, v)
        ref.append(k, v)
        rk, rv = ref.current_data()
        assert cache.current_seq_len == ref.current_seq_len
        assert np.array_equal(gk.view(np.uint32), rk.view(np.uint32))
        assert np.array_equal(gv.view(np.uint32), rv.view(np.uint32))
    # overflow: kv_cache.rs:48-53
    with pytest.raises(rb.RealmError) as e:
        cache.append(np.zeros(40 * n_kv * hd, np.float32), np.zeros(40 * n_kv * hd, np.float32))
    assert e.value.code == -22
    cache.clear()
    assert cache.current_seq_len == 0
    assert cache.current_data()[0].size == 0


def test_kv_pool_exhaustion_and_release(ctx):
    import realm_b200 as rb
    pool = ctx.kv_pool(1, 2, 64, rb.F16, n_pages=4, max_tenants=4, max_seq=256)
    pool.create(0)
    pool.create(1)
    z = np.zeros(48 * 2 * 64, np.float32)
    pool.append(0, 0, z, z)          # 3 pages
    with pytest.raises(rb.RealmError) as e:
        pool.append(1, 0, z, z)      # needs 3 more, only 1 left
    assert e.value.code == -21
    assert pool.len(1, 0) == 0       # all-or-nothing
    pool.clear(0)
    assert pool.free_pages() == 4
    pool.append(1, 0, z, z)
    assert pool.len(1, 0) == 48


def _oracle_attn(O, k_all, v_all, q, pos, n_heads, n_kv, hd):
    return O.attention(q, k_all, v_all, 1, pos + 1, pos, n_heads, n_kv, hd)


@pytest.mark.parametrize("n_heads,n_kv,hd,kv_dtype", [
    (32, 8, 128, "f16"),   # config 2 shape (GQA 4)
    (32, 32, 128, "f16"),  # Llama-2-7B (MHA)
    (32, 4, 64, "f32"),    # TinyLlama (GQA 8, fp32 KV as the reference)
    (16, 8, 64, "f16"),    # GQA 2
])
def test_paged_attention_vs_oracle(ctx, oracle, n_heads, n_kv, hd, kv_dtype):
    import realm_b200 as rb
    O = oracle
    rng = np.random.default_rng(n_heads * 7 + hd)
    f16 = kv_dtype == "f16"
    lens = [1, 15, 16, 17, 255, 256, 257, 700]  # page and split edges
    pool = ctx.kv_pool(2, n_kv, hd, rb.F16 if f16 else rb.F32, n_pages=sum((l + 16) // 16 + 1 for l in lens) + 4,
                       max_tenants=len(lens), max_seq=1024)
    pool.shuffle(99)  # permuted physical pages
    refs = []
    for t, L in enumerate(lens):
        pool.create(t)
        k = rng.normal(size=(L, n_kv, hd)).astype(np.float32)
        v = rng.normal(size=(L, n_kv, hd)).astype(np.float32)
        pool.append(t, 1, k, v)
        ref = O.KVCache(1024, n_kv, hd, kv_fp16=f16)
        ref.append(k, v)
        refs.append(ref)
    q = rng.normal(size=(len(lens), n_heads * hd)).astype(np.float32)
    scale = 1.0 / np.sqrt(hd)
    out = pool.attention_forward(1, list(range(len(lens))), q, n_heads, scale)
    for t, L in enumerate(lens):
        rk, rv = refs[t].current_data()
        exp = _oracle_attn(O, rk, rv, q[t], L - 1, n_heads, n_kv, hd)
        err = np.abs(out[t] - exp)
        assert err.max() <= 2e-3 and np.all(err <= 1e-3 * np.abs(exp) + 2e-5), (t, L, err.max())
    # attend to an earlier position (causal mask j > position)
    out2 = pool.attention_forward(1, [7], q[7:8], n_heads, scale, positions=[300])
    rk, rv = refs[7].current_data()
    exp = _oracle_attn(O, rk[:301 * n_kv * hd], rv[:301 * n_kv * hd], q[7], 300, n_heads, n_kv, hd)
    assert np.abs(out2[0] - exp).max() < 2e-5


def test_attention_append_then_attend(ctx, oracle):
    """Config-2 step: append one token per tenant, then attend over the full context."""
    import realm_b200 as rb
    O = oracle
    n_heads, n_kv, hd = 32, 8, 128
    rng = np.random.default_rng(2)
    lens = [40, 513]
    pool = ctx.kv_pool(1, n_kv, hd, rb.F16, n_pages=64, max_tenants=2, max_seq=1024)
    refs = []
    for t, L in enumerate(lens):
        pool.create(t)
        k = rng.normal(size=(L, n_kv, hd)).astype(np.float32)
        v = rng.normal(size=(L, n_kv, hd)).astype(np.float32)
        pool.append(t, 0, k, v)
        r = O.KVCache(1024, n_kv, hd, kv_fp16=True)
        r.append(k, v)
        refs.append(r)
    kn = rng.normal(size=(2, n_kv * hd)).astype(np.float32)
    vn = rng.normal(size=(2, n_kv * hd)).astype(np.float32)
    q = rng.normal(size=(2, n_heads * hd)).astype(np.float32)
    out = pool.attention_forward(0, [0, 1], q, n_heads, 1 / np.sqrt(hd), positions=lens, k_new=kn, v_new=vn)
    for t, L in enumerate(lens):
        refs[t].append(kn[t], vn[t])
        rk, rv = refs[t].current_data()
        exp = _oracle_attn(O, rk, rv, q[t], L, n_heads, n_kv, hd)
        assert np.abs(out[t] - exp).max() < 2e-5
        gk, gv = pool.gather(t, 0)
        assert np.array_equal(gk.view(np.uint32), rk.view(np.uint32))


@pytest.mark.parametrize("n_heads,n_kv,hd,kv_dtype", [
    (32, 32, 128, "f16"),  # MHA: 4 rows per pair
    (16, 8, 64, "f16"),    # GQA 2: 2 rows per pair
    (32, 8, 128, "f16"),   # GQA 4: one row per pair (hi and lo query parts packed)
    (32, 4, 64, "f16"),    # GQA 8, hd 64: the prompt-chunk kernel
    (64, 8, 128, "f16"),   # GQA 8, hd 128 (configs[4] heads): the prompt-chunk kernel
    (32, 4, 64, "f32"),    # fp32 pools: one row per pair
])
def test_prompt_chunk_rows_share_pages(ctx, oracle, n_heads, n_kv, hd, kv_dtype):
    """Consecutive rows of one tenant (a prompt chunk) attend as a group: each row
    still sees exactly positions [0, its own position] (per-column causal mask)."""
    import realm_b200 as rb
    O = oracle
    rng = np.random.default_rng(n_kv * 13 + hd)
    f16 = kv_dtype == "f16"
    L = 300
    pool = ctx.kv_pool(1, n_kv, hd, rb.F16 if f16 else rb.F32, n_pages=3 * (L // 16 + 2), max_tenants=3,
                       max_seq=512)
    pool.shuffle(5)
    ks, vs = [], []
    for t in range(3):
        pool.create(t)
        k = rng.normal(size=(L, n_kv, hd)).astype(np.float32)
        v = rng.normal(size=(L, n_kv, hd)).astype(np.float32)
        pool.append(t, 0, k, v)
        r = O.KVCache(512, n_kv, hd, kv_fp16=f16)
        r.append(k, v)
        ks.append(r)
    # tenant 0: 13 rows at positions 15..27 (a page edge inside), tenant 1: 6 rows
    # ending at the last position, tenant 2: one row, then tenant 0 again (new group)
    tenants = [0] * 13 + [1] * 6 + [2] + [0] * 3
    positions = list(range(15, 28)) + list(range(L - 6, L)) + [7] + [100, 101, 103]
    q = rng.normal(size=(len(tenants), n_heads * hd)).astype(np.float32)
    out = pool.attention_forward(0, tenants, q, n_heads, 1 / np.sqrt(hd), positions=positions)
    for i, (t, p) in enumerate(zip(tenants, positions)):
        rk, rv = ks[t].current_data()
        n = (p + 1) * n_kv * hd
        exp = _oracle_attn(O, rk[:n], rv[:n], q[i], p, n_heads, n_kv, hd)
        err = np.abs(out[i] - exp)
        assert err.max() <= 2e-3 and np.all(err <= 1e-3 * np.abs(exp) + 2e-5), (i, t, p, err.max())


@pytest.mark.parametrize("n_heads,n_kv,hd", [(32, 8, 128), (64, 8, 128), (32, 4, 64)])
def test_prompt_chunk_kernel_long_chunk(ctx, oracle, n_heads, n_kv, hd):
    """A 61-row prompt chunk deep into a long context (several 64-vector tiles
    per kv head, ~60 pages, split into segments over CTAs and merged) beside
    decode rows of other tenants in one call: at GQA 8 the chunk rows run on the
    prompt-chunk kernel and the others on the decode kernel; every row against
    the oracle at the attention bound."""
    import realm_b200 as rb
    O = oracle
    rng = np.random.default_rng(hd + n_heads)
    L = 1000
    pool = ctx.kv_pool(1, n_kv, hd, rb.F16, n_pages=3 * (L // 16 + 2), max_tenants=3, max_seq=1024)
    pool.shuffle(9)
    ks = []
    for t in range(3):
        pool.create(t)
        k = rng.normal(size=(L, n_kv, hd)).astype(np.float32)
        v = rng.normal(size=(L, n_kv, hd)).astype(np.float32)
        pool.append(t, 0, k, v)
        r = O.KVCache(1024, n_kv, hd, kv_fp16=True)
        r.append(k, v)
        ks.append(r)
    tenants = [1] + [0] * 61 + [2, 1]
    positions = [500] + list(range(L - 61, L)) + [L - 1, 17]
    q = rng.normal(size=(len(tenants), n_heads * hd)).astype(np.float32)
    out = pool.attention_forward(0, tenants, q, n_heads, 1 / np.sqrt(hd), positions=positions)
    assert ctx.last_forward_launches() == (2 if n_heads // n_kv == 8 else 1)
    for i, (t, p) in enumerate(zip(tenants, positions)):
        rk, rv = ks[t].current_data()
        n = (p + 1) * n_kv * hd
        exp = _oracle_attn(O, rk[:n], rv[:n], q[i], p, n_heads, n_kv, hd)
        err = np.abs(out[i] - exp)
        assert err.max() <= 2e-3 and np.all(err <= 1e-3 * np.abs(exp) + 2e-5), (i, t, p, err.max())
