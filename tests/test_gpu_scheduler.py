"""GPU parity of the continuous-batching scheduler (rb_scheduler_*).

Requests of different prompt lengths join while others decode, prompts are fed
in chunks next to decode rows, and requests leave at max_tokens / eos /
max_seq_len or by cancel. Every token a request gets is checked against the
oracle's Model::forward (crates/realm-models/src/model.rs:572-625) run on that
request alone, teacher-forced on the scheduler's own tokens. Bound (north star):
logits |err| <= 2e-3 + 1e-3 |ref| elementwise; the emitted token is the argmax
of its logits row (ties -> last) and equals the oracle's argmax wherever the
oracle's top-2 margin exceeds the logits bound.
"""
import numpy as np
import pytest

import synth

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-3


@pytest.fixture(scope="module")
def small(oracle):
    cfg = synth.SMALL
    return cfg, synth.make_weights(cfg, seed=0)


def _model(ctx, cfg, W, **kw):
    import realm_b200 as rb
    m = rb.Model(ctx, dict(cfg, kv_dtype=rb.F16, **kw))
    m.set_weights(W)
    return m


def _oracle_check(O, cfg, W, prompt, toks, logits):
    """Teacher-forced oracle run of one request; returns the number of compared steps."""
    om = O.Model(dict(cfg, kv_fp16=1), W)
    ref = om.forward(np.asarray(prompt, np.uint32), 0)
    pos = len(prompt)
    for i, (t, lg) in enumerate(zip(toks, logits)):
        if i > 0:
            ref = om.forward(np.asarray([toks[i - 1]], np.uint32), pos)
            pos += 1
        err = np.abs(lg - ref)
        assert np.all(err <= ATOL + RTOL * np.abs(ref)), (i, err.max())
        assert t == len(lg) - 1 - int(np.argmax(lg[::-1])), i       # argmax, ties -> last
        top2 = np.sort(ref)[-2:]
        if top2[1] - top2[0] > 2 * (ATOL + RTOL * abs(top2[1])):
            assert t == int(np.argmax(ref)), (i, t, int(np.argmax(ref)))
    return len(toks)


def test_scheduler_matches_oracle_with_joins_and_chunked_prefill(ctx, oracle, small):
    import realm_b200 as rb
    cfg, W = small
    m = _model(ctx, cfg, W, max_tenants=8)
    free0 = m.kv.free_pages()
    rng = np.random.default_rng(3)
    plens = [1, 5, 17, 40, 70, 3, 33, 9]
    maxt = [1, 6, 9, 4, 7, 12, 5, 8]
    prompts = {i: rng.integers(0, cfg["vocab"], n).tolist() for i, n in enumerate(plens)}
    s = rb.Scheduler(m, max_batch_size=4, prefill_chunk=16)
    toks = {i: [] for i in prompts}
    lgs = {i: [] for i in prompts}
    for i in range(5):
        s.submit(i, prompts[i], maxt[i])
    step = 0
    live_max = 0
    while True:
        if step == 3:                       # join while others decode
            for i in (5, 6, 7):
                s.submit(i, prompts[i], maxt[i])
        st = s.stats()
        if st["queued"] == 0 and st["live"] == 0 and step > 3:
            break
        ev, lg = s.step(want_logits=True)
        live_max = max(live_max, s.stats()["live"] + sum(e.finish is not None for e in ev))
        for e, row in zip(ev, lg):
            assert e.index == len(toks[e.request_id])
            toks[e.request_id].append(e.token)
            lgs[e.request_id].append(row)
        step += 1
        assert step < 200
    assert live_max <= 4
    n = 0
    for i in prompts:
        got, fin = s.result(i)
        assert got == toks[i] and len(got) == maxt[i] and fin == "max_tokens", (i, fin)
        n += _oracle_check(oracle, cfg, W, prompts[i], toks[i], lgs[i])
    assert n == sum(maxt)
    st = s.stats()
    assert st["tokens_generated"] == sum(maxt) and st["prefill_rows"] == sum(plens)
    assert st["decode_rows"] == sum(maxt) - len(maxt)
    assert m.kv.free_pages() == free0       # every page went back to the pool
    s.close()


def test_scheduler_eos_length_and_immediate_finishes(ctx, oracle, small):
    import realm_b200 as rb
    cfg, W = small
    m = _model(ctx, cfg, W, max_tenants=4)
    prompt = np.random.default_rng(4).integers(0, cfg["vocab"], 12).tolist()
    s = rb.Scheduler(m, max_batch_size=2)
    s.submit(1, prompt, 10)
    ref = s.run()[1]
    s.close()
    eos = ref[3]
    s = rb.Scheduler(m, max_batch_size=2, eos_token=eos, max_seq_len=len(prompt) + 6)
    s.submit(1, prompt, 10)                  # stops at the first eos
    s.submit(2, prompt[:5], 10)               # different prompt: its own tokens
    s.submit(3, prompt, 0)                    # finishes at once, no tokens
    s.submit(4, list(range(len(prompt) + 6)), 5)   # prompt >= max_seq_len: dropped
    out = s.run()
    k = ref.index(eos)
    assert s.result(1) == (ref[:k + 1], "eos")
    assert s.result(3) == ([], "max_tokens") and s.result(4) == ([], "length")
    assert 3 not in out and 4 not in out
    got2, fin2 = s.result(2)                  # 5 + 10 < max_seq_len: eos or max_tokens
    if fin2 == "eos":
        assert got2[-1] == eos and eos not in got2[:-1]
    else:
        assert fin2 == "max_tokens" and len(got2) == 10 and eos not in got2
    assert out[2] == got2
    s.close()
    s = rb.Scheduler(m, max_batch_size=2, max_seq_len=len(prompt) + 3)
    s.submit(1, prompt, 10)
    s.run()
    assert s.result(1) == (ref[:3], "length")   # prompt + 3 generated = max_seq_len
    s.close()


def test_scheduler_cancel_frees_pages_and_errors(ctx, oracle, small):
    import realm_b200 as rb
    cfg, W = small
    m = _model(ctx, cfg, W, max_tenants=4)
    free0 = m.kv.free_pages()
    s = rb.Scheduler(m, max_batch_size=2, prefill_chunk=8)
    rng = np.random.default_rng(5)
    s.submit(1, rng.integers(0, cfg["vocab"], 30).tolist(), 50)
    s.submit(2, rng.integers(0, cfg["vocab"], 4).tolist(), 50)
    s.submit(3, rng.integers(0, cfg["vocab"], 4).tolist(), 50)   # queued behind two live
    s.step()
    s.step()
    assert s.stats()["live"] == 2 and s.stats()["queued"] == 1
    s.cancel(3)                                # queued: ends now
    s.cancel(1)                                # live: retired by the next step
    assert s.result(3) == ([], "cancelled")
    s.step()
    assert s.result(1)[1] == "cancelled" and s.stats()["live"] == 1
    s.cancel(2)
    assert s.step() == [] and s.stats()["live"] == 0
    assert m.kv.free_pages() == free0
    with pytest.raises(rb.RealmError) as e:
        s.submit(2, [1, 2], 3)                 # id still known (finished)
    assert e.value.code == -3
    s.release(2)
    s.submit(2, [1, 2], 1)
    s.run()
    assert len(s.result(2)[0]) == 1
    with pytest.raises(rb.RealmError) as e:
        s.submit(9, [cfg["vocab"]], 3)         # token out of range
    assert e.value.code == -3
    with pytest.raises(rb.RealmError) as e:
        s.result(12345)
    assert e.value.code == -2
    with pytest.raises(rb.RealmError):
        rb.Scheduler(m, max_batch_size=65)
    with pytest.raises(rb.RealmError):
        rb.Scheduler(m, max_batch_size=2, tenant_base=3)   # tenants 3, 4 > max_tenants 4
    s.close()


def test_scheduler_admission_waits_for_kv_pages(ctx, oracle, small):
    """A pool of 12 pages (192 tokens) holds two requests of worst case 90 tokens
    (6 pages each) at a time; the others wait, then all finish with the oracle's tokens."""
    import realm_b200 as rb
    cfg, W = small
    m = _model(ctx, cfg, W, max_tenants=8, kv_pages=12)
    rng = np.random.default_rng(6)
    prompts = {i: rng.integers(0, cfg["vocab"], 80).tolist() for i in range(4)}
    s = rb.Scheduler(m, max_batch_size=8, prefill_chunk=32)
    for i in prompts:
        s.submit(i, prompts[i], 11)
    toks = {i: [] for i in prompts}
    lgs = {i: [] for i in prompts}
    for _ in range(100):
        st = s.stats()
        if st["live"] == 0 and st["queued"] == 0:
            break
        ev, lg = s.step(want_logits=True)
        assert s.stats()["live"] <= 2
        for e, row in zip(ev, lg):
            toks[e.request_id].append(e.token)
            lgs[e.request_id].append(row)
    for i in prompts:
        assert s.result(i)[1] == "max_tokens"
        _oracle_check(oracle, cfg, W, prompts[i], toks[i], lgs[i])
    with pytest.raises(rb.RealmError) as e:
        s.submit(99, list(range(150)), 100)     # worst case 249 tokens > 192 in the pool
    assert e.value.code == -21
    s.close()
