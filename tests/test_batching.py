"""ContinuousBatcher / BatchedRequest through the C ABI (rb_batcher_*), on CPU.

The cases restate the reference's unit tests of
crates/realm-runtime/src/batching.rs:222-355, its integration test
crates/realm-runtime/tests/integration_frameworks.rs:58-125 and
batch_forward.rs:193-208 (prepare_batch), plus the edge cases of the same rules.
"""
import threading

import pytest

import realm_b200 as rb
from realm_b200 import BatchedRequest, ContinuousBatcher, prepare_batch


def test_batcher_creation():
    assert ContinuousBatcher(32, 2048).active_count() == 0


def test_add_and_get_batch():
    b = ContinuousBatcher(32, 2048)
    b.add_request(BatchedRequest.new(1, [1, 2, 3], 100))
    b.add_request(BatchedRequest.new(2, [4, 5, 6], 100))
    batch = b.get_batch()
    assert [r.request_id for r in batch] == [1, 2]
    assert batch[0].prompt_tokens == [1, 2, 3] and batch[1].prompt_tokens == [4, 5, 6]
    assert batch[0].prompt_text is None


def test_update_request():
    b = ContinuousBatcher(32, 2048)
    b.add_request(BatchedRequest.new(1, [1, 2, 3], 100))
    b.update_request(1, 42)
    batch = b.get_batch()
    assert len(batch) == 1 and batch[0].generated_tokens == [42]


def test_complete_request():
    b = ContinuousBatcher(32, 2048)
    b.add_request(BatchedRequest.new(1, [1, 2, 3], 1))
    b.update_request(1, 42)
    assert b.active_count() == 0          # complete at max_tokens
    assert b.get_batch() == []


def test_batched_request_with_prompt_text():
    r = BatchedRequest.with_prompt_text(1, [1, 2, 3], "What is the capital of France?", 100)
    assert r.request_id == 1 and r.prompt_tokens == [1, 2, 3]
    assert r.prompt_text == "What is the capital of France?"
    assert r.max_tokens == 100 and not r.is_complete
    assert r.current_seq_len() == 3 and r.all_tokens() == [1, 2, 3]


def test_batch_stats():
    b = ContinuousBatcher(32, 2048)
    b.add_request(BatchedRequest.new(1, [1, 2, 3], 100))
    b.add_request(BatchedRequest.new(2, [4, 5, 6, 7], 100))
    s = b.stats()
    assert (s.total_requests, s.active_requests, s.average_sequence_length) == (2, 2, 3)  # 7 // 2


def test_batch_max_size():
    b = ContinuousBatcher(2, 2048)
    b.add_request(BatchedRequest.new(1, [1], 100))
    b.add_request(BatchedRequest.new(2, [2], 100))
    with pytest.raises(rb.RealmError) as e:
        b.add_request(BatchedRequest.new(3, [3], 100))
    assert e.value.code == -3 and "Batch queue is full" in str(e.value)


def test_batch_max_seq_len():
    b = ContinuousBatcher(32, 10)
    b.add_request(BatchedRequest.new(1, list(range(1, 12)), 100))
    assert b.get_batch() == []
    assert b.stats().total_requests == 0   # dropped, not kept


def test_remove_request():
    b = ContinuousBatcher(32, 2048)
    b.add_request(BatchedRequest.new(1, [1, 2, 3], 100))
    b.remove_request(1)
    assert b.active_count() == 0
    with pytest.raises(rb.RealmError) as e:
        b.remove_request(999)
    assert e.value.code == -2 and "Request 999 not found" in str(e.value)
    with pytest.raises(rb.RealmError):
        b.update_request(999, 1)


def test_batching_integration():
    b = ContinuousBatcher(32, 2048)
    texts = ["What is the capital of France?", "Tell me about Paris.", "France is a country."]
    for i, t in enumerate(texts):
        b.add_request(BatchedRequest.with_prompt_text(i + 1, [3 * i + 1, 3 * i + 2, 3 * i + 3], t, 50))
    for i in range(3):
        b.update_request(i + 1, 100 * (i + 1))
    batch = b.get_batch()
    assert len(batch) == 3
    assert [r.prompt_text for r in batch] == texts
    assert {r.request_id: r.generated_tokens for r in batch} == {1: [100], 2: [200], 3: [300]}
    assert b.stats().active_requests == 0  # get_batch removed them


def test_get_batch_caps_at_max_batch_and_keeps_order():
    b = ContinuousBatcher(3, 2048)
    for i in range(3):
        b.add_request(BatchedRequest.new(i, [i], 5))
    b.update_request(0, 7)
    for _ in range(4):
        b.update_request(1, 7)
    b.update_request(1, 7)                 # 5 tokens: request 1 complete
    batch = b.get_batch()
    assert [r.request_id for r in batch] == [0, 2]
    assert batch[0].all_tokens() == [0, 7] and batch[0].current_seq_len() == 2
    assert b.get_batch() == []


def test_get_batch_leaves_unreached_requests_queued():
    b = ContinuousBatcher(2, 2048)
    b.add_request(BatchedRequest.new(1, [1], 5))
    b.add_request(BatchedRequest.new(2, [2], 5))
    b2 = ContinuousBatcher(1, 2048)       # batch of one: the second call gets the next request
    b2.add_request(BatchedRequest.new(1, [1], 5))
    assert [r.request_id for r in b2.get_batch()] == [1]
    assert [r.request_id for r in b.get_batch()] == [1, 2]


def test_empty_prompt_and_zero_max_tokens():
    b = ContinuousBatcher(4, 2048)
    b.add_request(BatchedRequest.new(1, [], 3))
    b.add_request(BatchedRequest.new(2, [5], 0))  # generated 0 >= max_tokens 0: dropped
    batch = b.get_batch()
    assert [r.request_id for r in batch] == [1] and batch[0].prompt_tokens == []


def test_concurrent_adds_are_serialised():
    b = ContinuousBatcher(850, 2048)
    def add(base):
        for i in range(100):
            b.add_request(BatchedRequest.new(base + i, [1, 2], 10))
    ts = [threading.Thread(target=add, args=(k * 1000,)) for k in range(8)]
    for t in ts:
        t.start()
    for t in ts:
        t.join()
    assert b.stats().total_requests == 800
    with pytest.raises(rb.RealmError):
        add(99000)                         # the 850-request cap holds across threads


def test_prepare_batch():
    padded, masks = prepare_batch([[1, 2, 3], [4, 5, 6, 7, 8], [9, 10]], 5)
    assert [len(p) for p in padded] == [5, 5, 5]
    assert padded[2] == [9, 10, 0, 0, 0]
    assert masks[0] == [True, True, True, False, False]
    assert masks[1] == [True] * 5
    assert masks[2] == [True, True, False, False, False]


def test_scheduler_rejects_null_handles():
    lib = rb.lib()
    assert lib.rb_scheduler_step(None, None, 0, None) == -20
    assert lib.rb_scheduler_submit(None, 1, None, 0, 1) == -20
    assert lib.rb_scheduler_create(None, 0, None, None) == -20
    assert lib.rb_batcher_get_batch(None, None) == -20
