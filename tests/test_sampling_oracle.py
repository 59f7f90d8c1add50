"""CPU: the oracle's restatement of LogitsProcessor (oracle/oracle.cpp or_sample)
against the reference's own sampling tests (crates/realm-models/src/sampling.rs:304-362)
and hand-worked cases of each strategy, plus the counter-based uniform stream."""
import numpy as np

import realm_b200 as rb


def test_argmax_sampling(oracle):
    tok, _ = oracle.sample([1.0, 3.0, 2.0, 5.0, 1.5], 0.0, 1.0, 0, 1.0, [], 0.5)
    assert tok == 3


def test_temperature_sampling(oracle):
    for u in (0.0, 0.3, 0.9999):
        tok, _ = oracle.sample([1.0, 2.0, 3.0], 1.0, 1.0, 0, 1.0, [], u)
        assert tok < 3


def test_repetition_penalty(oracle):
    tok1, _ = oracle.sample([5.0, 3.0, 2.0], 0.0, 1.0, 0, 1.5, [], 0.0)
    assert tok1 == 0
    _, lg = oracle.sample([5.0, 3.0, 2.0], 0.0, 1.0, 0, 1.5, [0], 0.0)
    assert lg[0] < 5.0 and np.isclose(lg[0], 5.0 / 1.5)
    _, lg = oracle.sample([-2.0, 3.0, 2.0], 0.0, 1.0, 0, 1.5, [0, 0], 0.0)   # negative: multiplied, per occurrence
    assert lg[0] == np.float32(-2.0) * np.float32(1.5) * np.float32(1.5)


def test_topk_sampling(oracle):
    for u in np.linspace(0, 0.999, 25):
        tok, _ = oracle.sample([1.0, 5.0, 3.0, 2.0, 4.0], 1.0, 1.0, 2, 1.0, [], u)
        assert tok in (1, 4)


def test_topp_sampling(oracle):
    for u in np.linspace(0, 0.999, 25):
        tok, _ = oracle.sample([1.0, 10.0, 2.0, 1.0, 1.0], 1.0, 0.9, 0, 1.0, [], u)
        assert tok == 1   # token 1 alone holds > 0.9 of the mass


def test_multinomial_boundaries(oracle):
    """WeightedIndex: the index is the number of cumulative weights <= u * total."""
    lg = np.log(np.array([0.25, 0.25, 0.5], np.float32))
    assert oracle.sample(lg, 1.0, 1.0, 0, 1.0, [], 0.0)[0] == 0
    assert oracle.sample(lg, 1.0, 1.0, 0, 1.0, [], 0.2499)[0] == 0
    assert oracle.sample(lg, 1.0, 1.0, 0, 1.0, [], 0.2501)[0] == 1
    assert oracle.sample(lg, 1.0, 1.0, 0, 1.0, [], 0.7501)[0] == 2


def test_topk_then_topp(oracle):
    lg = np.log(np.array([0.05, 0.4, 0.3, 0.2, 0.05], np.float32))
    seen = {oracle.sample(lg, 1.0, 0.6, 3, 1.0, [], u)[0] for u in np.linspace(0, 0.999, 50)}
    assert seen == {1, 2}   # top-3 = {1, 2, 3}, renormalised 0.44, 0.33, 0.22: top-p 0.6 keeps 1 and 2


def test_all_masked_is_an_error(oracle):
    tok, _ = oracle.sample([-np.inf] * 4, 1.0, 1.0, 0, 1.0, [], 0.5)
    assert tok is None


def test_uniform_stream_is_deterministic_on_the_2e23_grid():
    u = [rb.sampling_uniform(42, i) for i in range(2000)]
    assert u == [rb.sampling_uniform(42, i) for i in range(2000)]
    assert all(0.0 <= x < 1.0 and (x * 2**23).is_integer() for x in u)
    assert abs(np.mean(u) - 0.5) < 0.03 and len(set(u)) > 1990
    assert rb.sampling_uniform(43, 0) != rb.sampling_uniform(42, 0)
