"""The library's expert-cache decision functions (moe_policy_*, host code) against the reference's
known-answer cases (src/moe/tests.rs) and against the oracle's restatement on random inputs.
CPU only: the functions make no CUDA call."""
import math

import numpy as np
import pytest

from oracle import oracle as O


@pytest.fixture(scope="module")
def P():
    from moe_b200 import policy
    return policy


def test_known_answers(P):
    assert P.top_k_ids([0.1, 0.9, 0.5, 0.9], 3) == [1, 3, 2]  # tests.rs:169-173
    assert P.top_k_ids([1.0, 2.0], 5) == [1, 0]
    assert P.top_k_ids([0.0, -0.0], 2) == [0, 1]
    assert P.top_k_ids([-math.inf, -1.0, math.inf], 3) == [2, 1, 0]
    assert P.top_k_ids([math.nan, math.inf], 1) == [0]
    assert P.union_by_votes([[3, 7, 9], [7, 3], [1, 7]]) == [7, 3, 1, 9]  # tests.rs:140-146
    misses = [[(1, 0.9), (3, 0.4)], [(3, 0.1), (2, 0.2)]]  # tests.rs:148-161
    assert P.streamed_misses(misses, 1.0, 3) == [1, 3, 2]
    assert P.streamed_misses(misses, 0.5, 3) == [1, 3]
    assert P.streamed_misses(misses, 1.0, 1) == [1]
    assert P.streamed_misses(misses, 0.0, 3) == []
    assert P.streamed_misses(misses, 1.0, 0) == []
    slots = [(10, True, 5), (11, True, 1), (12, True, 3)]  # tests.rs:175-186
    assert P.lru_victim(slots, [11]) == (12, 2)
    assert P.lru_victim(slots, []) == (11, 1)
    assert P.lru_victim(slots, [10, 11, 12]) is None
    assert P.lru_victim([(10, False, 0), (11, True, 9)], []) == (11, 1)
    assert P.fill_candidate([2, None], [0, 5, 9, 5]) == 1  # tests.rs:113-131
    assert P.fill_candidate([None, None], [0, 0, 0]) == 0
    assert P.fill_candidate([0, 1], [3, 3, 3]) is None
    assert P.fill_candidate([0, 1, None], [1, 1]) is None


def test_random_cases_match_oracle(P):
    rng = np.random.default_rng(0)
    for _ in range(300):
        n = int(rng.integers(1, 40))
        logits = rng.choice([-1.0, 0.0, -0.0, 0.5, 2.0, np.inf], size=n).astype(np.float32) if rng.random() < 0.3 \
            else rng.normal(size=n).astype(np.float32)
        k = int(rng.integers(0, n + 3))
        assert P.top_k_ids(logits, k) == O.top_k_ids(logits, k)
        rk = [list(rng.choice(12, size=int(rng.integers(1, 6)), replace=False)) for _ in range(int(rng.integers(1, 5)))]
        assert P.union_by_votes(rk) == O.union_by_votes(rk)
        misses = [[(int(rng.integers(0, 10)), float(np.float32(rng.choice([0.25, 0.5, rng.random()]))))
                   for _ in range(int(rng.integers(0, 5)))] for _ in range(int(rng.integers(1, 6)))]
        frac, cap = float(rng.choice([0.0, 0.3, 0.5, 1.0])), int(rng.integers(0, 6))
        assert P.streamed_misses(misses, frac, cap) == O.streamed_misses(misses, frac, cap)
        ns = int(rng.integers(1, 8))
        slots = [(None if rng.random() < 0.2 else int(rng.integers(0, 10)), bool(rng.random() < 0.9),
                  int(rng.integers(0, 5))) for _ in range(ns)]
        prot = list(rng.choice(10, size=int(rng.integers(0, 4)), replace=False))
        assert P.lru_victim(slots, prot) == O.lru_victim(slots, prot)
        hc = rng.integers(0, 4, size=int(rng.integers(1, 12))).astype(np.uint64)
        se = [None if rng.random() < 0.4 else int(rng.integers(0, hc.size)) for _ in range(ns)]
        assert P.fill_candidate(se, hc) == O.fill_candidate(se, list(hc))
