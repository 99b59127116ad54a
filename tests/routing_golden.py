"""Comparison rules for tests/golden/routing.npz (made by tests/golden/make_routing_golden.py from the
Hugging Face Qwen3-MoE and DeepSeek-V3 routers and its FP8 block dequantisation).

Tolerances, stated once and used by the CPU pins (tests/test_routing_golden.py) and the GPU pins
(tests/test_gpu_parity.py):

  * LOGIT_ATOL: |logit - HF f32 logit| <= 4e-6. Both are f32 dot products of the same bf16 values
    (exact products) summed in different orders; over H <= 2048 terms of size <= ~0.1 the
    difference measured 9.5e-7 at most.
  * Ids: for every token, the set of chosen experts equals HF's, except where the two sides' k-th
    and (k+1)-th scores lie within NEAR_TIE of each other (a near-tie that a 1e-6 logit difference
    can flip) or are exactly equal (torch.topk breaks ties in no stated order; the reference breaks
    them to the lowest index, cached_layer.rs:358-363). At such a token the chosen scores must
    still agree as a multiset.
  * Weights: a chosen expert's weight is within W_ULPS_SAME_LOGITS f32 ulps of HF's when both route
    the same logits (the exp and the sum order differ), and within W_ULPS_OWN_LOGITS when each side
    routes its own logits.
"""
import os

import numpy as np

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "routing.npz")
LOGIT_ATOL = 4e-6
NEAR_TIE = 1e-5
W_ULPS_SAME_LOGITS = 4
W_ULPS_OWN_LOGITS = 32

ROUTER_SOFTMAX, ROUTER_SOFTMAX_RENORM, ROUTER_SIGMOID_GROUP = 0, 1, 2
DSV3 = dict(n_group=8, topk_group=4, routed_scale=2.5)

# (case, logits key, ids key, weights key, k, router mode) of every routing fixture
CASES = [
    ("qwen_c1", "qwen_c1_logits", "qwen_c1_renorm_ids", "qwen_c1_renorm_weights", 2, ROUTER_SOFTMAX_RENORM),
    ("qwen_c1", "qwen_c1_logits", "qwen_c1_plain_ids", "qwen_c1_plain_weights", 2, ROUTER_SOFTMAX),
    ("qwen_c2", "qwen_c2_logits", "qwen_c2_ids", "qwen_c2_weights", 8, ROUTER_SOFTMAX_RENORM),
    ("qwen_ties", "qwen_ties_logits", "qwen_ties_ids", "qwen_ties_weights", 8, ROUTER_SOFTMAX_RENORM),
    ("dsv3_c5", "dsv3_c5_logits", "dsv3_c5_ids", "dsv3_c5_weights", 8, ROUTER_SIGMOID_GROUP),
    ("dsv3_ties", "dsv3_ties_logits", "dsv3_ties_ids", "dsv3_ties_weights", 8, ROUTER_SIGMOID_GROUP),
]


def load():
    return np.load(GOLDEN)


def ulps(a, b) -> np.ndarray:
    """Distance in f32 units in the last place (same-sign finite values)."""
    ia = np.asarray(a, np.float32).view(np.int32).astype(np.int64)
    ib = np.asarray(b, np.float32).view(np.int32).astype(np.int64)
    return np.abs(ia - ib)


def selection_scores(logits: np.ndarray, mode: int, bias=None) -> np.ndarray:
    """The score each router ranks experts by: the logit (softmax is monotone) or, for group-limited
    routing, sigmoid(logit) + bias."""
    if mode == ROUTER_SIGMOID_GROUP:
        s = 1.0 / (1.0 + np.exp(-logits.astype(np.float64)))
        return s + (0.0 if bias is None else bias.astype(np.float64))
    return logits.astype(np.float64)


def check_routing(ids, w, ref_ids, ref_w, scores, k: int, w_ulps: int):
    """Asserts the rules above. scores: [T, E] the selection scores of the side that chose `ids`."""
    ids = np.asarray(ids).astype(np.int64).reshape(-1, k)
    ref_ids = np.asarray(ref_ids).astype(np.int64).reshape(-1, k)
    w = np.asarray(w, np.float32).reshape(-1, k)
    ref_w = np.asarray(ref_w, np.float32).reshape(-1, k)
    exact = ties = 0
    for t in range(ids.shape[0]):
        a, b = dict(zip(ids[t], w[t])), dict(zip(ref_ids[t], ref_w[t]))
        assert len(a) == k and len(b) == k, f"token {t}: repeated expert"
        if set(a) == set(b):
            exact += 1
            for e in a:
                assert ulps(a[e], b[e]) <= w_ulps, f"token {t} expert {e}: {a[e]!r} vs {b[e]!r}"
            continue
        srt = np.sort(scores[t])[::-1]
        gap = srt[k - 1] - srt[k]
        assert gap <= NEAR_TIE * max(1.0, abs(srt[k - 1])), f"token {t}: ids {sorted(a)} vs {sorted(b)}, gap {gap}"
        sa = np.sort(scores[t][ids[t]])
        sb = np.sort(scores[t][ref_ids[t]])
        assert np.allclose(sa, sb, rtol=0, atol=NEAR_TIE), f"token {t}: chosen scores differ beyond a tie"
        if np.array_equal(sa, sb):  # exact ties: equal scores carry equal weights
            assert (ulps(np.sort(w[t]), np.sort(ref_w[t])) <= w_ulps).all(), f"token {t}: tied weights differ"
        ties += 1
    return exact, ties
