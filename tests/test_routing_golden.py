"""The oracle's router and FP8 block dequantisation against published implementations.

The reference's router lives in its un-vendored mistral.rs fork, so the oracle's routing is pinned
to the Hugging Face implementations of the two router families the configs name, through the
fixtures of tests/golden/routing.npz (tests/golden/make_routing_golden.py):
  * Qwen3-MoE (configs 1 and 2): softmax, top-k, optional renormalisation over the k;
  * DeepSeek-V3 (config 5): sigmoid, bias for the choice, top-2-sum group scores, group-limited
    top-k, weights renormalised and scaled;
  * FP8 e4m3fn decode and 128x128 block dequantisation (DeepSeek-V3 checkpoints).
Tolerances are stated in tests/routing_golden.py. The GPU router is bit-exact against the oracle
(tests/test_gpu_parity.py) and is also checked against these fixtures there.
"""
import numpy as np
import pytest

import routing_golden as RG
from oracle import oracle as O


@pytest.fixture(scope="module")
def g():
    return RG.load()


@pytest.mark.parametrize("case", ["qwen_c1", "qwen_c2", "dsv3_c5"])
def test_router_logits_match_hf_f32(g, case):
    got = O.router_logits(g[case + "_x"], g[case + "_w"])
    ref = g[case + "_logits"]
    assert got.shape == ref.shape
    assert np.abs(got - ref).max() <= RG.LOGIT_ATOL


@pytest.mark.parametrize("case,lk,ik,wk,k,mode", RG.CASES, ids=[f"{c[0]}-{c[2]}" for c in RG.CASES])
def test_route_matches_hf_on_the_same_logits(g, case, lk, ik, wk, k, mode):
    """Given HF's own logits, the oracle chooses HF's experts with HF's weights (within 4 ulps)."""
    logits = g[lk]
    bias = g["dsv3_bias"] if mode == RG.ROUTER_SIGMOID_GROUP else None
    kw = dict(RG.DSV3, bias=bias) if mode == RG.ROUTER_SIGMOID_GROUP else {}
    ids, w = O.route(logits, k, mode, **kw)
    exact, ties = RG.check_routing(ids, w, g[ik], g[wk], RG.selection_scores(logits, mode, bias), k,
                                   RG.W_ULPS_SAME_LOGITS)
    if "ties" not in case:
        assert ties == 0  # random logits: no near-tie at the k-th place in these fixtures
    else:
        assert exact + ties == logits.shape[0]


@pytest.mark.parametrize("case,ik,wk,k,mode", [
    ("qwen_c1", "qwen_c1_renorm_ids", "qwen_c1_renorm_weights", 2, RG.ROUTER_SOFTMAX_RENORM),
    ("qwen_c1", "qwen_c1_plain_ids", "qwen_c1_plain_weights", 2, RG.ROUTER_SOFTMAX),
    ("qwen_c2", "qwen_c2_ids", "qwen_c2_weights", 8, RG.ROUTER_SOFTMAX_RENORM),
    ("dsv3_c5", "dsv3_c5_ids", "dsv3_c5_weights", 8, RG.ROUTER_SIGMOID_GROUP),
])
def test_route_end_to_end_matches_hf(g, case, ik, wk, k, mode):
    """x and the gate in, ids and weights out: the oracle's own logits against HF's whole router."""
    logits = O.router_logits(g[case + "_x"], g[case + "_w"])
    bias = g["dsv3_bias"] if mode == RG.ROUTER_SIGMOID_GROUP else None
    kw = dict(RG.DSV3, bias=bias) if mode == RG.ROUTER_SIGMOID_GROUP else {}
    ids, w = O.route(logits, k, mode, **kw)
    RG.check_routing(ids, w, g[ik], g[wk], RG.selection_scores(logits, mode, bias), k, RG.W_ULPS_OWN_LOGITS)


def test_fp8_e4m3_codes_match_torch(g):
    """Every one of the 256 e4m3fn codes decodes to torch's value (NaN at S.1111.111)."""
    codes = np.tile(np.arange(256, dtype=np.uint8), 64)
    got = O.dequantize(O.DT_FP8, codes, (128, 128), np.ones((1, 1), np.float32)).reshape(-1)[:256]
    ref = g["fp8_code_values"]
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(got), nan) and nan.sum() == 2
    assert np.array_equal(got[~nan].view(np.uint32), ref[~nan].view(np.uint32))


def test_fp8_block_dequant_matches_hf(g):
    """128x128 block scales: bit-exact with transformers' Fp8Dequantize on every finite code."""
    got = O.dequantize(O.DT_FP8, g["fp8_q"].reshape(-1), (256, 256), g["fp8_scales"])
    assert np.array_equal(got.view(np.uint32), g["fp8_dequant"].view(np.uint32))
