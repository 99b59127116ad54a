"""The CPU oracle against the reference's own known-answer tests and the golden format vectors.

Known answers are the assertions of flaneur2020/naiwa-rs src/moe/tests.rs (cited per test);
format vectors come from tests/golden/formats.npz (made by tests/golden/make_golden.py with the
gguf package).
"""
import math
import os

import numpy as np
import pytest

from oracle import oracle as O

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "formats.npz")


# ---- reference known-answer tests (src/moe/tests.rs) ----------------------------------------

def test_top_k_ids_orders_by_logit_then_index():  # tests.rs:169-173
    assert O.top_k_ids([0.1, 0.9, 0.5, 0.9], 3) == [1, 3, 2]
    assert O.top_k_ids([1.0, 2.0], 5) == [1, 0]


def test_top_k_ids_total_order_edges():
    # total_cmp: -0.0 < +0.0, -inf lowest, NaN (positive) above +inf
    assert O.top_k_ids([0.0, -0.0], 2) == [0, 1]
    assert O.top_k_ids([-math.inf, -1.0, math.inf], 3) == [2, 1, 0]
    assert O.top_k_ids([math.nan, math.inf], 1) == [0]


def test_union_by_votes_orders_by_votes_then_rank():  # tests.rs:140-146
    assert O.union_by_votes([[3, 7, 9], [7, 3], [1, 7]]) == [7, 3, 1, 9]
    assert O.union_by_votes([[4, 2]]) == [4, 2]


def test_streamed_misses_ranks_by_total_weight_and_dedups():  # tests.rs:148-161
    misses = [[(1, 0.9), (3, 0.4)], [(3, 0.1), (2, 0.2)]]
    assert O.streamed_misses(misses, 1.0, 3) == [1, 3, 2]
    assert O.streamed_misses(misses, 0.5, 3) == [1, 3]
    assert O.streamed_misses(misses, 1.0, 1) == [1]
    assert O.streamed_misses(misses, 0.0, 3) == []
    assert O.streamed_misses(misses, 1.0, 0) == []


def test_lru_victim_skips_protected_and_prefers_oldest():  # tests.rs:175-186
    slots = [(10, True, 5), (11, True, 1), (12, True, 3)]
    assert O.lru_victim(slots, [11]) == (12, 2)
    assert O.lru_victim(slots, []) == (11, 1)
    assert O.lru_victim(slots, [10, 11, 12]) is None
    # an unpublished slot is never a victim
    assert O.lru_victim([(10, False, 0), (11, True, 9)], []) == (11, 1)


def test_fill_candidate_prefers_hot_unreserved_experts():  # tests.rs:113-131
    assert O.fill_candidate([2, None], [0, 5, 9, 5]) == 1
    assert O.fill_candidate([None, None], [0, 0, 0]) == 0
    assert O.fill_candidate([0, 1], [3, 3, 3]) is None
    assert O.fill_candidate([0, 1, None], [1, 1]) is None


def test_expert_ranges_tile_the_stack_exactly():  # tests.rs:49-63
    E, N, K = 4, 8, 64
    stride = O.block_bytes(O.DT_Q8_0, N * K)
    for e in range(E):
        assert O.expert_range(O.DT_Q8_0, E, N, K, e) == (e * stride, (e + 1) * stride)
    with pytest.raises(IndexError):
        O.expert_range(O.DT_Q8_0, E, N, K, E)
    with pytest.raises(IndexError):
        O.expert_range(O.DT_Q8_0, E, N, 48, 0)


def test_slot_bytes_count_three_projections():  # tests.rs:78-83 (slot.rs:99-111)
    E, N, K = 2, 8, 64
    per = O.block_bytes(O.DT_Q8_0, E * N * K) // E
    assert per == N * K // 32 * 34
    assert 3 * per == 3 * O.block_bytes(O.DT_Q8_0, N * K)


def test_single_expert_slice_matches_stack():  # tests.rs:65-76
    E, N, K = 3, 4, 32
    data = ((np.arange(E * N * K) % 97).astype(np.float32) * np.float32(0.01) - np.float32(0.4))
    q, _ = O.quantize(O.DT_Q8_0, data)
    b, e = O.expert_range(O.DT_Q8_0, E, N, K, 1)
    one = O.dequantize(O.DT_Q8_0, q[b:e], (N, K))
    full = O.dequantize(O.DT_Q8_0, q, (E, N, K))[1]
    assert np.array_equal(one, full)


# ---- block formats against gguf golden vectors ------------------------------------------------

def test_q8_0_quantize_matches_gguf_bytes():
    g = np.load(GOLDEN)
    q, _ = O.quantize(O.DT_Q8_0, g["q8_inputs"])
    assert np.array_equal(q, g["q8_bytes"])


def test_q4_k_dequantize_matches_gguf():
    g = np.load(GOLDEN)
    deq = O.dequantize(O.DT_Q4_K, g["q4k_bytes"], g["q4k_inputs"].shape)
    np.testing.assert_allclose(deq, g["q4k_dequant"], rtol=0, atol=1e-6 * np.abs(g["q4k_dequant"]).max())
    # the oracle's own quantiser reproduces the committed bytes (fixture stability)
    q, _ = O.quantize(O.DT_Q4_K, g["q4k_inputs"])
    assert np.array_equal(q, g["q4k_bytes"])


def test_q4_k_round_trip_error_is_bounded():
    rng = np.random.default_rng(1)
    w = rng.normal(0, 0.02, size=(16, 256)).astype(np.float32)
    q, _ = O.quantize(O.DT_Q4_K, w)
    assert q.size == 16 * 144
    d = O.dequantize(O.DT_Q4_K, q, w.shape)
    # 4-bit: error below one step (range/15) of each 32-weight sub-block
    for j in range(8):
        sub = w[:, 32 * j:32 * j + 32]
        step = (sub.max(1) - np.minimum(sub.min(1), 0)) / 15
        err = np.abs(d[:, 32 * j:32 * j + 32] - sub).max(1)
        assert np.all(err <= 1.5 * step + 1e-6)


def test_q2_0_pack_round_trips_through_the_decoder():  # resident.rs:190-218
    """The reference's own known answers for its Q2_0 packer: a sin-pattern row decodes within half a
    step of its block maximum (err <= 0.55 amax), and a zero block decodes to zeros, not to -d."""
    x = (np.sin(np.arange(4096, dtype=np.float32) * np.float32(0.017)) * np.float32(1.5) - np.float32(0.25)).astype(np.float32)
    q, _ = O.quantize(O.DT_Q2_0, x)
    assert q.size == 4096 // 64 * 18 == O.block_bytes(O.DT_Q2_0, 4096)
    back = O.dequantize(O.DT_Q2_0, q, x.shape)
    assert np.abs(x - back).max() <= np.abs(x).max() * 0.55
    z, _ = O.quantize(O.DT_Q2_0, np.zeros(128, np.float32))
    assert np.all(O.dequantize(O.DT_Q2_0, z, (128,)) == 0.0)
    # layout: f16 d then 16 code bytes, weight j at bits 2*(j%4) of byte j/4, value (code - 1) * d
    blk = q[:18]
    d = np.frombuffer(blk[:2].tobytes(), dtype=np.float16)[0].astype(np.float32)
    codes = np.array([(blk[2 + j // 4] >> (2 * (j % 4))) & 3 for j in range(64)], dtype=np.float32)
    assert np.array_equal(back[:64], (codes - 1.0) * d)


def test_q2_0_scale_ladder_beats_the_block_maximum():
    """The quantiser keeps the ladder candidate with the least squared error, so it is never worse
    than the plain block-maximum scale (ladder fraction 1)."""
    rng = np.random.default_rng(5)
    x = rng.normal(0, 0.02, 64 * 200).astype(np.float32)
    q, _ = O.quantize(O.DT_Q2_0, x)
    back = O.dequantize(O.DT_Q2_0, q, x.shape)
    err = ((x - back).reshape(-1, 64) ** 2).sum(1)
    for b, blk in enumerate(x.reshape(-1, 64)):
        amax = np.abs(blk).max()
        d = np.float32(np.float16(amax))
        codes = np.clip(np.sign(blk / d) * np.floor(np.abs(blk / d) + 0.5) + 1, 0, 3)
        naive = ((blk - (codes - 1) * d) ** 2).sum()
        assert err[b] <= naive * (1 + 1e-6)


def test_fp8_e4m3_codes():
    L = O.lib()
    # every finite code round-trips
    for b in range(256):
        v = L.orc_fp8e4m3_to_f32(b)
        if math.isnan(v):
            assert b & 0x7F == 0x7F
            continue
        back = L.orc_f32_to_fp8e4m3(v)
        assert back == b or (v == 0.0 and (back & 0x7F) == 0)
    assert L.orc_fp8e4m3_to_f32(0x7E) == 448.0
    assert L.orc_fp8e4m3_to_f32(0x01) == 2.0 ** -9
    assert L.orc_f32_to_fp8e4m3(1000.0) == 0x7E  # saturates
    # round to nearest even between 1.0 (0x38) and 1.125 (0x39)
    assert L.orc_f32_to_fp8e4m3(1.0625) == 0x38
    assert L.orc_f32_to_fp8e4m3(1.1875) == 0x3A


def test_fp8_block_quant_round_trip():
    rng = np.random.default_rng(2)
    w = rng.normal(0, 0.02, size=(2, 256, 128)).astype(np.float32)
    q, s = O.quantize(O.DT_FP8, w)
    assert s.shape == (2 * 2 * 1,)
    d = O.dequantize(O.DT_FP8, q, w.shape, s)
    rel = np.abs(d - w).max() / np.abs(w).max()
    assert rel < 1.0 / 16


def test_bf16_rounding_matches_torch():
    torch = pytest.importorskip("torch")
    x = np.random.default_rng(3).normal(0, 3, 10000).astype(np.float32)
    ours = O.f32_to_bf16(x)
    theirs = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(ours, theirs)


# ---- deterministic exp --------------------------------------------------------------------------

def test_exp_accuracy():
    xs = np.linspace(-87, 88, 20001, dtype=np.float32)
    ours = np.array([O.exp(float(v)) for v in xs], dtype=np.float64)
    ref = np.exp(xs.astype(np.float64))
    rel = np.abs(ours - ref) / ref
    assert rel.max() < 4e-7
    assert O.exp(-200.0) == 0.0 and math.isinf(O.exp(100.0))
    assert O.exp(0.0) == 1.0


# ---- router -------------------------------------------------------------------------------------

def _bf16(rng, shape, std):
    return O.f32_to_bf16(rng.normal(0, std, size=shape).astype(np.float32))


def test_router_logits_close_to_double():
    rng = np.random.default_rng(4)
    x = _bf16(rng, (5, 512), 1.0)
    w = _bf16(rng, (16, 512), 0.02)
    got = O.router_logits(x, w)
    ref = O.bf16_to_f32(x).astype(np.float64) @ O.bf16_to_f32(w).astype(np.float64).T
    assert np.abs(got - ref).max() < 1e-5


def test_route_softmax_modes():
    rng = np.random.default_rng(5)
    logits = rng.normal(0, 1, size=(7, 16)).astype(np.float32)
    for mode in (0, 1):
        ids, w = O.route(logits, 2, mode)
        for t in range(7):
            assert list(ids[t]) == O.top_k_ids(logits[t], 2)
            p = np.exp(logits[t].astype(np.float64) - logits[t].max())
            if mode == 0:
                want = p[ids[t]] / p.sum()
            else:
                want = p[ids[t]] / p[ids[t]].sum()
            np.testing.assert_allclose(w[t], want, rtol=1e-6)


def test_route_sigmoid_group_limited():
    rng = np.random.default_rng(6)
    E, G, TG, k = 64, 8, 4, 8
    logits = rng.normal(0, 1, size=(9, E)).astype(np.float32)
    bias = rng.normal(0, 0.1, size=E).astype(np.float32)
    ids, w = O.route(logits, k, 2, bias=bias, n_group=G, topk_group=TG, routed_scale=2.5)
    for t in range(9):
        s = 1.0 / (1.0 + np.exp(-logits[t].astype(np.float64)))
        sel = s + bias
        gs = np.array([np.sort(sel[g * 8:(g + 1) * 8])[-2:].sum() for g in range(G)])
        keep = np.argsort(-gs, kind="stable")[:TG]
        allowed = np.concatenate([np.arange(g * 8, g * 8 + 8) for g in keep])
        order = allowed[np.argsort(-sel[allowed], kind="stable")][:k]
        assert set(ids[t]) == set(order.tolist())
        assert list(ids[t]) == sorted(ids[t], key=lambda e: (-sel[e], e))
        np.testing.assert_allclose(w[t], s[ids[t]] / s[ids[t]].sum() * 2.5, rtol=1e-6)


# ---- permute ------------------------------------------------------------------------------------

def test_permute_is_a_stable_counting_sort():
    rng = np.random.default_rng(7)
    E = 32
    ids = rng.integers(0, E, size=(100, 4)).astype(np.uint32)
    counts, offsets, perm, active = O.permute(ids, E)
    flat = ids.reshape(-1)
    assert np.array_equal(counts, np.bincount(flat, minlength=E))
    assert np.array_equal(perm, np.argsort(flat, kind="stable"))
    assert offsets[0] == 0 and offsets[-1] == flat.size
    assert np.array_equal(active, np.nonzero(counts)[0])


def test_permute_rejects_bad_ids_and_handles_empty():
    with pytest.raises(ValueError):
        O.permute(np.array([[0, 9]], dtype=np.uint32), 8)
    counts, offsets, perm, active = O.permute(np.zeros((0, 2), dtype=np.uint32), 8)
    assert counts.sum() == 0 and perm.size == 0 and active.size == 0


# ---- expert FFN: the reference's own split-vs-full fixtures --------------------------------------

def sin_stack(E, N, K, seed):
    """src/moe/tests.rs:190-200 / prefill_stream.rs:1801-1807: sin(i*0.37 + seed)*0.5 as Q8_0."""
    i = np.arange(E * N * K, dtype=np.float32)
    data = (np.sin(i * np.float32(0.37) + np.float32(seed)) * np.float32(0.5)).astype(np.float32)
    q, _ = O.quantize(O.DT_Q8_0, data)
    return q, O.dequantize(O.DT_Q8_0, q, (E, N, K))


def test_fused_cpu_decode_matches_dequantised_reference():
    # prefill_stream.rs:1911-2000: E=4, hidden 64, inter 32, 3 tokens, TOL 2e-2
    E, H, I = 4, 64, 32
    gq, gd = sin_stack(E, I, H, 0.1)
    uq, ud = sin_stack(E, I, H, 0.7)
    dq, dd = sin_stack(E, H, I, 1.3)
    x = np.cos(np.arange(3 * H, dtype=np.float32) * np.float32(0.11)).reshape(3, H)
    ids = np.array([[0, 2], [3, 1], [2, 0]], dtype=np.uint32)
    ws = np.array([[0.6, 0.4], [0.3, 0.7], [0.5, 0.5]], dtype=np.float32)
    want = O.moe_forward_f32(x, ids, ws, gd, ud, dd)
    got = O.fused_moe_decode_q8_0(gq, uq, dq, x, ids, ws, E, H, I, threads=2)
    assert np.abs(got - want).max() < 2e-2
    assert np.abs(got - want).max() / np.abs(want).max() < 1e-4
    # subset of the top-k, and weight-0 padding (cpu_miss.rs:90-100) contributes nothing
    sub = O.moe_forward_f32(x, ids[:, :1].copy(), ws[:, :1].copy(), gd, ud, dd)
    pad_ids = np.stack([ids[:, 0], ids[:, 0]], 1).astype(np.uint32)
    pad_w = np.stack([ws[:, 0], np.zeros(3, np.float32)], 1).astype(np.float32)
    got = O.fused_moe_decode_q8_0(gq, uq, dq, x, pad_ids, pad_w, E, H, I, threads=3)
    assert np.abs(got - sub).max() < 2e-2
    # a swapped weight moves the output far beyond the tolerance (the test has teeth)
    bad = O.moe_forward_f32(x, ids, ws[:, ::-1].copy(), gd, ud, dd)
    assert np.abs(bad - want).max() > 0.1


# ---- the timed CPU baseline (oracle/cpu_baseline.c) against the strict-order oracle ---------------

@pytest.mark.parametrize("T", [1, 5, 33])
def test_cpu_baseline_matches_strict_oracle(T):
    """bench.py's reference arm times orc_baseline_decode_q8_0; it must compute the strict oracle's
    fused decode (up to f32 summation order), including weight-0 slots and a repeated expert."""
    rng = np.random.default_rng(40 + T)
    E, k, H, I = 16, 4, 256, 128
    q = [O.quantize(O.DT_Q8_0, rng.normal(0, 0.02, s).astype(np.float32))[0] for s in ((E, I, H), (E, I, H), (E, H, I))]
    x = rng.normal(0, 1, (T, H)).astype(np.float32)
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.uint32)
    w = rng.dirichlet(np.ones(k), T).astype(np.float32)
    w[0, -1] = 0.0           # weight-0 padding is skipped
    ids[-1, 1] = ids[-1, 0]  # a repeated expert: one pair, the weights summed
    want = O.fused_moe_decode_q8_0(q[0], q[1], q[2], x, ids, w, E, H, I, 2)
    got = O.baseline_decode_q8_0(q[0], q[1], q[2], x, ids, w, E, H, I, 3)
    assert np.abs(got - want).max() <= 1e-5 * np.abs(want).max()
