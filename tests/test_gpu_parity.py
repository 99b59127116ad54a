"""Parity of the sm_100a path (through the C ABI) against the CPU oracle.

Integer/index work (router ids, histogram, permutation) must be bit-exact; router weights are
bit-exact too (shared deterministic exp, IEEE division). Expert outputs must stay within the
max |y - ref| / max |ref| <= 1e-2, ref = the dequantised f32/double
reference (or, at full config size, the oracle's multithreaded Q8_0 fused decode, itself pinned to
the dequantised reference in tests/test_oracle.py). Every token is also held to the elementwise
bound of tests/tolerance.py.
"""
import numpy as np
import pytest

import routing_golden as RG
from oracle import oracle as O
from tolerance import assert_close

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

REL_TOL = 1e-2  # north star: max relative error <= 1e-2 against the dequantised reference


def M():
    import moe_b200

    return moe_b200


def rel_err(got, ref):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


def bf16_tensor(a_u16, dev="cuda"):
    return torch.from_numpy(np.ascontiguousarray(a_u16).view(np.int16)).view(torch.bfloat16).to(dev)


def make_stacks(rng, E, H, I, dtype, std=0.02):
    gate = rng.normal(0, std, (E, I, H)).astype(np.float32)
    up = rng.normal(0, std, (E, I, H)).astype(np.float32)
    down = rng.normal(0, std, (E, H, I)).astype(np.float32)
    q = [O.quantize(dtype, w)[0] for w in (gate, up, down)]
    d = [O.dequantize(dtype, qq, shape) for qq, shape in zip(q, [gate.shape, up.shape, down.shape])]
    return q, d


def build_layer(q, E, k, H, I, dtype, router=None, bias=None, mode=1, n_group=1, topk_group=1, scale=1.0,
                max_tokens=256):
    m = M()
    cfg = m.MoeConfig(num_experts=E, num_experts_per_tok=k, hidden_size=H, moe_intermediate_size=I,
                      router_mode=mode, n_group=n_group, topk_group=topk_group, routed_scaling_factor=scale)
    ctx = m.ExpertLoadContext(layer=0, device=0, config=cfg, wdtype=dtype, gate=q[0], up=q[1], down=q[2],
                              router_weight=router, router_bias=bias, max_tokens=max_tokens)
    return m.RoutedExpertsProvider().build(ctx)


# ---- router ------------------------------------------------------------------------------------

@pytest.mark.parametrize("T,H,E,k,mode", [(1, 2048, 128, 8, 1), (37, 2048, 128, 8, 1), (64, 1024, 16, 2, 0),
                                          (300, 1024, 16, 2, 1), (5, 512, 64, 6, 0),
                                          # two experts per warp on f32-staged tokens (4 or 8 per CTA)
                                          (256, 2048, 128, 8, 1), (129, 2048, 128, 8, 1), (300, 1024, 64, 6, 0),
                                          (301, 512, 72, 4, 1)])
def test_router_softmax_bit_exact(T, H, E, k, mode):
    rng = np.random.default_rng(T * 7 + E)
    x = O.f32_to_bf16(rng.normal(0, 1, (T, H)).astype(np.float32))
    w = O.f32_to_bf16(rng.normal(0, 0.02, (E, H)).astype(np.float32))
    ids, wt = M().route_tokens(bf16_tensor(x), bf16_tensor(w), k, mode)
    logits = O.router_logits(x, w)
    rid, rw = O.route(logits, k, mode)
    assert np.array_equal(ids.cpu().numpy().astype(np.uint32), rid)
    assert np.array_equal(wt.cpu().numpy().view(np.uint32), rw.view(np.uint32))


def test_router_workspace_reused_across_batch_sizes():
    """One layer (and one Router workspace) routes batches that grow and shrink: every call's ids and
    weights are the oracle's. The arrival counters must sit where no call's logits land, or a shorter
    call after a longer one finds no last CTA and leaves the ids unwritten."""
    rng = np.random.default_rng(77)
    E, k, H = 16, 4, 256
    w = O.f32_to_bf16(rng.normal(0, 0.05, (E, H)).astype(np.float32))
    q, _ = make_stacks(rng, E, H, 128, O.DT_Q8_0)
    layer = build_layer(q, E, k, H, 128, O.DT_Q8_0, router=w.reshape(E, H), mode=1, max_tokens=64)
    router = M().Router(bf16_tensor(w.reshape(E, H)), k, 1, max_tokens=64)
    for T in (16, 7, 64, 1, 33, 2, 64, 5):
        x = O.f32_to_bf16(rng.normal(0, 1, (T, H)).astype(np.float32))
        rid, rw = O.route(O.router_logits(x, w.reshape(E, H)), k, 1)
        for got_ids, got_w in (layer.route(bf16_tensor(x)), router.route(bf16_tensor(x))):
            assert np.array_equal(got_ids.cpu().numpy().astype(np.uint32), rid), T
            assert np.array_equal(got_w.cpu().numpy().view(np.uint32), rw.view(np.uint32)), T


def test_router_ties_go_to_lowest_id():
    # identical router rows give identical logits: the top-k must be the lowest ids (tests.rs:169-173)
    H, E, k = 256, 32, 4
    x = O.f32_to_bf16(np.ones((3, H), np.float32))
    w = O.f32_to_bf16(np.full((E, H), 0.01, np.float32))
    ids, _ = M().route_tokens(bf16_tensor(x), bf16_tensor(w), k, 1)
    assert ids.cpu().numpy().tolist() == [[0, 1, 2, 3]] * 3


@pytest.mark.parametrize("T,E,G,TG,k", [(3, 256, 8, 4, 8), (70, 64, 8, 4, 8), (16, 32, 4, 2, 3)])
def test_router_sigmoid_group_bit_exact(T, E, G, TG, k):
    rng = np.random.default_rng(E + T)
    H = 1024
    x = O.f32_to_bf16(rng.normal(0, 1, (T, H)).astype(np.float32))
    w = O.f32_to_bf16(rng.normal(0, 0.02, (E, H)).astype(np.float32))
    bias = rng.normal(0, 0.05, E).astype(np.float32)
    ids, wt = M().route_tokens(bf16_tensor(x), bf16_tensor(w), k, 2, bias=torch.from_numpy(bias).cuda(),
                               n_group=G, topk_group=TG, routed_scale=2.5)
    rid, rw = O.route(O.router_logits(x, w), k, 2, bias=bias, n_group=G, topk_group=TG, routed_scale=2.5)
    assert np.array_equal(ids.cpu().numpy().astype(np.uint32), rid)
    assert np.array_equal(wt.cpu().numpy().view(np.uint32), rw.view(np.uint32))


# ---- router against the published routers (tests/golden/routing.npz) -----------------------------

@pytest.mark.parametrize("case,ik,wk,k,mode", [
    ("qwen_c1", "qwen_c1_renorm_ids", "qwen_c1_renorm_weights", 2, RG.ROUTER_SOFTMAX_RENORM),
    ("qwen_c1", "qwen_c1_plain_ids", "qwen_c1_plain_weights", 2, RG.ROUTER_SOFTMAX),
    ("qwen_c2", "qwen_c2_ids", "qwen_c2_weights", 8, RG.ROUTER_SOFTMAX_RENORM),
    ("dsv3_c5", "dsv3_c5_ids", "dsv3_c5_weights", 8, RG.ROUTER_SIGMOID_GROUP),
])
def test_router_matches_published_router(case, ik, wk, k, mode):
    """x and the gate of the fixture through the library's router: HF's experts and weights (within
    the stated ulps), and bit-exact with the oracle on the same inputs."""
    g = RG.load()
    x, w = g[case + "_x"], g[case + "_w"]
    bias = g["dsv3_bias"] if mode == RG.ROUTER_SIGMOID_GROUP else None
    kw = dict(bias=torch.from_numpy(bias).cuda(), n_group=8, topk_group=4, routed_scale=2.5) if bias is not None else {}
    ids, wt = M().route_tokens(bf16_tensor(x), bf16_tensor(w), k, mode, **kw)
    ids, wt = ids.cpu().numpy().astype(np.uint32), wt.cpu().numpy()
    logits = O.router_logits(x, w)
    okw = dict(RG.DSV3, bias=bias) if bias is not None else {}
    rid, rw = O.route(logits, k, mode, **okw)
    assert np.array_equal(ids, rid) and np.array_equal(wt.view(np.uint32), rw.view(np.uint32))
    RG.check_routing(ids, wt, g[ik], g[wk], RG.selection_scores(logits, mode, bias), k, RG.W_ULPS_OWN_LOGITS)


@pytest.mark.parametrize("case,k,mode", [("qwen_ties", 8, RG.ROUTER_SOFTMAX_RENORM),
                                         ("dsv3_ties", 8, RG.ROUTER_SIGMOID_GROUP)])
def test_router_tie_heavy_logits_match_published_router(case, k, mode):
    """Logits on a 1/8 grid (many exact ties) fed through an identity gate (bf16 holds them exactly,
    x . e_i is exact): HF's choice up to the order among equal scores, which the library breaks to the
    lowest id (cached_layer.rs:358-363), exactly as the oracle does."""
    g = RG.load()
    logits = g[case + "_logits"]
    E = logits.shape[1]
    x = O.f32_to_bf16(logits)
    assert np.array_equal(O.bf16_to_f32(x).reshape(logits.shape), logits)
    eye = O.f32_to_bf16(np.eye(E, dtype=np.float32))
    bias = g["dsv3_bias"] if mode == RG.ROUTER_SIGMOID_GROUP else None
    kw = dict(bias=torch.from_numpy(bias).cuda(), n_group=8, topk_group=4, routed_scale=2.5) if bias is not None else {}
    ids, wt = M().route_tokens(bf16_tensor(x), bf16_tensor(eye), k, mode, **kw)
    ids, wt = ids.cpu().numpy().astype(np.uint32), wt.cpu().numpy()
    okw = dict(RG.DSV3, bias=bias) if bias is not None else {}
    rid, rw = O.route(logits, k, mode, **okw)
    assert np.array_equal(ids, rid) and np.array_equal(wt.view(np.uint32), rw.view(np.uint32))
    RG.check_routing(ids, wt, g[case + "_ids"], g[case + "_weights"], RG.selection_scores(logits, mode, bias), k,
                     RG.W_ULPS_SAME_LOGITS)


# ---- plan (histogram + stable permute) -----------------------------------------------------------

@pytest.mark.parametrize("n_pairs,E,skew", [(8, 128, 0), (2048, 128, 0), (4096, 128, 1), (9000, 256, 1),
                                            (65536, 256, 0), (65536, 128, 1), (1, 16, 0)])
def test_plan_bit_exact(n_pairs, E, skew):
    rng = np.random.default_rng(n_pairs + E)
    if skew:
        p = 1.0 / np.arange(1, E + 1) ** 1.1
        ids = rng.choice(E, size=n_pairs, p=p / p.sum()).astype(np.uint32)
    else:
        ids = rng.integers(0, E, n_pairs).astype(np.uint32)
    counts, offsets, perm, active, n_active, err = M().plan_pairs(torch.from_numpy(ids.view(np.int32)).cuda(), E)
    rc, ro, rp, ra = O.permute(ids, E)
    assert np.array_equal(counts.cpu().numpy(), rc)
    assert np.array_equal(offsets.cpu().numpy(), ro)
    assert np.array_equal(perm.cpu().numpy(), rp)
    assert int(n_active.item()) == ra.size
    assert np.array_equal(active.cpu().numpy()[: ra.size], ra)
    assert int(err.item()) == 0


def test_plan_flags_bad_ids_without_writing_them():
    ids = np.array([3, 99, 1, 3], dtype=np.uint32)
    counts, offsets, perm, active, n_active, err = M().plan_pairs(torch.from_numpy(ids.view(np.int32)).cuda(), 8)
    assert int(err.item()) == 5  # MOE_ERR_BAD_IDS
    assert counts.cpu().numpy().tolist() == [0, 1, 0, 2, 0, 0, 0, 0]
    assert perm.cpu().numpy()[:3].tolist() == [2, 0, 3]


# ---- expert FFN: the reference's own fixtures ----------------------------------------------------

def sin_stack(E, N, K, seed):
    i = np.arange(E * N * K, dtype=np.float32)
    data = (np.sin(i * np.float32(0.37) + np.float32(seed)) * np.float32(0.5)).astype(np.float32)
    q, _ = O.quantize(O.DT_Q8_0, data)
    return q, O.dequantize(O.DT_Q8_0, q, (E, N, K))


def _fixture_layer(E, k):
    H, I = 64, 32
    gq, gd = sin_stack(E, I, H, 0.1)
    uq, ud = sin_stack(E, I, H, 0.7)
    dq, dd = sin_stack(E, H, I, 1.3)
    return build_layer([gq, uq, dq], E, k, H, I, O.DT_Q8_0, max_tokens=8), (gd, ud, dd)


def _run(layer, x, ids, ws):
    xt = bf16_tensor(O.f32_to_bf16(x))
    y = layer.forward(xt, torch.from_numpy(ws).cuda(), torch.from_numpy(ids.view(np.int32)).cuda())
    torch.cuda.synchronize()
    layer.check()
    return y.float().cpu().numpy()


def test_decode_split_matches_every_expert_on_cpu():  # tests.rs:253-280 (TOL 2e-2)
    layer, (gd, ud, dd) = _fixture_layer(8, 2)
    x = np.cos(np.arange(64, dtype=np.float32) * np.float32(0.11)).reshape(1, 64)
    xb = O.bf16_to_f32(O.f32_to_bf16(x))
    ids = np.array([[0, 3]], np.uint32)
    ws = np.array([[0.6, 0.4]], np.float32)
    got = _run(layer, x, ids, ws)
    want = O.moe_forward_f32(xb, ids, ws, gd, ud, dd)
    assert np.abs(got - want).max() < 2e-2
    assert rel_err(got, want) < REL_TOL


def test_verify_rows_split_matches_every_expert_on_cpu():  # tests.rs:282-308
    layer, (gd, ud, dd) = _fixture_layer(8, 2)
    x = np.cos(np.arange(3 * 64, dtype=np.float32) * np.float32(0.11)).reshape(3, 64)
    xb = O.bf16_to_f32(O.f32_to_bf16(x))
    ids = np.array([[0, 3], [2, 0], [3, 5]], np.uint32)
    ws = np.array([[0.6, 0.4], [0.7, 0.3], [0.5, 0.5]], np.float32)
    got = _run(layer, x, ids, ws)
    want = O.moe_forward_f32(xb, ids, ws, gd, ud, dd)
    assert np.abs(got - want).max() < 2e-2
    assert rel_err(got, want) < REL_TOL


def test_from_qtensors_matches_dequantised_reference():  # prefill_stream.rs:1911-2000
    layer, (gd, ud, dd) = _fixture_layer(4, 2)
    x = np.cos(np.arange(3 * 64, dtype=np.float32) * np.float32(0.11)).reshape(3, 64)
    xb = O.bf16_to_f32(O.f32_to_bf16(x))
    ids = np.array([[0, 2], [3, 1], [2, 0]], np.uint32)
    ws = np.array([[0.6, 0.4], [0.3, 0.7], [0.5, 0.5]], np.float32)
    want = O.moe_forward_f32(xb, ids, ws, gd, ud, dd)
    assert np.abs(_run(layer, x, ids, ws) - want).max() < 2e-2
    # a subset of the routed experts (one per token): the miss path's shape
    sub_i, sub_w = ids[:, :1].copy(), ws[:, :1].copy()
    want = O.moe_forward_f32(xb, sub_i, sub_w, gd, ud, dd)
    assert np.abs(_run(layer, x, sub_i, sub_w) - want).max() < 2e-2
    # a swapped routing weight moves the output past the tolerance
    bad = O.moe_forward_f32(xb, ids, ws[:, ::-1].copy(), gd, ud, dd)
    assert np.abs(_run(layer, x, ids, ws) - bad).max() > 0.1


# ---- expert FFN: random layers against the dequantised reference ---------------------------------

@pytest.mark.parametrize("dtype", [O.DT_Q8_0, O.DT_BF16])
@pytest.mark.parametrize("T", [1, 5, 33, 100, 140])
def test_forward_matches_dequantised_reference(dtype, T):
    """A Q8_0 layer this small (too few GEMM work items to fill the GPU) keeps the decode GEMV below 16
    tokens per expert: T = 1, 5 and 33 run the GEMV, T = 100 and 140 the tcgen05 GEMM."""
    rng = np.random.default_rng(100 + T + dtype)
    E, k, H, I = 16, 4, 256, 128
    q, d = make_stacks(rng, E, H, I, dtype)
    layer = build_layer(q, E, k, H, I, dtype, max_tokens=max(128, T))
    x = rng.normal(0, 1, (T, H)).astype(np.float32)
    xb = O.bf16_to_f32(O.f32_to_bf16(x))
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.uint32)
    ws = rng.dirichlet(np.ones(k), T).astype(np.float32)
    got = _run(layer, x, ids, ws)
    want = O.moe_forward_f32(xb, ids, ws, *d)
    assert_close(got, want)


def test_weight_zero_padding_is_inert():
    # gpu.rs:100-131: short rows are padded with weight-0 entries on an expert some row hits
    rng = np.random.default_rng(7)
    E, k, H, I = 8, 2, 128, 64
    q, d = make_stacks(rng, E, H, I, O.DT_Q8_0)
    layer = build_layer(q, E, k, H, I, O.DT_Q8_0, max_tokens=16)
    x = rng.normal(0, 1, (3, H)).astype(np.float32)
    ids = np.array([[1, 4], [2, 5], [6, 1]], np.uint32)
    ws = np.array([[0.5, 0.5], [0.9, 0.1], [0.3, 0.7]], np.float32)
    base = _run(layer, x, ids, ws)
    pad_i = np.concatenate([ids, np.full((3, 2), 1, np.uint32)], 1)
    pad_w = np.concatenate([ws, np.zeros((3, 2), np.float32)], 1)
    got = _run(layer, x, pad_i, pad_w)
    assert np.array_equal(got, base)


def test_empty_call_and_bad_ids():
    rng = np.random.default_rng(8)
    E, k, H, I = 8, 2, 128, 64
    q, _ = make_stacks(rng, E, H, I, O.DT_Q8_0)
    layer = build_layer(q, E, k, H, I, O.DT_Q8_0, max_tokens=16)
    x = torch.zeros((0, H), dtype=torch.bfloat16, device="cuda")
    y = layer.forward(x, torch.zeros((0, k), device="cuda"), torch.zeros((0, k), dtype=torch.int32, device="cuda"))
    assert y.shape == (0, H)
    xb = torch.randn((2, H), device="cuda").to(torch.bfloat16)
    ids = torch.tensor([[1, 9], [0, 2]], dtype=torch.int32, device="cuda")
    layer.forward(xb, torch.ones((2, k), device="cuda"), ids)
    with pytest.raises(M().MoeError) as ei:
        layer.check()
    assert ei.value.status == 5
    layer.check()  # the error word is cleared once read
    with pytest.raises(M().MoeError):  # more pairs than the scratch was sized for
        layer.forward(torch.zeros((17, H), dtype=torch.bfloat16, device="cuda"),
                      torch.ones((17, k), device="cuda"), torch.zeros((17, k), dtype=torch.int32, device="cuda"))
    layer.warmup(64)
    layer.forward(torch.zeros((17, H), dtype=torch.bfloat16, device="cuda"),
                  torch.ones((17, k), device="cuda"), torch.zeros((17, k), dtype=torch.int32, device="cuda"))
    torch.cuda.synchronize()


# ---- BASELINE configs at full size ---------------------------------------------------------------

def test_config1_bf16_full_size():
    """H 1024, 16 experts, top-2, I 2816, bf16 N(0, 0.02), 64 tokens, seed 0."""
    rng = np.random.default_rng(0)
    E, k, H, I, T = 16, 2, 1024, 2816, 64
    q, d = make_stacks(rng, E, H, I, O.DT_BF16)
    router = O.f32_to_bf16(rng.normal(0, 0.02, (E, H)).astype(np.float32))
    layer = build_layer(q, E, k, H, I, O.DT_BF16, router=router, mode=1, max_tokens=T)
    x = O.f32_to_bf16(rng.normal(0, 1, (T, H)).astype(np.float32))
    xt = bf16_tensor(x)
    ids, ws = layer.route(xt)
    y = layer.forward(xt, ws, ids)
    torch.cuda.synchronize()
    rid, rw = O.route(O.router_logits(x, router), k, 1)
    assert np.array_equal(ids.cpu().numpy().astype(np.uint32), rid)
    want = O.moe_forward_f32(O.bf16_to_f32(x).reshape(T, H), rid, rw, *d)
    assert_close(y.float().cpu().numpy(), want)


@pytest.mark.parametrize("T", [1, 32, 256])
def test_config2_q8_0_full_size(T):
    """Qwen3-30B-A3B-shaped decode layer, Q8_0, top-8 renormalised softmax. The
    weights sit in 128 x 128 units; T = 1 and 32 run the decode GEMV, T = 256 the tcgen05 GEMM."""
    rng = np.random.default_rng(2)
    E, k, H, I = 128, 8, 2048, 768
    gate = rng.normal(0, 0.02, (E, I, H)).astype(np.float32)
    up = rng.normal(0, 0.02, (E, I, H)).astype(np.float32)
    down = rng.normal(0, 0.02, (E, H, I)).astype(np.float32)
    q = [O.quantize(O.DT_Q8_0, w)[0] for w in (gate, up, down)]
    del gate, up, down
    router = O.f32_to_bf16(rng.normal(0, 0.02, (E, H)).astype(np.float32))
    layer = build_layer(q, E, k, H, I, O.DT_Q8_0, router=router, mode=1, max_tokens=256)
    x = O.f32_to_bf16(rng.normal(0, 1, (T, H)).astype(np.float32))
    xt = bf16_tensor(x)
    ids, ws = layer.route(xt)
    y = layer.forward(xt, ws, ids)
    torch.cuda.synchronize()
    rid, rw = O.route(O.router_logits(x, router), k, 1)
    assert np.array_equal(ids.cpu().numpy().astype(np.uint32), rid)
    assert np.array_equal(ws.cpu().numpy().view(np.uint32), rw.view(np.uint32))
    want = O.moe_forward_ref(O.DT_Q8_0, q, O.bf16_to_f32(x).reshape(T, H), rid, rw, E, H, I)
    assert_close(y.float().cpu().numpy(), want)
