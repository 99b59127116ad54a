"""Tensor-core (tcgen05) grouped-GEMM path: Q4_K and FP8 e4m3 (128x128 block scales) layers.

Weights are dequantised to f16 inside the kernel; activations are staged as f16 with a
power-of-two row scale. Outputs must stay within max |y - ref| / max |ref| <= 1e-2 of the oracle's
double-accumulated dequantised reference and within the elementwise bound
of tests/tolerance.py on every token.
"""
import numpy as np
import pytest

from oracle import oracle as O
from tolerance import assert_close

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

def bf16_tensor(a_u16):
    return torch.from_numpy(np.ascontiguousarray(a_u16).view(np.int16)).view(torch.bfloat16).cuda()


def quant_stacks(rng, E, H, I, dtype, std=0.02):
    out_q, out_s, out_d = [], [], []
    for shape in ((E, I, H), (E, I, H), (E, H, I)):
        w = rng.normal(0, std, shape).astype(np.float32)
        q, s = O.quantize(dtype, w)
        out_q.append(q)
        out_s.append(s)
        out_d.append(O.dequantize(dtype, q, shape, s))
    return out_q, out_s, out_d


def build(q, s, E, k, H, I, dtype, max_tokens, router=None):
    import moe_b200 as M

    cfg = M.MoeConfig(num_experts=E, num_experts_per_tok=k, hidden_size=H, moe_intermediate_size=I,
                      router_mode=M.ROUTER_SOFTMAX_RENORM)
    ctx = M.ExpertLoadContext(layer=0, device=0, config=cfg, wdtype=dtype, gate=q[0], up=q[1], down=q[2],
                              gate_scale=s[0], up_scale=s[1], down_scale=s[2], router_weight=router,
                              max_tokens=max_tokens)
    return M.RoutedExpertsProvider().build(ctx)


def run(layer, x_u16, ids, ws):
    y = layer.forward(bf16_tensor(x_u16), torch.from_numpy(ws).cuda(), torch.from_numpy(ids.view(np.int32)).cuda())
    torch.cuda.synchronize()
    layer.check()
    return y.float().cpu().numpy()


def random_routing(rng, T, E, k, skew=0.0):
    if skew:
        p = 1.0 / np.arange(1, E + 1) ** skew
        p /= p.sum()
        ids = np.stack([rng.choice(E, size=k, replace=False, p=p) for _ in range(T)])
    else:
        ids = np.stack([rng.permutation(E)[:k] for _ in range(T)])
    return ids.astype(np.uint32), rng.dirichlet(np.ones(k), T).astype(np.float32)


@pytest.mark.parametrize("dtype,H,I", [(O.DT_Q4_K, 512, 256), (O.DT_FP8, 256, 256), (O.DT_FP8, 384, 128)])
@pytest.mark.parametrize("T", [1, 37, 60, 96, 300])
def test_tc_layer_matches_dequantised_reference(dtype, H, I, T):
    rng = np.random.default_rng(1000 + T + dtype + H)
    E, k = 8, 2
    q, s, d = quant_stacks(rng, E, H, I, dtype)
    layer = build(q, s, E, k, H, I, dtype, max_tokens=max(T, 8))
    x = O.f32_to_bf16(rng.normal(0, 1, (T, H)).astype(np.float32))
    ids, ws = random_routing(rng, T, E, k, skew=1.1 if T > 50 else 0.0)
    got = run(layer, x, ids, ws)
    want = O.moe_forward_f32(O.bf16_to_f32(x).reshape(T, H), ids, ws, *d)
    assert_close(got, want)


def test_tc_weight_zero_padding_and_bad_ids():
    rng = np.random.default_rng(5)
    E, k, H, I = 8, 2, 256, 256
    q, s, d = quant_stacks(rng, E, H, I, O.DT_Q4_K)
    layer = build(q, s, E, k, H, I, O.DT_Q4_K, max_tokens=16)
    x = O.f32_to_bf16(rng.normal(0, 1, (4, H)).astype(np.float32))
    ids, ws = random_routing(rng, 4, E, k)
    base = run(layer, x, ids, ws)
    pad_i = np.concatenate([ids, ids[:, :1]], 1).astype(np.uint32)
    pad_w = np.concatenate([ws, np.zeros((4, 1), np.float32)], 1)
    assert np.array_equal(run(layer, x, pad_i, pad_w), base)


def fast_stacks(rng, E, H, I, dtype, std=0.02):
    """Quantised stacks (and FP8 block scales) of seeded N(0, std) weights, without dequantised copies."""
    qs, ss = [], []
    for shape in ((E, I, H), (E, I, H), (E, H, I)):
        w = rng.standard_normal(shape, dtype=np.float32)
        w *= np.float32(std)
        q, s = O.quantize(dtype, w)
        del w
        qs.append(q)
        ss.append(s)
    return qs, ss


def test_config3_shaped_q4k_prefill_chunk():
    """the config-2 layer in Q4_K, a full 512-token prefill chunk, Zipf(1.1) routing,
    every token against the dequantised reference."""
    rng = np.random.default_rng(3)
    E, k, H, I, T = 128, 8, 2048, 768, 512
    q, s = fast_stacks(rng, E, H, I, O.DT_Q4_K)
    layer = build(q, s, E, k, H, I, O.DT_Q4_K, max_tokens=T)
    x = O.f32_to_bf16(rng.normal(0, 1, (T, H)).astype(np.float32))
    ids, ws = random_routing(rng, T, E, k, skew=1.1)
    got = run(layer, x, ids, ws)
    want = O.moe_forward_ref(O.DT_Q4_K, q, O.bf16_to_f32(x).reshape(T, H), ids, ws, E, H, I)
    assert_close(got, want, what="config 3, 512-token chunk")


def test_config5_shaped_fp8_shard():
    """BASELINE config 5 shapes (H 7168, I 2048, FP8 e4m3 128x128): one GPU's shard of an 8-way split,
    32 local experts, 128 tokens of top-8; every token against the dequantised reference."""
    rng = np.random.default_rng(5)
    E, k, H, I, T = 32, 8, 7168, 2048, 128
    q, s = fast_stacks(rng, E, H, I, O.DT_FP8)
    layer = build(q, s, E, k, H, I, O.DT_FP8, max_tokens=T)
    x = O.f32_to_bf16(rng.normal(0, 1, (T, H)).astype(np.float32))
    ids, ws = random_routing(rng, T, E, k)
    got = run(layer, x, ids, ws)
    want = O.moe_forward_ref(O.DT_FP8, q, O.bf16_to_f32(x).reshape(T, H), ids, ws, E, H, I, scales=s)
    assert_close(got, want, what="config 5, E32 shard")


def test_tc_back_to_back_calls_and_graph_replay_bit_exact():
    """The GEMM launches take their work items from per-launch counters that the tile-list kernel zeroes
    at every call. Calls of different sizes issued back to back on one stream (no host sync between
    them), and the same calls replayed from a CUDA graph, must give bit-for-bit the outputs of the same
    calls run one at a time: which CTA takes which item may change, an item's arithmetic may not."""
    rng = np.random.default_rng(77)
    E, k, H, I = 16, 4, 512, 256
    q, s, _ = quant_stacks(rng, E, H, I, O.DT_Q4_K)
    layer = build(q, s, E, k, H, I, O.DT_Q4_K, max_tokens=400)
    cases = []
    for T in (300, 40, 400, 129):  # prefill and decode token tiles, counters reused across sizes
        x = bf16_tensor(O.f32_to_bf16(rng.normal(0, 1, (T, H)).astype(np.float32)))
        ids, ws = random_routing(rng, T, E, k, skew=1.1)
        cases.append((x, torch.from_numpy(ws).cuda(), torch.from_numpy(ids.view(np.int32)).cuda()))
    alone = []
    for x, w, i in cases:
        alone.append(layer.forward(x, w, i).clone())
        torch.cuda.synchronize()
    layer.check()
    outs = [torch.empty_like(c[0]) for c in cases]
    for _ in range(2):
        for (x, w, i), o in zip(cases, outs):
            layer.forward(x, w, i, out=o)
    torch.cuda.synchronize()
    layer.check()
    for a, o in zip(alone, outs):
        assert torch.equal(a, o), "back-to-back calls differ from single calls"
    stream = torch.cuda.Stream()
    gouts = [torch.empty_like(c[0]) for c in cases]
    with torch.cuda.stream(stream):  # capture needs a warmed-up, non-default stream
        for (x, w, i), o in zip(cases, gouts):
            layer.forward(x, w, i, out=o, stream=stream)
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        for (x, w, i), o in zip(cases, gouts):
            layer.forward(x, w, i, out=o, stream=stream)
    for _ in range(3):
        for o in gouts:
            o.zero_()
        graph.replay()
        torch.cuda.synchronize()
        for a, o in zip(alone, gouts):
            assert torch.equal(a, o), "graph replay differs from single calls"
    del graph
    layer.check()
    layer.close()
