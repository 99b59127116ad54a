"""The paged decode flow on the GPU: top-k and activation doorbells, route split, streamed uploads,
CPU executor for the remaining misses, result doorbell, fold into the GPU output. Its output must
match an all-resident layer within the north-star tolerance (the GPU part is bf16-rounded before the
CPU rows are added, so the comparison is not bit-exact)."""
import numpy as np
import pytest

from oracle import oracle as O
from tolerance import assert_close

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def setup(E=16, k=4, H=256, I=128, slots=4, T_max=16, seed=9):
    import moe_b200 as M

    rng = np.random.default_rng(seed)
    q = [O.quantize(O.DT_Q8_0, rng.normal(0, 0.02, shape).astype(np.float32))[0]
         for shape in ((E, I, H), (E, I, H), (E, H, I))]
    cfg = M.MoeConfig(num_experts=E, num_experts_per_tok=k, hidden_size=H, moe_intermediate_size=I)

    def build(slots_):
        return M.RoutedExpertsProvider().build(M.ExpertLoadContext(
            layer=0, device=0, config=cfg, wdtype=O.DT_Q8_0, gate=q[0], up=q[1], down=q[2], max_tokens=T_max,
            cache_slots=slots_))

    return rng, build(0), build(slots), M.CpuExperts(E, k, H, I, O.DT_Q8_0, *q, threads=4)


@pytest.mark.parametrize("frac", [0.0, 0.5, 1.0])
def test_paged_decode_matches_resident_layer(frac):
    import moe_b200 as M

    E, k, H = 16, 4, 256
    rng, full, cached, cpu = setup()
    cached.cache_upload([0, 1, 2, 3])  # the fill thread's work: the most-routed experts first
    paged = M.PagedMoE(cached, cpu=cpu, pcie_frac=frac, max_tokens=16)
    pop = 1.0 / np.arange(1, E + 1) ** 1.1
    pop /= pop.sum()
    for step in range(25):
        T = int(rng.integers(1, 17))
        ids = np.stack([rng.choice(E, size=k, replace=False, p=pop) for _ in range(T)]).astype(np.int32)
        w = rng.dirichlet(np.ones(k), T).astype(np.float32)
        x = torch.from_numpy(O.f32_to_bf16(rng.normal(0, 1, (T, H)).astype(np.float32)).view(np.int16)) \
            .view(torch.bfloat16).cuda()
        ids_t, w_t = torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda()
        y = paged.forward(x, w_t, ids_t)
        ref = full.forward(x, w_t, ids_t)
        torch.cuda.synchronize()
        assert_close(y.float().cpu().numpy(), ref.float().cpu().numpy(), what=f"step {step}")
    paged.check()
    s = paged.stats
    assert s["hits"] > 0
    if frac == 0.0:
        assert s["streamed"] == 0 and s["cpu_pairs"] > 0
    if frac == 1.0:
        assert s["streamed"] > 0
    paged.close()


def test_executor_latches_worker_errors():
    import moe_b200 as M

    E, k, H = 16, 4, 256
    rng, full, cached, cpu = setup()
    ring = M.Ring(0, 2, 4 * H * 4)
    ex = M.Executor(cpu, ring)
    x = O.f32_to_bf16(rng.normal(0, 1, (2, H)).astype(np.float32)).reshape(2, H)
    w = np.ones((2, k), np.float32)
    t1 = ex.submit(x, np.full((2, k), 99, np.uint32), w)  # ids >= E: the job fails, publishes zeros
    dst = torch.full((2 * H,), 7.0, device="cuda")
    ring.device_take(t1, dst)
    ring.check()
    assert torch.count_nonzero(dst).item() == 0
    with pytest.raises(M.MoeError) as e:
        ex.submit(x, np.zeros((2, k), np.uint32), w)
    assert e.value.status == 7  # MOE_ERR_WORKER, from the earlier job
    t2 = ex.submit(x, np.zeros((2, k), np.uint32), w)  # the executor keeps working
    ring.device_take(t2, dst)
    ring.check()
    want = cpu.forward(x, np.zeros((2, k), np.uint32), w).reshape(-1)
    assert np.allclose(dst.cpu().numpy(), want)
    ex.close()
    ring.close()


def test_chunked_forward_matches_single_pass():
    import moe_b200 as M

    E, k, H = 16, 4, 256
    rng, full, cached, cpu = setup(T_max=16)
    T = 100  # > max_tokens: six chunks and a ragged tail
    ids = torch.from_numpy(np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)).cuda()
    w = torch.from_numpy(rng.dirichlet(np.ones(k), T).astype(np.float32)).cuda()
    x = torch.from_numpy(O.f32_to_bf16(rng.normal(0, 1, (T, H)).astype(np.float32)).view(np.int16)) \
        .view(torch.bfloat16).cuda()
    y = full.forward_chunked(x, w, ids)
    for c0 in range(0, T, 16):  # each chunk alone, bit-exact
        assert torch.equal(y[c0:c0 + 16], full.forward(x[c0:c0 + 16], w[c0:c0 + 16], ids[c0:c0 + 16]))
    paged = M.PagedMoE(cached, cpu=None, max_tokens=16)
    yp = paged.prefill(x, w, ids)  # every chunk touches all 16 experts: resident wave + 2 staged waves
    torch.cuda.synchronize()
    # waves leave per-pair outputs and one combine per chunk sums them: the resident layer's bits
    assert torch.equal(yp, y)
    s = paged.stats
    assert s["prefill_waves"] >= 2 * ((T + 15) // 16) and s["prefill_uploads"] > 0
    paged.check()
    paged.close()


# ---- the native paged runtime: staging, lookahead, bit-exactness -----------------------------------

def setup_chain(n_layers=2, E=16, k=4, H=256, I=128, slots=4, T_max=16, same_router=False, seed=21):
    """n_layers cached layers (with routers) and their all-resident twins."""
    import moe_b200 as M

    rng = np.random.default_rng(seed)
    cfg = M.MoeConfig(num_experts=E, num_experts_per_tok=k, hidden_size=H, moe_intermediate_size=I)
    router0 = O.f32_to_bf16(rng.normal(0, 0.05, (E, H)).astype(np.float32)).reshape(E, H)
    full, cached = [], []
    for li in range(n_layers):
        q = [O.quantize(O.DT_Q8_0, rng.normal(0, 0.02, shape).astype(np.float32))[0]
             for shape in ((E, I, H), (E, I, H), (E, H, I))]
        router = router0 if same_router else O.f32_to_bf16(rng.normal(0, 0.05, (E, H)).astype(np.float32)).reshape(E, H)

        def build(slots_):
            return M.RoutedExpertsProvider().build(M.ExpertLoadContext(
                layer=li, device=0, config=cfg, wdtype=O.DT_Q8_0, gate=q[0], up=q[1], down=q[2], router_weight=router,
                max_tokens=T_max, cache_slots=slots_))

        full.append(build(0))
        cached.append(build(slots))
    return rng, full, cached


def test_gpu_part_is_bit_exact_with_staging_and_lookahead():
    """No CPU path, staging slots for every miss, a two-layer lookahead chain: every output equals the
    all-resident layer's bit for bit, while the cache, the staging slots and the lookahead all work."""
    import moe_b200 as M

    E, k, H = 16, 4, 256
    rng, full, cached = setup_chain()
    for c in cached:
        c.cache_upload([0, 1, 2, 3])
    paged = [M.PagedMoE(c, cpu=None, max_tokens=16, staging_slots=12, stream_cap=12) for c in cached]
    paged[0].set_next(paged[1])
    for step in range(12):
        T = int(rng.integers(1, 17))
        x = torch.from_numpy(O.f32_to_bf16(rng.normal(0, 1, (T, H)).astype(np.float32)).view(np.int16)) \
            .view(torch.bfloat16).cuda()
        for li in range(2):
            ids, w = full[li].route(x)
            y = paged[li].forward(x, w, ids)
            ref = full[li].forward(x, w, ids)
            torch.cuda.synchronize()
            assert torch.equal(y, ref), (step, li)
        M.PagedMoE.drain_lookahead()
    for p in paged:
        p.check()
    s0, s1 = paged[0].stats, paged[1].stats
    assert s0["staged_experts"] > 0 and s0["cpu_pairs"] == 0 and s1["cpu_pairs"] == 0
    assert s1["lookahead_passes"] == 12 and s1["lookahead_loads"] > 0
    for p in paged:
        p.close()


def test_lookahead_prediction_turns_misses_into_hits():
    """Layer 1 has layer 0's router and sees the same activation: the lookahead predicts its experts
    exactly, so after layer 0's call (and the prediction) layer 1 runs with every pair a hit."""
    import moe_b200 as M

    E, k, H = 16, 2, 256
    rng, full, cached = setup_chain(k=k, slots=8, same_router=True, seed=5)
    paged = [M.PagedMoE(c, cpu=None, max_tokens=16, staging_slots=8, stream_cap=8, lookahead_swaps=4)
             for c in cached]
    paged[0].set_next(paged[1])
    hits_before = paged[1].stats["hits"]
    x = torch.from_numpy(O.f32_to_bf16(rng.normal(0, 1, (2, H)).astype(np.float32)).view(np.int16)) \
        .view(torch.bfloat16).cuda()
    ids, w = full[0].route(x)
    paged[0].forward(x, w, ids)
    M.PagedMoE.drain_lookahead()
    y1 = paged[1].forward(x, w, ids)  # same router, same x: the prediction was exact
    torch.cuda.synchronize()
    s1 = paged[1].stats
    assert s1["lookahead_loads"] > 0
    assert s1["hits"] - hits_before == s1["pairs"] and s1["staged_experts"] == 0
    assert torch.equal(y1, full[1].forward(x, w, ids))
    for p in paged:
        p.check()
        p.close()
