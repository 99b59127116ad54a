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
    yp = paged.prefill(x, w, ids)  # every chunk touches all 16 experts: 4 waves of 4 slots
    torch.cuda.synchronize()
    assert_close(yp.float().cpu().numpy(), y.float().cpu().numpy())
    paged.check()
    paged.close()
