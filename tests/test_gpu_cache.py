"""Expert cache on the GPU: route split (a2), paging (a8), cached forward.

A cached layer (cache_slots < E) must give bit-for-bit the output of an all-resident layer whose
non-resident experts' pairs are replaced by MOE_ID_NONE: the slot only relocates the same repacked
bytes. Steps are issued back to back without host syncs, so uploads for step s run on the copy
stream while earlier forwards still read the slots they will overwrite (the read fence orders them).
"""
import numpy as np
import pytest

from oracle import oracle as O

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def quant_stacks(rng, E, H, I, dtype, std=0.02):
    out_q, out_s = [], []
    for shape in ((E, I, H), (E, I, H), (E, H, I)):
        q, s = O.quantize(dtype, rng.normal(0, std, shape).astype(np.float32))
        out_q.append(q)
        out_s.append(s)
    return out_q, out_s


def build(q, s, E, k, H, I, dtype, max_tokens, slots=0):
    import moe_b200 as M

    cfg = M.MoeConfig(num_experts=E, num_experts_per_tok=k, hidden_size=H, moe_intermediate_size=I)
    return M.RoutedExpertsProvider().build(M.ExpertLoadContext(
        layer=0, device=0, config=cfg, wdtype=dtype, gate=q[0], up=q[1], down=q[2], gate_scale=s[0],
        up_scale=s[1], down_scale=s[2], max_tokens=max_tokens, cache_slots=slots))


def to_dev_bf16(a):
    return torch.from_numpy(O.f32_to_bf16(a).view(np.int16)).view(torch.bfloat16).cuda()


@pytest.mark.parametrize("dtype,E,k,H,I,slots,tmax", [(O.DT_Q8_0, 16, 4, 256, 128, 6, 12),
                                                       (O.DT_FP8, 8, 2, 256, 256, 3, 40)])
def test_cached_forward_matches_resident_layer(dtype, E, k, H, I, slots, tmax):
    rng = np.random.default_rng(21 + dtype)
    q, s = quant_stacks(rng, E, H, I, dtype)
    full = build(q, s, E, k, H, I, dtype, tmax)
    cached = build(q, s, E, k, H, I, dtype, tmax, slots=slots)
    assert cached.cache_slots == slots and list(cached.cache_resident()) == [-1] * slots
    pop = 1.0 / np.arange(1, E + 1) ** 1.2
    pop /= pop.sum()
    outs, refs = [], []
    n_routed = 0
    for step in range(40):
        T = int(rng.integers(1, tmax + 1))
        ids = np.stack([rng.choice(E, size=k, replace=False, p=pop) for _ in range(T)]).astype(np.uint32)
        w = rng.dirichlet(np.ones(k), T).astype(np.float32)
        x = to_dev_bf16(rng.normal(0, 1, (T, H)).astype(np.float32))
        hit = cached.cache_split(ids)
        n_routed += ids.size
        miss = sorted(set(ids.reshape(-1)[hit == 0].tolist()))
        keep = sorted(set(ids.reshape(-1)[hit == 1].tolist()))
        cached.cache_upload(miss, protect=keep)  # may bring in fewer than asked when slots run out
        resident = set(int(e) for e in cached.cache_resident() if e >= 0)
        ids_t = torch.from_numpy(ids.view(np.int32)).cuda()
        w_t = torch.from_numpy(w).cuda()
        outs.append(cached.forward(x, w_t, ids_t))
        masked = np.where(np.isin(ids, list(resident)), ids, np.uint32(O.ID_NONE)).astype(np.uint32)
        refs.append(full.forward(x, w_t, torch.from_numpy(masked.view(np.int32)).cuda()))
    torch.cuda.synchronize()
    cached.check()
    full.check()
    for a, b in zip(outs, refs):
        assert torch.equal(a, b)
    st = cached.cache_stats()
    assert st["hits"] + st["misses"] == n_routed and st["uploads"] > slots and st["hits"] > 0
    assert int(st["hit_counts"].sum()) == n_routed


def test_lru_replacement_and_protection():
    rng = np.random.default_rng(4)
    E, k, H, I = 8, 1, 64, 64
    q, s = quant_stacks(rng, E, H, I, O.DT_Q8_0)
    L = build(q, s, E, k, H, I, O.DT_Q8_0, 4, slots=2)
    assert L.cache_upload([0, 1]) == 2
    assert sorted(L.cache_resident().tolist()) == [0, 1]
    assert L.cache_split(np.array([[0]])).tolist() == [1]  # touch 0: expert 1 is now least recent
    assert L.cache_upload([2]) == 1
    assert sorted(L.cache_resident().tolist()) == [0, 2]
    assert L.cache_upload([3], protect=[0]) == 1  # 0 protected: 2 goes
    assert sorted(L.cache_resident().tolist()) == [0, 3]
    assert L.cache_upload([4, 5, 6], protect=[]) == 2  # only two slots: the third cannot come in
    assert sorted(L.cache_resident().tolist()) == [4, 5]
    assert L.cache_split(np.array([[5], [7], [0xFFFFFFFF]], np.uint32)).tolist() == [1, 0, 2]
    torch.cuda.synchronize()
    L.check()
