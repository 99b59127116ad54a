"""The resident Q2_0 pool on the GPU (the reference's resident.rs): the device requantiser against the
oracle's restatement of quantize_q2_0, and Q2_0 layers through the decode expert kernels against the
dequantised reference.

  * moe_requantize_q2_0 must give the oracle's bytes exactly, from BF16, Q8_0 and Q4_K stacks: the
    oracle dequantises the source and runs the same scale-ladder search on the CPU;
  * a Q2_0 layer's outputs must meet the north-star tolerance (tests/tolerance.py) against
    moe_forward_ref of its own dequantised weights, at batch sizes from 1 to 256, including the
    config-2 shape;
  * RoutedExpertsProvider.build_resident (requantise on the device, then build) must give the same
    bits as building from the oracle's requantised stacks.
"""
import numpy as np
import pytest

from oracle import oracle as O
from tolerance import assert_close

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def M():
    if not torch.cuda.is_available():
        pytest.skip("needs a GPU")
    import moe_b200
    return moe_b200


def bf16_tensor(a_f32):
    return torch.from_numpy(O.f32_to_bf16(a_f32).view(np.int16)).view(torch.bfloat16).cuda()


@pytest.mark.parametrize("src_dtype,N,K", [(O.DT_Q8_0, 48, 256), (O.DT_Q4_K, 32, 512), (O.DT_BF16, 16, 192),
                                           (O.DT_Q8_0, 768, 2048)])
def test_requantize_matches_oracle_bytes(M, src_dtype, N, K):
    rng = np.random.default_rng(40 + src_dtype + N)
    E = 3
    w = rng.normal(0, 0.02, (E, N, K)).astype(np.float32)
    w[1, 2, :64] = 0.0  # an all-zero block
    w[2, 5, 64:128] = rng.normal(0, 1e-7, 64).astype(np.float32)  # a block near the f16 floor
    src, _ = O.quantize(src_dtype, w)
    want, _ = O.quantize(O.DT_Q2_0, O.dequantize(src_dtype, src, w.shape))
    got = M.requantize_q2_0(src, src_dtype, E, N, K).cpu().numpy()
    assert got.shape == want.shape
    bad = np.nonzero(got != want)[0]
    assert bad.size == 0, f"{bad.size} bytes differ, first at {bad[:8]}"


def _layer(M, E, k, H, I, seed, max_tokens, resident_from=None):
    rng = np.random.default_rng(seed)
    f = [rng.normal(0, 0.02, s).astype(np.float32) for s in ((E, I, H), (E, I, H), (E, H, I))]
    if resident_from is None:
        q = [O.quantize(O.DT_Q2_0, a)[0] for a in f]
        dtype = O.DT_Q2_0
    else:
        q = [O.quantize(resident_from, a)[0] for a in f]
        dtype = resident_from
    cfg = M.MoeConfig(num_experts=E, num_experts_per_tok=k, hidden_size=H, moe_intermediate_size=I)
    ctx = M.ExpertLoadContext(layer=0, device=0, config=cfg, wdtype=dtype, gate=q[0], up=q[1], down=q[2],
                              max_tokens=max_tokens)
    prov = M.RoutedExpertsProvider()
    layer = prov.build_resident(ctx) if resident_from is not None else prov.build(ctx)
    return layer, q


@pytest.mark.parametrize("E,k,H,I,Ts", [(16, 4, 256, 128, (1, 9, 33, 100)), (32, 8, 512, 256, (5, 256)),
                                        (128, 8, 2048, 768, (1, 32))])
def test_q2_0_layer_matches_dequantised_reference(M, E, k, H, I, Ts):
    layer, q = _layer(M, E, k, H, I, seed=7 + E, max_tokens=max(Ts))
    rng = np.random.default_rng(100 + E)
    for T in Ts:
        x = rng.normal(0, 1, (T, H)).astype(np.float32)
        xb = O.f32_to_bf16(x)
        ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.uint32)
        w = rng.dirichlet(np.ones(k), T).astype(np.float32)
        y = layer.forward(bf16_tensor(x), torch.from_numpy(w).cuda(), torch.from_numpy(ids.view(np.int32)).cuda())
        torch.cuda.synchronize()
        layer.check()
        want = O.moe_forward_ref(O.DT_Q2_0, q, O.bf16_to_f32(xb).reshape(T, H), ids, w, E, H, I)
        assert_close(y.float().cpu().numpy(), want, what=f"Q2_0 E{E} T{T}")
    layer.close()


@pytest.mark.parametrize("src", [O.DT_Q8_0, O.DT_Q4_K])
def test_build_resident_equals_oracle_requantised_layer(M, src):
    E, k, H, I, T = 16, 4, 256, 256, 24
    resident, q_src = _layer(M, E, k, H, I, seed=3, max_tokens=T, resident_from=src)
    q2 = [O.quantize(O.DT_Q2_0, O.dequantize(src, a, shape))[0]
          for a, shape in zip(q_src, ((E, I, H), (E, I, H), (E, H, I)))]
    cfg = M.MoeConfig(num_experts=E, num_experts_per_tok=k, hidden_size=H, moe_intermediate_size=I)
    direct = M.RoutedExpertsProvider().build(M.ExpertLoadContext(
        layer=0, device=0, config=cfg, wdtype=M.DTYPE_Q2_0, gate=q2[0], up=q2[1], down=q2[2], max_tokens=T))
    rng = np.random.default_rng(9)
    x = bf16_tensor(rng.normal(0, 1, (T, H)).astype(np.float32))
    ids = torch.from_numpy(np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.int32)).cuda()
    w = torch.from_numpy(rng.dirichlet(np.ones(k), T).astype(np.float32)).cuda()
    a = resident.forward(x, w, ids)
    b = direct.forward(x, w, ids)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    resident.close()
    direct.close()
