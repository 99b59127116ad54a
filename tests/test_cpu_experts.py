"""The library's CPU expert path (moe_cpu_forward, host threads) against the oracle's dequantised
f32 reference, with a selection mask, empty slots and weight-0 slots. CPU only."""
import numpy as np
import pytest

from oracle import oracle as O


@pytest.mark.parametrize("dtype", [O.DT_Q8_0, O.DT_BF16])
def test_cpu_forward_matches_oracle(dtype):
    import moe_b200 as M

    rng = np.random.default_rng(8 + dtype)
    E, k, H, I, T = 8, 3, 256, 128, 9
    q, d = [], []
    for shape in ((E, I, H), (E, I, H), (E, H, I)):
        wq, s = O.quantize(dtype, rng.normal(0, 0.05, shape).astype(np.float32))
        q.append(wq)
        d.append(O.dequantize(dtype, wq, shape, s))
    cpu = M.CpuExperts(E, k, H, I, dtype, *q, threads=3)
    x = O.f32_to_bf16(rng.normal(0, 1, (T, H)).astype(np.float32)).reshape(T, H)
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.uint32)
    ids[0, 1] = O.ID_NONE
    w = rng.random((T, k)).astype(np.float32)
    w[2, 0] = 0.0
    sel = (rng.random(T * k) < 0.6).astype(np.uint8)
    y = cpu.forward(x, ids, w, sel)
    masked = np.where(sel.reshape(T, k) != 0, ids, np.uint32(O.ID_NONE)).astype(np.uint32)
    want = O.moe_forward_f32(O.bf16_to_f32(x).reshape(T, H), masked, w, *d)
    assert np.abs(y - want).max() <= 1e-4 * max(np.abs(want).max(), 1e-6) + 1e-6
    assert np.array_equal(cpu.forward(x, ids, w, np.zeros(T * k, np.uint8)), np.zeros((T, H), np.float32))
    with pytest.raises(M.MoeError):
        cpu.forward(x, np.full((T, k), 99, np.uint32), w)
    cpu.close()
