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


_ISA_CHECK = r"""
import sys
import numpy as np
sys.path.insert(0, {root!r}); sys.path.insert(0, {pkg!r})
from oracle import oracle as O
import moe_b200 as M
print(M.cpu_isa())
for dtype in (O.DT_Q8_0, O.DT_BF16):
    rng = np.random.default_rng(31 + dtype)
    E, k, H, I, T = 6, 2, 288, 160, 7
    q, d = [], []
    for shape in ((E, I, H), (E, I, H), (E, H, I)):
        wq, s = O.quantize(dtype, rng.normal(0, 0.05, shape).astype(np.float32))
        q.append(wq)
        d.append(O.dequantize(dtype, wq, shape, s))
    cpu = M.CpuExperts(E, k, H, I, dtype, *q, threads=2)
    x = O.f32_to_bf16(rng.normal(0, 1, (T, H)).astype(np.float32)).reshape(T, H)
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.uint32)
    ids[:, 0] = 1  # one expert serves every token: the row dots take 7 vectors, chunked by 4
    w = rng.random((T, k)).astype(np.float32)
    y = cpu.forward(x, ids, w)
    want = O.moe_forward_f32(O.bf16_to_f32(x).reshape(T, H), ids, w, *d)
    assert np.abs(y - want).max() <= 1e-4 * max(np.abs(want).max(), 1e-6) + 1e-6, dtype
    cpu.close()
"""


@pytest.mark.parametrize("isa", ["scalar", "avx2", "native"])
def test_cpu_dot_builds_match_oracle(isa):
    """Each build of the row dot products (MOE_CPU_ISA caps the one the host would pick) against the
    oracle, in a fresh process because the choice is made once per process."""
    import os
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    env = dict(os.environ)
    env.pop("MOE_CPU_ISA", None)
    if isa != "native":
        env["MOE_CPU_ISA"] = isa
    code = _ISA_CHECK.format(root=root, pkg=os.path.join(root, "naiwa-rs_b200"))
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    got = r.stdout.split()[0]
    if isa == "scalar":
        assert got == "scalar"
    elif isa == "avx2":
        assert got in ("avx2", "scalar")  # a host without AVX2 stays scalar
