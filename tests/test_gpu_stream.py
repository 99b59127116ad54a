"""The shared-memory weight stream (csrc/expert_stream.cu) against the dequantised reference and the
register-staged decode GEMV.

Each warp of the stream sums its 16 rows over the whole K in block order, as the GEMV does when one
warp owns a full row tile; at small batches the GEMV splits K across warps instead, so the two agree
to rounding, not bit for bit. Both must meet the north-star tolerance against the dequantised
reference at every batch size, through the expert cache's slot map too. The kernel choice is read
from MOE_DECODE once per process, so each variant runs in its own child process on the same seeded
inputs and writes its outputs.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

from oracle import oracle as O
from tolerance import assert_close

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)

CHILD = r'''
import sys, numpy as np, torch
sys.path[:0] = [sys.argv[2], sys.argv[3]]
import moe_b200 as M
from oracle import oracle as O
E, k, H, I = int(sys.argv[4]), 8, int(sys.argv[5]), int(sys.argv[6])
rng = np.random.default_rng(7)
q = [O.quantize(O.DT_Q8_0, rng.normal(0, 0.02, s).astype(np.float32))[0] for s in ((E, I, H), (E, I, H), (E, H, I))]
cfg = M.MoeConfig(num_experts=E, num_experts_per_tok=k, hidden_size=H, moe_intermediate_size=I)
out = {}
for slots in (0, E // 2):
    L = M.RoutedExpertsProvider().build(M.ExpertLoadContext(layer=0, device=0, config=cfg, wdtype=M.DTYPE_Q8_0,
        gate=q[0], up=q[1], down=q[2], max_tokens=256, cache_slots=slots))
    if slots:
        L.cache_upload(range(0, E, 2))  # every other expert resident: the slot map skips the rest
    for T in (1, 5, 32, 100, 256):
        r = np.random.default_rng(100 + T)
        x = torch.from_numpy(O.f32_to_bf16(r.normal(0, 1, (T, H)).astype(np.float32)).view(np.int16)).view(torch.bfloat16).cuda()
        ids = np.stack([r.permutation(E)[:k] for _ in range(T)]).astype(np.int32)
        w = r.dirichlet(np.ones(k), T).astype(np.float32)
        y = L.forward(x, torch.from_numpy(w).cuda(), torch.from_numpy(ids).cuda())
        torch.cuda.synchronize()
        L.check()
        out[f"s{slots}_T{T}"] = y.view(torch.int16).cpu().numpy()
        out[f"s{slots}_T{T}_x"] = x.view(torch.int16).cpu().numpy()
        out[f"s{slots}_T{T}_ids"] = ids
        out[f"s{slots}_T{T}_w"] = w
    L.close()
np.savez(sys.argv[1], **out)
'''


def _run(tmp_path, mode, E, H, I):
    path = str(tmp_path / f"{mode}.npz")
    env = dict(os.environ, MOE_DECODE=mode, MOE_Q8_PATH="gemv")  # no tcgen05 hand-over: both sides stream
    r = subprocess.run(["timeout", "-k", "10", "600", sys.executable, "-c", CHILD, path, ROOT,
                        os.path.join(ROOT, "naiwa-rs_b200"), str(E), str(H), str(I)],
                       capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-3000:]
    return np.load(path)


@pytest.mark.parametrize("E,H,I", [(16, 256, 128), (128, 2048, 768)])
def test_stream_matches_reference_and_gemv(tmp_path, E, H, I):
    a = _run(tmp_path, "gemv", E, H, I)
    b = _run(tmp_path, "stream", E, H, I)
    rng = np.random.default_rng(7)
    q = [O.quantize(O.DT_Q8_0, rng.normal(0, 0.02, s).astype(np.float32))[0]
         for s in ((E, I, H), (E, I, H), (E, H, I))]
    for key in a.files:
        if not key.endswith(("_x", "_ids", "_w")):
            T = int(key.split("_T")[1])
            got = O.bf16_to_f32(b[key].view(np.uint16)).reshape(T, H)
            gemv = O.bf16_to_f32(a[key].view(np.uint16)).reshape(T, H)
            assert_close(got, gemv, what=f"{key} stream vs gemv")
            if key.startswith("s0"):  # resident layer: against the dequantised reference
                x = O.bf16_to_f32(b[key + "_x"].view(np.uint16)).reshape(T, H)
                want = O.moe_forward_ref(O.DT_Q8_0, q, x, b[key + "_ids"].astype(np.uint32), b[key + "_w"], E, H, I)
                assert_close(got, want, what=f"{key} stream vs reference")
