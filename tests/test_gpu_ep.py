"""Expert parallelism on the GPU.

* the dispatch-plan, pack and combine kernels against the oracle's restatement (bit-exact: integer
  plans, copied rows, f32 sums of bf16 values rounded once);
* the whole EP data path with W ranks emulated on one GPU (each rank's local layer built from its
  slice of the expert stacks, the all-to-alls replaced by concatenations) against one full layer;
* the real NCCL path on two GPUs (torchrun, one process per GPU) when two GPUs are visible.
"""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

from oracle import oracle as O
from tolerance import assert_close

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def random_ids(rng, T, E, k, none_frac=0.0):
    ids = np.stack([rng.permutation(E)[:k] for _ in range(T)]).astype(np.uint32)
    if none_frac:
        ids[rng.random((T, k)) < none_frac] = O.ID_NONE
    return ids


@pytest.mark.parametrize("T,k,epr,world", [(1, 8, 32, 8), (3000, 8, 32, 8), (777, 4, 5, 3), (2048, 2, 1, 64)])
def test_dispatch_plan_bit_exact(T, k, epr, world):
    import moe_b200 as M

    rng = np.random.default_rng(T + world)
    ids = random_ids(rng, T, epr * world, k, none_frac=0.05)
    w = rng.random((T, k)).astype(np.float32)
    plan = M.ep_dispatch(torch.from_numpy(ids.view(np.int32)).cuda(), torch.from_numpy(w).cuda(), epr, world)
    torch.cuda.synchronize()
    rc, tr, st, sid, sw = O.ep_dispatch_plan(ids, w, epr, world)
    n = int(plan["n_send"].item())
    assert n == rc.sum()
    assert np.array_equal(plan["rank_counts"].cpu().numpy(), rc)
    assert np.array_equal(plan["token_rows"].cpu().numpy()[:T], tr)
    assert np.array_equal(plan["send_token"].cpu().numpy()[:n], st)
    assert np.array_equal(plan["send_ids"].cpu().numpy()[:n].view(np.uint32), sid)
    assert np.array_equal(plan["send_w"].cpu().numpy()[:n], sw)
    assert int(plan["error_word"].item()) == 0


def test_dispatch_plan_flags_bad_ids():
    import moe_b200 as M

    ids = np.array([[0, 70], [3, 1]], dtype=np.uint32)  # 70 >= 8 * 4
    w = np.ones((2, 2), np.float32)
    plan = M.ep_dispatch(torch.from_numpy(ids.view(np.int32)).cuda(), torch.from_numpy(w).cuda(), 4, 8)
    torch.cuda.synchronize()
    assert int(plan["error_word"].item()) == 5  # MOE_ERR_BAD_IDS
    assert plan["rank_counts"].cpu().tolist() == [2, 0, 0, 0, 0, 0, 0, 0]


def test_pack_and_combine_match_oracle():
    import moe_b200 as M

    rng = np.random.default_rng(7)
    T, H, k, epr, world = 300, 512, 8, 4, 8
    ids = random_ids(rng, T, epr * world, k)
    w = rng.random((T, k)).astype(np.float32)
    x = O.f32_to_bf16(rng.normal(0, 1, (T, H)).astype(np.float32))
    xt = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).cuda()
    plan = M.ep_dispatch(torch.from_numpy(ids.view(np.int32)).cuda(), torch.from_numpy(w).cuda(), epr, world)
    send_x = M.ep_pack_rows(xt, plan["send_token"], plan["n_send"], plan["cap"])
    torch.cuda.synchronize()
    rc, tr, st, _, _ = O.ep_dispatch_plan(ids, w, epr, world)
    n = int(rc.sum())
    assert np.array_equal(send_x[:n].cpu().view(torch.int16).numpy().view(np.uint16), x[st])
    yb = O.f32_to_bf16(rng.normal(0, 1, (n, H)).astype(np.float32))
    add = O.f32_to_bf16(rng.normal(0, 1, (T, H)).astype(np.float32))
    ybt = torch.from_numpy(yb.view(np.int16)).view(torch.bfloat16).cuda()
    addt = torch.from_numpy(add.view(np.int16)).view(torch.bfloat16).cuda()
    y = M.ep_combine(ybt, plan["token_rows"], T, y_add=addt)
    torch.cuda.synchronize()
    want = O.f32_to_bf16(O.ep_combine(O.bf16_to_f32(yb).reshape(n, H), tr, O.bf16_to_f32(add).reshape(T, H)))
    assert np.array_equal(y.cpu().view(torch.int16).numpy().view(np.uint16), want)


def quant_stacks(rng, E, H, I, dtype, std=0.02):
    out_q, out_s, out_d = [], [], []
    for shape in ((E, I, H), (E, I, H), (E, H, I)):
        wt = rng.normal(0, std, shape).astype(np.float32)
        q, s = O.quantize(dtype, wt)
        out_q.append(q)
        out_s.append(s)
        out_d.append(O.dequantize(dtype, q, shape, s))
    return out_q, out_s, out_d


def build(q, s, E, k, H, I, dtype, max_tokens):
    import moe_b200 as M

    cfg = M.MoeConfig(num_experts=E, num_experts_per_tok=k, hidden_size=H, moe_intermediate_size=I)
    ctx = M.ExpertLoadContext(layer=0, device=0, config=cfg, wdtype=dtype, gate=q[0], up=q[1], down=q[2],
                              gate_scale=s[0], up_scale=s[1], down_scale=s[2], max_tokens=max_tokens)
    return M.RoutedExpertsProvider().build(ctx)


def _slice(arrs, E, e0, e1):
    """Experts e0 .. e1-1 of stacked per-expert arrays (quant bytes or block scales)."""
    return [None if a is None else np.ascontiguousarray(np.asarray(a).reshape(E, -1)[e0:e1]).reshape(-1) for a in arrs]


@pytest.mark.parametrize("dtype,H,I", [(O.DT_FP8, 256, 256), (O.DT_Q8_0, 256, 128)])
def test_ep_emulated_ranks_match_full_layer(dtype, H, I):
    import moe_b200 as M

    rng = np.random.default_rng(11 + dtype)
    world, epr, k, T = 2, 8, 4, 64
    E = world * epr
    q, s, _ = quant_stacks(rng, E, H, I, dtype)
    full = build(q, s, E, k, H, I, dtype, max_tokens=T)
    locs = [build(_slice(q, E, r * epr, (r + 1) * epr), _slice(s, E, r * epr, (r + 1) * epr), epr, k,
                  H, I, dtype, max_tokens=T * world) for r in range(world)]
    xs, idss, ws = [], [], []
    for r in range(world):
        xs.append(torch.from_numpy(O.f32_to_bf16(rng.normal(0, 1, (T, H)).astype(np.float32)).view(np.int16))
                  .view(torch.bfloat16).cuda())
        idss.append(torch.from_numpy(random_ids(rng, T, E, k).view(np.int32)).cuda())
        ws.append(torch.from_numpy(rng.dirichlet(np.ones(k), T).astype(np.float32)).cuda())
    plans = [M.ep_dispatch(idss[r], ws[r], epr, world) for r in range(world)]
    send_x = [M.ep_pack_rows(xs[r], plans[r]["send_token"], plans[r]["n_send"], plans[r]["cap"]) for r in range(world)]
    counts = [plans[r]["rank_counts"].cpu().tolist() for r in range(world)]
    starts = [np.concatenate([[0], np.cumsum(c)]) for c in counts]
    # emulated all-to-all: rank q receives section q of every source, in source order
    y_parts = {}
    for qd in range(world):
        rx = torch.cat([send_x[r][starts[r][qd]:starts[r][qd + 1]] for r in range(world)])
        ri = torch.cat([plans[r]["send_ids"][starts[r][qd]:starts[r][qd + 1]] for r in range(world)])
        rw = torch.cat([plans[r]["send_w"][starts[r][qd]:starts[r][qd + 1]] for r in range(world)])
        yq = locs[qd].forward(rx, rw, ri)
        off = 0
        for r in range(world):
            nr = counts[r][qd]
            y_parts[(r, qd)] = yq[off:off + nr]
            off += nr
    for r in range(world):
        y_back = torch.cat([y_parts[(r, qd)] for qd in range(world)])
        y = M.ep_combine(y_back, plans[r]["token_rows"], T)
        ref = full.forward(xs[r], ws[r], idss[r])
        torch.cuda.synchronize()
        assert_close(y.float().cpu().numpy(), ref.float().cpu().numpy())
    for L in locs + [full]:
        L.check()


def _free_port():
    sk = socket.socket()
    sk.bind(("127.0.0.1", 0))
    p = sk.getsockname()[1]
    sk.close()
    return p


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_ep_nccl_two_ranks():
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(HERE, "ep_nccl_worker.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]


@pytest.mark.parametrize("dtype,H,I,T", [(O.DT_Q8_0, 256, 128, 5), (O.DT_FP8, 256, 256, 40)])
def test_none_slots_are_skipped(dtype, H, I, T):
    """An MOE_ID_NONE slot contributes nothing and raises no error: [ids | NONE] == ids."""
    rng = np.random.default_rng(3)
    E, k = 8, 2
    q, s, _ = quant_stacks(rng, E, H, I, dtype)
    layer = build(q, s, E, k, H, I, dtype, max_tokens=2 * T)  # room for width k + 1
    x = torch.from_numpy(O.f32_to_bf16(rng.normal(0, 1, (T, H)).astype(np.float32)).view(np.int16)).view(torch.bfloat16).cuda()
    ids = random_ids(rng, T, E, k)
    w = rng.dirichlet(np.ones(k), T).astype(np.float32)
    base = layer.forward(x, torch.from_numpy(w).cuda(), torch.from_numpy(ids.view(np.int32)).cuda())
    pid = np.concatenate([ids, np.full((T, 1), O.ID_NONE, np.uint32)], 1)
    pw = np.concatenate([w, rng.random((T, 1)).astype(np.float32)], 1)  # the weight of an empty slot is ignored
    padded = layer.forward(x, torch.from_numpy(pw).cuda(), torch.from_numpy(pid.view(np.int32)).cuda())
    torch.cuda.synchronize()
    layer.check()
    assert torch.equal(base, padded)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_ep_peer_two_ranks():
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(HERE, "ep_p2p_worker.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_ep_peer_failure_propagates():
    """Rank 1 drops its dispatch of one epoch (a host-side failure). Both ranks' bounded waits run out,
    the failure reaches both through the return flags (MOE_ERR_TIMEOUT on each, no returned row
    added), and the next epoch is bit-exact again."""
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           "--nproc-per-node=2", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           os.path.join(HERE, "ep_p2p_fail_worker.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, capture_output=True, text=True, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
