"""Worker of tests/test_gpu_ep.py::test_ep_peer_failure_propagates (torch.distributed.run, one process
per GPU, two ranks): a dropped dispatch must surface on every rank, and the next epoch must be exact.

The failure is made on the host, never on the GPU: in epoch 2 rank 1 does not call
moe_ep_peer_dispatch (a message that is dropped), so no flag of rank 1's arrives anywhere. Both
ranks' receive waits run out after a short limit (moe_ep_peer_set_wait_limit), their return flags
carry the failed bit, and both combines add no returned row. The test checks, on each rank, that
moe_ep_peer_check reports MOE_ERR_TIMEOUT, that epoch 2's output is exactly zero (no y_add, no
returned row), and that epoch 3, on epoch 1's inputs, reproduces epoch 1's output bit for bit.
Epochs 4-6 repeat this through the one-launch routed dispatch (moe_ep_peer_dispatch_routed, whose
receive is inside it): epoch 4 must equal epoch 1 bit for bit, rank 1 drops its call in epoch 5, and
epoch 6 must equal epoch 4. Exits non-zero on any mismatch."""
import ctypes
import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, os.path.join(os.path.dirname(HERE), "naiwa-rs_b200"))

import moe_b200 as M  # noqa: E402
from moe_b200._lib import MOE_ERR_TIMEOUT, MOE_OK, check, lib  # noqa: E402
from oracle import oracle as O  # noqa: E402

WAIT_US = 500_000  # the receive and return waits run out after half a second


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", local))
    ok = True
    try:
        E_per, k, H, I, T = 4, 2, 128, 128, 24
        E = E_per * world
        rng = np.random.default_rng(11)
        q = [O.quantize(O.DT_Q8_0, rng.normal(0, 0.02, shape).astype(np.float32))[0]
             for shape in ((E, I, H), (E, I, H), (E, H, I))]
        mine = [np.ascontiguousarray(a.reshape(E, -1)[rank * E_per:(rank + 1) * E_per]).reshape(-1) for a in q]
        cfg = M.MoeConfig(num_experts=E_per, num_experts_per_tok=k, hidden_size=H, moe_intermediate_size=I)
        layer = M.RoutedExpertsProvider().build(M.ExpertLoadContext(
            layer=0, device=local, config=cfg, wdtype=M.DTYPE_Q8_0, gate=mine[0], up=mine[1], down=mine[2],
            max_tokens=T * world))
        peer = M.PeerExpertParallelMoE(layer, rank, world, E_per, max_tokens=T, wait_limit_us=WAIT_US)
        r2 = np.random.default_rng(200 + rank)
        x = torch.from_numpy(O.f32_to_bf16(r2.normal(0, 1, (T, H)).astype(np.float32)).view(np.int16)) \
            .view(torch.bfloat16).cuda()
        ids = torch.from_numpy(np.stack([r2.permutation(E)[:k] for _ in range(T)]).astype(np.int32)).cuda()
        w = torch.from_numpy(r2.dirichlet(np.ones(k), T).astype(np.float32)).cuda()
        stream = torch.cuda.current_stream()
        st = ctypes.c_void_p(stream.cuda_stream)
        L = lib()
        recv_rows = ctypes.c_void_p(peer.recv_rows)

        def epoch(e: int, send: bool):
            plan = M.ep_dispatch(ids, w, E_per, world)
            if send:
                check(L.moe_ep_peer_dispatch(peer._h, x.data_ptr(), T, plan["rank_counts"].data_ptr(),
                                             plan["send_token"].data_ptr(), plan["send_ids"].data_ptr(),
                                             plan["send_w"].data_ptr(), e, st))
            check(L.moe_ep_peer_receive(peer._h, e, peer.recv_ids.data_ptr(), peer.recv_w.data_ptr(), st))
            check(L.moe_forward(layer._h, recv_rows, world * T, peer.recv_ids.data_ptr(), peer.recv_w.data_ptr(), k,
                                peer.y_local.data_ptr(), st))
            check(L.moe_ep_peer_return(peer._h, peer.y_local.data_ptr(), e, st))
            y = torch.empty((T, H), dtype=torch.bfloat16, device=x.device)
            check(L.moe_ep_peer_combine(peer._h, e, T, plan["rank_counts"].data_ptr(), plan["token_rows"].data_ptr(),
                                        None, y.data_ptr(), st))
            return y

        R = ctypes.c_void_p(peer.region_ids), ctypes.c_void_p(peer.region_w)
        P = peer.plan

        def routed(e: int, send: bool):
            if send:
                check(L.moe_ep_peer_dispatch_routed(peer._h, x.data_ptr(), T, ids.data_ptr(), w.data_ptr(), E_per, e,
                                                    P["rank_counts"].data_ptr(), P["token_rows"].data_ptr(),
                                                    P["error_word"].data_ptr(), st))
            check(L.moe_forward(layer._h, recv_rows, world * T, R[0], R[1], k, peer.y_local.data_ptr(), st))
            check(L.moe_ep_peer_return(peer._h, peer.y_local.data_ptr(), e, st))
            y = torch.empty((T, H), dtype=torch.bfloat16, device=x.device)
            check(L.moe_ep_peer_combine(peer._h, e, T, P["rank_counts"].data_ptr(), P["token_rows"].data_ptr(),
                                        None, y.data_ptr(), st))
            return y

        def status():
            return L.moe_ep_peer_check(peer._h, st)

        y1 = epoch(1, True)
        s1 = status()
        dist.barrier()
        y2 = epoch(2, rank != 1)  # rank 1 drops its dispatch of epoch 2
        s2 = status()
        dist.barrier()
        y3 = epoch(3, True)
        s3 = status()
        dist.barrier()
        y4 = routed(4, True)
        s4 = status()
        dist.barrier()
        y5 = routed(5, rank != 1)  # rank 1 drops its routed dispatch of epoch 5
        s5 = status()
        dist.barrier()
        y6 = routed(6, True)
        s6 = status()
        torch.cuda.synchronize()
        zero2 = bool((y2.float() == 0).all())
        same3 = torch.equal(y1, y3)
        nonzero1 = bool((y1.float() != 0).any())
        print(f"rank {rank}: status {s1} {s2} {s3}; epoch-2 output all zero {zero2}; epoch 3 == epoch 1 {same3}",
              flush=True)
        zero5 = bool((y5.float() == 0).all())
        same4, same6 = torch.equal(y4, y1), torch.equal(y6, y4)
        print(f"rank {rank}: routed status {s4} {s5} {s6}; epoch-5 output all zero {zero5}; epoch 4 == epoch 1 "
              f"{same4}; epoch 6 == epoch 4 {same6}", flush=True)
        ok = (s1 == MOE_OK and s2 == MOE_ERR_TIMEOUT and s3 == MOE_OK and zero2 and same3 and nonzero1
              and s4 == MOE_OK and s5 == MOE_ERR_TIMEOUT and s6 == MOE_OK and zero5 and same4 and same6)
        layer.check()
        flag = torch.tensor([1 if ok else 0], device="cuda")
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        ok = int(flag.item()) == 1
        peer.close()
        layer.close()
    finally:
        dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
