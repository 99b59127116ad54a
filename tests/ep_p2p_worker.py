"""Worker of tests/test_gpu_ep.py::test_ep_peer_two_ranks (torch.distributed.run, one process per GPU):
the NVLink peer-memory exchange (PeerExpertParallelMoE) against the NCCL one (ExpertParallelMoE),
bit for bit, and both against a full-expert layer within the north-star tolerance, over several
epochs with fresh inputs (region and flag reuse). The plan the one-launch routed dispatch writes
(rank_counts, token_rows) must equal the oracle's ep_dispatch_plan bit for bit. A last epoch has rank
1 send no token at all and rank 0 send tokens with an empty (MOE_ID_NONE) slot each. Exits non-zero
on a mismatch."""
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
from oracle import oracle as O  # noqa: E402


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", local))
    ok = True
    try:
        E_per, k, H, I, T = 8, 4, 256, 256, 96
        E = E_per * world
        rng = np.random.default_rng(5)
        q, s = [], []
        for shape in ((E, I, H), (E, I, H), (E, H, I)):
            qq, ss = O.quantize(O.DT_FP8, rng.normal(0, 0.02, shape).astype(np.float32))
            q.append(qq)
            s.append(ss)

        def build(qs, ss, n, max_tokens):
            cfg = M.MoeConfig(num_experts=n, num_experts_per_tok=k, hidden_size=H, moe_intermediate_size=I)
            return M.RoutedExpertsProvider().build(M.ExpertLoadContext(
                layer=0, device=local, config=cfg, wdtype=M.DTYPE_FP8_E4M3_B128, gate=qs[0], up=qs[1], down=qs[2],
                gate_scale=ss[0], up_scale=ss[1], down_scale=ss[2], max_tokens=max_tokens))

        def sl(arrs):
            return [np.ascontiguousarray(np.asarray(a).reshape(E, -1)[rank * E_per:(rank + 1) * E_per]).reshape(-1)
                    for a in arrs]

        full = build(q, s, E, T)
        nccl_ep = M.ExpertParallelMoE(build(sl(q), sl(s), E_per, T * world), rank, world, E_per)
        peer_ep = M.PeerExpertParallelMoE(build(sl(q), sl(s), E_per, T * world), rank, world, E_per, max_tokens=T)
        r2 = np.random.default_rng(100 + rank)
        for epoch in range(4):
            Tn = T - 13 * epoch  # ragged across epochs
            x = torch.from_numpy(O.f32_to_bf16(r2.normal(0, 1, (Tn, H)).astype(np.float32)).view(np.int16)) \
                .view(torch.bfloat16).cuda()
            ids = torch.from_numpy(np.stack([r2.permutation(E)[:k] for _ in range(Tn)]).astype(np.int32)).cuda()
            w = torch.from_numpy(r2.dirichlet(np.ones(k), Tn).astype(np.float32)).cuda()
            yp = peer_ep.forward(x, w, ids)
            yn = nccl_ep.forward(x, w, ids)
            ref = full.forward(x, w, ids)
            torch.cuda.synchronize()
            same = torch.equal(yp, yn)
            err = float((yp.float() - ref.float()).abs().max() / ref.float().abs().max())
            rc, tr, _, _, _ = O.ep_dispatch_plan(ids.cpu().numpy().view(np.uint32), w.cpu().numpy(), E_per, world)
            plan_ok = (np.array_equal(peer_ep.plan["rank_counts"].cpu().numpy(), rc)
                       and np.array_equal(peer_ep.plan["token_rows"][:Tn].cpu().numpy(), tr))
            print(f"rank {rank} epoch {epoch + 1}: peer == nccl {same}, plan == oracle {plan_ok}, "
                  f"rel err vs full {err:.2e}", flush=True)
            ok = ok and same and plan_ok and err < 1e-2
        # ragged extreme: rank 1 sends nothing; rank 0's tokens each carry one empty slot
        Tn = 17 if rank == 0 else 0
        x = torch.from_numpy(O.f32_to_bf16(r2.normal(0, 1, (Tn, H)).astype(np.float32)).view(np.int16)) \
            .view(torch.bfloat16).cuda()
        idn = np.array([r2.permutation(E)[:k] for _ in range(Tn)], dtype=np.int64).reshape(Tn, k)
        idn[:, 1] = O.ID_NONE
        ids = torch.from_numpy(idn.astype(np.uint32).view(np.int32)).cuda()
        w = torch.from_numpy(r2.dirichlet(np.ones(k), Tn).astype(np.float32).reshape(Tn, k)).cuda()
        yp = peer_ep.forward(x, w, ids)
        torch.cuda.synchronize()
        if Tn:
            ref = full.forward(x, w, ids)
            torch.cuda.synchronize()
            err = float((yp.float() - ref.float()).abs().max() / ref.float().abs().max())
            print(f"rank {rank} ragged epoch: rel err vs full {err:.2e}", flush=True)
            ok = ok and err < 1e-2
        else:
            print(f"rank {rank} ragged epoch: sent no token, output {tuple(yp.shape)}", flush=True)
            ok = ok and tuple(yp.shape) == (0, H)
        peer_ep.check()
        flag = torch.tensor([1 if ok else 0], device="cuda")
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        ok = int(flag.item()) == 1
        peer_ep.close()
    finally:
        dist.destroy_process_group()
    sys.exit(0 if ok else 1)


if __name__ == "__main__":
    main()
