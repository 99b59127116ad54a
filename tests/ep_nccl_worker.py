"""Worker of tests/test_gpu_ep.py::test_ep_nccl_two_ranks (launched by torch.distributed.run, one
process per GPU, NCCL): every rank builds the same seeded FP8 expert stacks, keeps its own slice as
the local layer, runs ExpertParallelMoE.forward on its own tokens and checks the result against a
full-expert layer on the same tokens. Exits non-zero on a mismatch."""
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
        loc = build(sl(q), sl(s), E_per, T * world)
        layer = M.ExpertParallelMoE(loc, rank, world, E_per)
        r2 = np.random.default_rng(100 + rank)
        x = torch.from_numpy(O.f32_to_bf16(r2.normal(0, 1, (T, H)).astype(np.float32)).view(np.int16)) \
            .view(torch.bfloat16).cuda()
        ids = torch.from_numpy(np.stack([r2.permutation(E)[:k] for _ in range(T)]).astype(np.int32)).cuda()
        w = torch.from_numpy(r2.dirichlet(np.ones(k), T).astype(np.float32)).cuda()
        for _ in range(3):
            y = layer.forward(x, w, ids)
        ref = full.forward(x, w, ids)
        torch.cuda.synchronize()
        err = float((y.float() - ref.float()).abs().max() / ref.float().abs().max())
        loc.check()
        ok = torch.tensor([1 if err < 1e-2 else 0], device="cuda")
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        print(f"rank {rank}: rel err {err:.2e}, counts {layer.last_counts}", flush=True)
        if int(ok.item()) != 1:
            sys.exit(1)
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
