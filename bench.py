#!/usr/bin/env python
"""MoE-layer tokens/s on B200 — BASELINE config 2 (Qwen3-30B-A3B-shaped decode layer, Q8_0).

Workload ("step"): a ragged decode sweep — batches of T = 1, 2, 4, ..., 256 tokens — each pushed
through a stack of 48 distinct MoE layers (hidden 2048, 128 experts, top-8 renormalised softmax,
moe_intermediate 768, SwiGLU, Q8_0 weights ~ N(0, 0.02), router ~ N(0, 0.02), activations
~ N(0, 1), seeded). Per (T, layer): router + top-k then the routed experts. The metric counts tokens
through one MoE layer: 511 tokens x 48 layers per step per GPU. The 48 layers hold 30.8 GB of
expert weights, far more than the 126 MB L2, so every layer reads its experts from HBM (no L2 flush
needed).

N = 1: every expert on the GPU; per (T, layer) moe_route + moe_forward. N > 1 (torchrun, one process
per GPU): expert parallel — each GPU holds 128/N experts of every layer and routes its own ragged
sweep over all 128; rows go to the GPUs owning their experts and outputs come back through the
library's NVLink peer-memory dispatch / return kernels (PeerExpertParallelMoE), per-GPU work fixed
("weak"); an in-run check compares one layer's output on rank 0 with the unsharded layer.

`value` is device time of CUDA-graph replays with inputs resident in HBM (max over ranks); `e2e` is
the same sweep through the public API (eager calls) with the activations copied in from pinned host
memory and the outputs copied back, inside the timed region. At N = 1 the line also carries
`prefill`: BASELINE config 3 (4096-token prompt, 48 Q4_K layers, Zipf(1.1) routing) in 512-token
chunks and as one grouped pass, with tensor and HBM fractions, and `cpu_baseline`.

--impl reference times the reference's CPU expert path (oracle/cpu_baseline.c: CPU router + the
two-pass fused Q8_0 decode, AVX2, all host threads) on the same step, bounded to about a minute.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "naiwa-rs_b200"))
sys.path.insert(0, ROOT)

E, K_TOP, H, I = 128, 8, 2048, 768
PLAN_SINGLE_MAX = 8 * 1024  # pairs the plan handles in one CTA (plan.cu)
RAGGED = [1, 2, 4, 8, 16, 32, 64, 128, 256]
BYTES_PER_EXPERT = 3 * I * H * 34 // 32  # 5,013,504 B of Q8_0 per expert (gate + up + down)
METRIC = "MoE-layer tokens/s per B200 (decode, Qwen3-30B-A3B-shaped Q8_0 layer, ragged batch 1-256)"


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi samples (200 ms) of SM clock and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def cpu_info():
    model = "unknown"
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                model = ln.split(":", 1)[1].strip()
                break
    except Exception:
        pass
    return model, os.cpu_count() or 1


# ---------------------------------------------------------------------------------------------
# reference arm: the CPU path of the reference, restated in the oracle
# ---------------------------------------------------------------------------------------------

REF_DISTINCT_LAYERS = 4  # host layers the reference arm cycles through (641 MB each, far above any LLC)
REF_BUDGET_S = 60.0      # the reference arm's timed region stops after the step that passes this


def decode_config(world: int, layers: int) -> dict:
    """The `config` of the decode line, identical in both arms at the same N and layer count."""
    epr = E // max(world, 1)
    return {"workload": "BASELINE config 2: Qwen3-30B-A3B-shaped MoE decode, E128 top-8 renorm-softmax H2048 I768 "
                        f"Q8_0; ragged batches T=1,2,4,...,256 per GPU through {layers} distinct layers",
            "layers": layers, "tokens_per_step_per_gpu": sum(RAGGED) * layers, "ragged_batches": list(RAGGED),
            "l2": "inputs larger than L2 (30.8 GB of expert weights over the GPUs, cycled per step)",
            "parallelism": (f"ep{world}: experts split {epr} per GPU per layer; every GPU routes its own batch over "
                            "all 128 experts; rows and outputs exchanged through NVLink peer memory (dispatch / "
                            "return kernels, no collective library call)" if world > 1
                            else "single GPU, all 128 experts per layer")}


def host_threads() -> int:
    return len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)


def reference_layers(n_distinct: int, seed: int = 2):
    """Host Q8_0 layers for the reference arm: layer 0 from seeded N(0, 0.02) weights, layers 1.. its
    experts rotated into fresh memory (the same work, no cache reuse between layers); one f32 router
    per layer."""
    import numpy as np

    from oracle import oracle as O

    rng = np.random.Generator(np.random.Philox(seed))
    q0 = []
    for shape in ((E, I, H), (E, I, H), (E, H, I)):
        w = rng.standard_normal(shape, dtype=np.float32)
        w *= np.float32(0.02)
        q0.append(O.quantize(O.DT_Q8_0, w)[0])
        del w
    layers = [q0] + [[np.roll(q.reshape(E, -1), 37 * li, axis=0).reshape(-1).copy() for q in q0]
                     for li in range(1, n_distinct)]
    routers = [O.bf16_to_f32(O.f32_to_bf16(rng.standard_normal((E, H), dtype=np.float32) * np.float32(0.02)))
               .reshape(E, H) for _ in range(n_distinct)]
    return layers, routers


def reference_sweep(layers, routers, xs, threads, layer_calls):
    """One ragged sweep: each batch through `layer_calls` layer calls (cycling the given layers), each a
    CPU router (f32 logits, renormalised softmax top-8) and the two-pass fused Q8_0 decode."""
    import numpy as np

    from oracle import oracle as O

    tokens = 0
    for T in RAGGED:
        x = xs[T]
        for li in range(layer_calls):
            q, wr = layers[li % len(layers)], routers[li % len(routers)]
            logits = np.ascontiguousarray(x @ wr.T, dtype=np.float32)
            ids, w = O.route(logits, K_TOP, 1)
            O.baseline_decode_q8_0(q[0], q[1], q[2], x, ids, w, E, H, I, threads)
        tokens += T * layer_calls
    return tokens


def reference_inputs(seed: int):
    import numpy as np

    from oracle import oracle as O

    rng = np.random.Generator(np.random.Philox(seed))
    return {T: O.bf16_to_f32(O.f32_to_bf16(rng.standard_normal((T, H), dtype=np.float32))).reshape(T, H)
            for T in RAGGED}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    model, _ = cpu_info()
    ncpu = host_threads()
    layers, routers = reference_layers(REF_DISTINCT_LAYERS)
    xs = reference_inputs(7)
    # one untimed step starts the thread pool and touches every page; the timed steps stop at K or
    # once REF_BUDGET_S have passed (at least one), so the arm ends within a few minutes at any K
    warm = min(args.warmup, 1)
    for _ in range(warm):
        reference_sweep(layers, routers, xs, ncpu, args.layers)
    t0 = time.perf_counter()
    tokens = steps = 0
    while steps < args.steps and (steps == 0 or time.perf_counter() - t0 < REF_BUDGET_S):
        tokens += reference_sweep(layers, routers, xs, ncpu, args.layers)
        steps += 1
    dt = time.perf_counter() - t0
    value = tokens / dt
    sample = (f"the whole step: ragged sweep T=1..256 (511 tokens) through {args.layers} layer calls per batch, "
              f"cycling {REF_DISTINCT_LAYERS} distinct host Q8_0 layers (641 MB each); per call a CPU router (f32 "
              f"logits, renormalised top-8) and the reference's two-pass fused Q8_0 decode restated with AVX2 "
              f"(oracle/cpu_baseline.c); {ncpu} threads on {model}; {steps} timed steps (at most {args.steps}, "
              f"stopping after {REF_BUDGET_S:.0f} s)")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": steps, "warmup": warm, "ms_per_step": dt / steps * 1e3,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "q8_0 weights, f32 compute",
        "data": "synthetic: seeded N(0,0.02) Q8_0 experts and router, N(0,1) activations rounded to bf16",
        "config": decode_config(world, args.layers),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": ncpu, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


# ---------------------------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------------------------

def cpu_baseline_from_layer(stacks_host, router_host, budget_s=12.0):
    """The reference's CPU path (CPU router + two-pass fused decode, oracle/cpu_baseline.c) over layer
    0's own bytes on all host threads: repeated ragged sweeps until ~budget_s of CPU work."""
    from oracle import oracle as O

    model, _ = cpu_info()
    ncpu = host_threads()
    xs = reference_inputs(7)
    router = O.bf16_to_f32(router_host).reshape(E, H)
    reference_sweep([stacks_host], [router], xs, ncpu, 1)  # warm
    t0 = time.perf_counter()
    tokens = sweeps = 0
    while time.perf_counter() - t0 < budget_s or sweeps == 0:
        tokens += reference_sweep([stacks_host], [router], xs, ncpu, 1)
        sweeps += 1
    dt = time.perf_counter() - t0
    return {"value": tokens / dt, "unit": "tokens/s", "cores": ncpu, "kind": "port",
            "sample": f"{sweeps} ragged sweeps (T=1..256) through layer 0 of the same stack; CPU router + the "
                      f"reference's two-pass fused Q8_0 decode restated with AVX2 (oracle/cpu_baseline.c); "
                      f"{ncpu} threads on {model}"}


def _uses_gemm(live_pairs, E_local, sms=148):
    """The layer's Q8_0 path choice (layer.cu, q8_uses_gemm): the tcgen05 GEMM from 4 live tokens per
    expert when its gate/up items (E x 2I/128) fill two CTAs per SM, else from 16."""
    fills = E_local * (2 * I // 128) >= 2 * sms
    return live_pairs >= (4 if fills else 16) * E_local


def _launches_local(pairs, E_local, live_pairs=None):
    """Kernel launches of one moe_forward over `pairs` routed pairs (`live_pairs` of them live): plan
    (one CTA up to 8 K pairs, else histogram / scan / scatter), the decode GEMV pair or the tcgen05
    path (tile list, token gather, gate/up GEMM, h gather, down GEMM), combine."""
    plan = 1 if pairs <= PLAN_SINGLE_MAX else 3
    experts = 5 if _uses_gemm(pairs if live_pairs is None else live_pairs, E_local) else 2
    return plan + experts + 1


def run_ours(args):
    import ctypes

    import numpy as np
    import torch

    import moe_b200 as M
    from moe_b200 import synth

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    if E % world:
        raise SystemExit(f"--gpus {world}: the {E} experts of a layer do not split evenly")
    ep = world > 1
    epr = E // world
    L = args.layers
    TMAX = max(RAGGED)
    provider = M.RoutedExpertsProvider()
    layers, routers = [], []
    host_layer0 = None
    full0 = None  # rank 0 at N > 1: layer 0 with every expert, for the in-run parity check
    for li in range(L):
        g, u, d = synth.expert_stacks(E, H, I, M.DTYPE_Q8_0, 0.02, seed=1000 + li, device=dev)
        router = synth.router_weight(E, H, 0.02, seed=5000 + li, device=dev)
        if ep:
            # this rank's experts [rank * epr, (rank + 1) * epr): whole experts are contiguous byte
            # ranges of a GGML stack (expert.rs:123-145)
            mine = [t.view(E, -1)[rank * epr:(rank + 1) * epr].reshape(-1) for t in (g, u, d)]
            cfg = M.MoeConfig(num_experts=epr, num_experts_per_tok=K_TOP, hidden_size=H, moe_intermediate_size=I)
            layers.append(provider.build(M.ExpertLoadContext(
                layer=li, device=local, config=cfg, wdtype=M.DTYPE_Q8_0, gate=mine[0], up=mine[1], down=mine[2],
                max_tokens=world * TMAX)))
            routers.append(M.Router(router, K_TOP, M.ROUTER_SOFTMAX_RENORM, max_tokens=TMAX))
            if li == 0 and rank == 0:
                cfg0 = M.MoeConfig(num_experts=E, num_experts_per_tok=K_TOP, hidden_size=H, moe_intermediate_size=I)
                full0 = M.RoutedExpertsProvider().build(M.ExpertLoadContext(
                    layer=0, device=local, config=cfg0, wdtype=M.DTYPE_Q8_0, gate=g, up=u, down=d, max_tokens=TMAX))
            del mine
        else:
            cfg = M.MoeConfig(num_experts=E, num_experts_per_tok=K_TOP, hidden_size=H, moe_intermediate_size=I,
                              router_mode=M.ROUTER_SOFTMAX_RENORM)
            layers.append(provider.build(M.ExpertLoadContext(
                layer=li, device=local, config=cfg, wdtype=M.DTYPE_Q8_0, gate=g, up=u, down=d, router_weight=router,
                max_tokens=TMAX)))
            if li == 0 and not args.no_cpu_baseline:
                host_layer0 = ([t.cpu().numpy() for t in (g, u, d)],
                               router.view(torch.int16).cpu().numpy().view(np.uint16))
        del g, u, d, router
    torch.cuda.empty_cache()

    gen = torch.Generator(device=dev)
    gen.manual_seed(77 + rank)
    xs = {T: torch.randn((T, H), generator=gen, device=dev).to(torch.bfloat16) for T in RAGGED}
    ids = {T: torch.empty((T, K_TOP), dtype=torch.int32, device=dev) for T in RAGGED}
    wts = {T: torch.empty((T, K_TOP), dtype=torch.float32, device=dev) for T in RAGGED}
    ys = {T: torch.empty((T, H), dtype=torch.bfloat16, device=dev) for T in RAGGED}
    # one peer-memory exchange per batch size (its regions hold world * T rows), shared by the layers
    peers = {T: M.PeerExpertParallelMoE(layers[0], rank, world, epr, max_tokens=T) for T in RAGGED} if ep else {}
    for layer in layers if ep else []:  # every local layer runs world * T received rows, ~1/world of them live
        layer.set_live_hint(1.0 / world)

    def call(T, li, xin, yout, marks=None):
        if ep:
            routers[li].route(xin, out_ids=ids[T], out_weights=wts[T])
            peers[T].forward(xin, wts[T], ids[T], out=yout, layer=layers[li], marks=marks)
        else:
            layers[li].route(xin, out_ids=ids[T], out_weights=wts[T])
            layers[li].forward(xin, wts[T], ids[T], out=yout)

    def sweep():
        for T in RAGGED:
            for li in range(L):
                call(T, li, xs[T], ys[T])

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(v):
        if dist is None:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    stream = torch.cuda.Stream(device=dev)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        for _ in range(max(1, args.warmup)):
            sweep()
    torch.cuda.synchronize()
    for layer in layers:
        layer.check()
    for p in peers.values():
        p.check()
    barrier()

    # one CUDA graph per step: 9 batch sizes x L layers of (route + forward) [+ the exchange at N > 1]
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        sweep()
    torch.cuda.synchronize()
    barrier()
    with torch.cuda.stream(stream):  # replays run on the current stream
        for _ in range(args.warmup):
            graph.replay()
    torch.cuda.synchronize()
    barrier()

    tokens_per_step = sum(RAGGED) * L  # per rank
    with ClockSampler(local) as clk:
        barrier()
        torch.cuda.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            ev0.record(stream)
            for _ in range(args.steps):
                graph.replay()
            ev1.record(stream)
        torch.cuda.synchronize()
        barrier()
        ms = max_over_ranks(ev0.elapsed_time(ev1) / args.steps)
    value = tokens_per_step * world / (ms / 1e3)
    for p in peers.values():
        p.check()

    # ---- algorithmic bytes: the distinct experts each rank reads, from this step's routing -----------
    # (at N > 1 a rank reads its own experts that any rank's tokens chose)
    local_distinct = {T: 0 for T in RAGGED}
    with torch.cuda.stream(stream):
        for T in RAGGED:
            for li in range(L):
                if ep:
                    routers[li].route(xs[T], out_ids=ids[T], out_weights=wts[T])
                    allids = torch.empty((world,) + tuple(ids[T].shape), dtype=torch.int32, device=dev)
                    dist.all_gather_into_tensor(allids, ids[T])
                    u = torch.unique(allids)
                    local_distinct[T] += int(((u >= rank * epr) & (u < (rank + 1) * epr)).sum().item())
                else:
                    layers[li].route(xs[T], out_ids=ids[T], out_weights=wts[T])
                    local_distinct[T] += int(torch.unique(ids[T]).numel())
    torch.cuda.synchronize()
    weight_bytes = {T: local_distinct[T] * BYTES_PER_EXPERT for T in RAGGED}
    # DRAM bytes (read + write) over algorithmic weight bytes in one ncu --set full capture of each
    # path on this workload: the GEMV at T = 32 (372.1 / 367.7 MB gate/up, 189.4 / 183.8 MB down) and
    # the tcgen05 GEMM at T = 256 (441.2 / 427.8 MB gate/up, 222.7 / 213.9 MB down)
    gemv_ratio, gemm_ratio = (372.1 + 189.4) / (367.7 + 183.8), (441.2 + 222.7) / (427.8 + 213.9)
    traffic_per_step = sum(weight_bytes[T] * (gemm_ratio if _uses_gemm(T * K_TOP, E // world) else gemv_ratio)
                           for T in RAGGED)

    # ---- stage timing: one captured step with events between the stages ---------------------------
    lib = M.lib()
    if ep:  # route | routed dispatch (plan, rows out, receive) | local forward | return | combine
        names = ["route", "dispatch_receive", "local_forward", "return", "combine"]
    else:   # route | plan | gate/up | down | combine
        names = ["route", "plan", "gate_up", "down", "combine"]
    nev = len(RAGGED) * L
    evs = [[torch.cuda.Event(enable_timing=True, external=True) for _ in range(len(names) + 1)] for _ in range(nev)]
    ev_arrays = []
    for row in evs:
        for e_ in row:
            e_.record(stream)
        if not ep:  # moe_forward_marked records the five events after the route
            ev_arrays.append((ctypes.c_void_p * 5)(*[e_.cuda_event for e_ in row[1:]]))
    torch.cuda.synchronize()

    def marked_sweep():
        i = 0
        for T in RAGGED:
            for li in range(L):
                row = evs[i]
                row[0].record(stream)
                if ep:
                    routers[li].route(xs[T], out_ids=ids[T], out_weights=wts[T])
                    row[1].record(stream)
                    peers[T].forward(xs[T], wts[T], ids[T], out=ys[T], layer=layers[li], marks=row[2:])
                else:
                    layers[li].route(xs[T], out_ids=ids[T], out_weights=wts[T])
                    st = ctypes.c_void_p(stream.cuda_stream)
                    M._lib.check(lib.moe_forward_marked(layers[li]._h, xs[T].data_ptr(), T, ids[T].data_ptr(),
                                                        wts[T].data_ptr(), K_TOP, ys[T].data_ptr(), st,
                                                        ev_arrays[i]))
                i += 1

    mgraph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(mgraph, stream=stream):
        marked_sweep()
    torch.cuda.synchronize()
    barrier()
    with torch.cuda.stream(stream):
        mgraph.replay()
    torch.cuda.synchronize()
    barrier()
    stage = {n: 0.0 for n in names}
    per_T_expert_ms = {T: 0.0 for T in RAGGED}
    expert_stage = ["local_forward"] if ep else ["gate_up", "down"]
    i = 0
    for T in RAGGED:
        for _ in range(L):
            row = evs[i]
            for j, n in enumerate(names):
                d = row[j].elapsed_time(row[j + 1])
                stage[n] += d
                if n in expert_stage:
                    per_T_expert_ms[T] += d
            i += 1
    stage_max = {n: max_over_ranks(v) for n, v in stage.items()}
    expert_ms = sum(stage[n] for n in expert_stage)
    total_w_bytes = sum(weight_bytes.values())
    hbm_peak, peak_kind = peaks()
    achieved = total_w_bytes / (expert_ms / 1e3) / 1e9
    per_batch = {}
    for T in RAGGED:
        gbs = weight_bytes[T] / (per_T_expert_ms[T] / 1e3) / 1e9
        per_batch[str(T)] = {"expert_gbs": round(gbs, 1), "frac": round(gbs / hbm_peak, 3),
                             "distinct_experts_per_layer": round(local_distinct[T] / L, 2),
                             "expert_ms_per_layer": round(per_T_expert_ms[T] / L, 4)}
    step_frac = total_w_bytes / (ms / 1e3) / 1e9 / hbm_peak

    # ---- in-run parity (N > 1): one layer through the exchange against the unsharded layer -----------
    parity = None
    if ep:
        Tc = 32
        with torch.cuda.stream(stream):
            routers[0].route(xs[Tc], out_ids=ids[Tc], out_weights=wts[Tc])
            y_ep = peers[Tc].forward(xs[Tc], wts[Tc], ids[Tc], layer=layers[0])
            if full0 is not None:
                y_full = full0.forward(xs[Tc], wts[Tc], ids[Tc])
        torch.cuda.synchronize()
        if full0 is not None:
            a, b = y_ep.double(), y_full.double()
            err = float((a - b).abs().max() / b.abs().max())
            parity = {"layer": 0, "tokens": Tc, "rank": 0, "max_rel_err_vs_unsharded": err, "ok": err <= 1e-2}
        barrier()

    # ---- e2e: public API, activations from pinned host memory, outputs back to the host -----------
    hx = {T: xs[T].cpu().pin_memory() for T in RAGGED}
    hy = {T: torch.empty((T, H), dtype=torch.bfloat16).pin_memory() for T in RAGGED}
    dx = {T: torch.empty_like(xs[T]) for T in RAGGED}
    h2d = sum(T * H * 2 for T in RAGGED)
    d2h = h2d

    def e2e_step():
        for T in RAGGED:
            dx[T].copy_(hx[T], non_blocking=True)
            for li in range(L):
                call(T, li, dx[T], ys[T])
            hy[T].copy_(ys[T], non_blocking=True)

    with torch.cuda.stream(stream):
        e2e_step()
        torch.cuda.synchronize()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            e2e_step()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    e2e_value = tokens_per_step * world / (e2e_ms / 1e3)

    for layer in layers:
        layer.check()
    for p in peers.values():
        p.check()
    del graph, mgraph

    # launches per step of this rank: route, then (N > 1) the routed dispatch, the local forward on
    # world * T rows, return, combine
    def launches_for(T):
        if ep:
            return 1 + 1 + _launches_local(world * T * K_TOP, epr, T * K_TOP) + 2
        return 1 + _launches_local(T * K_TOP, E)
    launches_per_step = L * sum(launches_for(T) for T in RAGGED)

    out = None
    if rank == 0:
        out = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "q8_0 weights, f16 tensor-core MMA, f32 accumulate",
            "data": "synthetic: seeded N(0,0.02) Q8_0 experts and router, N(0,1) bf16 activations",
            "config": decode_config(world, args.layers),
            "roofline": {"kernel": ("expert FFN on this GPU's experts" + (" (rank 0)" if ep else "") +
                                    ": decode GEMV below 4 tokens per expert, tcgen05 GEMM at or above (gate/up+"
                                    "SwiGLU and down*weight, Q8_0 units)"),
                         "bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(achieved / hbm_peak, 4), "peak_source": peak_kind,
                         "frac_over_whole_step": round(step_frac, 4),
                         "traffic": round(traffic_per_step),
                         "traffic_unit": "DRAM bytes per step, the step's algorithmic bytes scaled by the "
                                         "DRAM/algorithmic ratio of each path's ncu capture (profiles/)",
                         "algorithmic_bytes": "5,013,504 B per distinct expert per layer read by this GPU "
                                              "(Q8_0 gate+up+down)"},
            "stage_ms_per_step": {n: round(v, 3) for n, v in stage.items()},
            "stage_ms_per_step_max_over_ranks": {n: round(v, 3) for n, v in stage_max.items()} if ep else None,
            "per_batch": per_batch,
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": h2d * world,
                    "d2h_bytes_per_step": d2h * world},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk.summary(),
            "ep_parity": parity,
        }
    for p in peers.values():
        p.close()
    for layer in layers:
        layer.close()
    if full0 is not None:
        full0.close()
    del layers
    torch.cuda.empty_cache()
    if rank == 0 and not ep:
        if not args.no_prefill:
            out["prefill"] = prefill_record(args, local)
        if host_layer0 is not None:
            out["cpu_baseline"] = cpu_baseline_from_layer(host_layer0[0], host_layer0[1], budget_s=args.cpu_seconds)
    if rank == 0:
        out.setdefault("cpu_baseline", None)
        print(json.dumps(out), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------------------------------------
# prefill: Q4_K layers, 4096-token prompt in 512-token chunks or in one pass
# ---------------------------------------------------------------------------------------------

Q4K_BYTES_PER_EXPERT = 3 * I * H // 256 * 144  # 2,654,208 B
PROMPT = 4096


def _prefill_pass(M, layers, xs, ids, wts, ys, chunk, steps, warmup, stream, local):
    """Times `steps` CUDA-graph replays of the prompt through every layer in `chunk`-token passes;
    returns (device ms per step, gate/up ms, down ms, e2e ms, clocks)."""
    import ctypes

    import torch

    L = len(layers)
    nch = len(xs)

    def step():
        for layer in layers:
            for c in range(nch):
                layer.forward(xs[c], wts[c], ids[c], out=ys[c])

    with torch.cuda.stream(stream):
        for _ in range(max(1, warmup)):
            step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    with torch.cuda.stream(stream), ClockSampler(local) as clk:
        for _ in range(warmup):
            graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    del graph
    # end to end through the public API with host buffers: every layer-chunk copies its pinned
    # activations, routing ids and weights in and its output back, inside the timed region
    hx = [x.cpu().pin_memory() for x in xs]
    hid = [t.cpu().pin_memory() for t in ids]
    hw = [t.cpu().pin_memory() for t in wts]
    hy = [torch.empty_like(x, device="cpu").pin_memory() for x in xs]
    dx, did, dw, dy = (torch.empty_like(xs[0]), torch.empty_like(ids[0]), torch.empty_like(wts[0]),
                       torch.empty_like(xs[0]))

    def e2e_step():
        for layer in layers:
            for c in range(nch):
                dx.copy_(hx[c], non_blocking=True)
                did.copy_(hid[c], non_blocking=True)
                dw.copy_(hw[c], non_blocking=True)
                layer.forward(dx, dw, did, out=dy)
                hy[c].copy_(dy, non_blocking=True)

    with torch.cuda.stream(stream):
        e2e_step()
        torch.cuda.synchronize()
        f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        for _ in range(steps):
            e2e_step()
        f1.record(stream)
        torch.cuda.synchronize()
    e2e_ms = f0.elapsed_time(f1) / steps
    # stage-marked pass (one captured step): gate/up and down kernel times
    evs = [[torch.cuda.Event(enable_timing=True, external=True) for _ in range(5)] for _ in range(L * nch)]
    arrs = []
    for row in evs:
        for ev in row:
            ev.record(stream)
        arrs.append((ctypes.c_void_p * 5)(*[ev.cuda_event for ev in row]))
    torch.cuda.synchronize()
    lib = M.lib()

    def marked():
        i = 0
        for layer in layers:
            for c in range(nch):
                M._lib.check(lib.moe_forward_marked(layer._h, xs[c].data_ptr(), xs[c].shape[0], ids[c].data_ptr(),
                                                    wts[c].data_ptr(), K_TOP, ys[c].data_ptr(),
                                                    ctypes.c_void_p(stream.cuda_stream), arrs[i]))
                i += 1

    mg = torch.cuda.CUDAGraph()
    with torch.cuda.graph(mg, stream=stream):
        marked()
    with torch.cuda.stream(stream):
        mg.replay()
    torch.cuda.synchronize()
    gu = sum(r[1].elapsed_time(r[2]) for r in evs)
    dn = sum(r[2].elapsed_time(r[3]) for r in evs)
    del mg
    return ms, gu, dn, e2e_ms, clk.summary()


def prefill_record(args, local):
    """BASELINE config 3 on one GPU: the 4096-token prompt through `args.layers` distinct Q4_K layers,
    in 512-token chunks (the configured workload) and as one grouped pass per layer (the 4096-token
    one-pass variant the tensor-core target is stated on). Returns the nested `prefill` record."""
    import torch

    import moe_b200 as M
    from moe_b200 import synth

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    L = args.layers
    cfg = M.MoeConfig(num_experts=E, num_experts_per_tok=K_TOP, hidden_size=H, moe_intermediate_size=I)
    prov = M.RoutedExpertsProvider()
    layers = []
    for li in range(L):
        g, u, d = synth.expert_stacks(E, H, I, M.DTYPE_Q4_K, 0.02, seed=2000 + li, device=dev)
        layers.append(prov.build(M.ExpertLoadContext(layer=li, device=local, config=cfg, wdtype=M.DTYPE_Q4_K,
                                                     gate=g, up=u, down=d, max_tokens=args.chunk)))
        del g, u, d
    torch.cuda.empty_cache()
    gen = torch.Generator(device=dev)
    gen.manual_seed(33)
    zipf = 1.0 / torch.arange(1, E + 1, device=dev, dtype=torch.float32) ** 1.1
    x_all = torch.randn((PROMPT, H), generator=gen, device=dev).to(torch.bfloat16)
    id_all = torch.multinomial(zipf.expand(PROMPT, E), K_TOP, replacement=False, generator=gen).to(torch.int32)
    w_all = torch.softmax(torch.randn((PROMPT, K_TOP), generator=gen, device=dev), -1)
    try:
        peaks_j = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        tpeak, tsus, hpeak, kind = (float(peaks_j["bf16_tflops"]), float(peaks_j["bf16_tflops_sustained"]),
                                    float(peaks_j["hbm_gbs"]), "measured")
    except Exception:
        tpeak, tsus, hpeak, kind = 1590.0, 1400.0, 6650.0, "fallback"
    stream = torch.cuda.Stream(device=dev)
    rec = {}
    for name, chunk in (("chunked", args.chunk), ("one_pass", PROMPT)):
        if chunk > args.chunk:
            for layer in layers:
                layer.warmup(chunk)
        nch = PROMPT // chunk
        xs = [x_all[c * chunk:(c + 1) * chunk] for c in range(nch)]
        ids = [id_all[c * chunk:(c + 1) * chunk] for c in range(nch)]
        wts = [w_all[c * chunk:(c + 1) * chunk] for c in range(nch)]
        ys = [torch.empty_like(x) for x in xs]
        steps = max(3, args.steps // 2)
        ms, gu, dn, e2e_ms, clocks = _prefill_pass(M, layers, xs, ids, wts, ys, chunk, steps, args.warmup, stream,
                                                   local)
        flops = 2.0 * 3 * H * I * PROMPT * K_TOP * L
        distinct = sum(int(torch.unique(t).numel()) for t in ids) * L
        wbytes = distinct * Q4K_BYTES_PER_EXPERT
        tflops = flops / ((gu + dn) / 1e3) / 1e12
        gbs = wbytes / ((gu + dn) / 1e3) / 1e9
        h2d = L * nch * (chunk * H * 2 + chunk * K_TOP * 8)
        rec[name] = {
            "workload": (f"{PROMPT}-token prompt in {chunk}-token chunks" if chunk < PROMPT else
                         f"the {PROMPT}-token prompt as one grouped pass per layer") +
                        f" through {L} distinct Q4_K layers (E128 k8 H2048 I768), Zipf(1.1) routing",
            "value": PROMPT * L / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms, "steps": steps,
            "tensor": {"kernel": "expert_gemm_tc gate/up + down (tcgen05)", "achieved_tflops": round(tflops, 1),
                       "peak_tflops": tsus, "peak_source": f"bf16_tflops_sustained ({kind})",
                       "frac": round(tflops / tsus, 4), "frac_of_burst": round(tflops / tpeak, 4)},
            "hbm": {"achieved_gbs": round(gbs, 1), "peak_gbs": hpeak, "frac": round(gbs / hpeak, 4),
                    "algorithmic_bytes": f"{Q4K_BYTES_PER_EXPERT} B per distinct expert per layer-chunk"},
            "whole_step_tflops": round(flops / (ms / 1e3) / 1e12, 1),
            "stage_ms_per_step": {"gate_up": round(gu, 3), "down": round(dn, 3)},
            "e2e": {"value": PROMPT * L / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": L * nch * chunk * H * 2},
            "gpu_launches": 7 * L * nch * steps,
            "clocks": clocks,
        }
    for layer in layers:
        layer.check()
        layer.close()
    torch.cuda.empty_cache()
    return rec


def run_prefill(args):
    """--workload prefill: the prefill record alone, as its own line."""
    local = int(os.environ.get("LOCAL_RANK", "0"))
    rec = prefill_record(args, local)
    c = rec["chunked"]
    print(json.dumps({
        "metric": f"MoE-layer tokens/s per B200 (prefill, Qwen3-30B-A3B-shaped Q4_K layer, {args.chunk}-token chunks)",
        "value": c["value"], "unit": "tokens/s", "n_gpus": 1, "steps": c["steps"], "warmup": args.warmup,
        "ms_per_step": c["ms_per_step"], "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "q4_k weights dequantised to f16 in tensor memory, tcgen05 f16 MMA, f32 accumulate",
        "data": "synthetic: seeded N(0,0.02) Q4_K experts, N(0,1) bf16 activations, Zipf(1.1) routing",
        "config": {"workload": "BASELINE config 3: " + c["workload"], "layers": args.layers,
                   "l2": "inputs larger than L2 (340 MB of Q4_K experts per layer)"},
        "roofline": {"kernel": c["tensor"]["kernel"], "bound": "tensor", "achieved": c["tensor"]["achieved_tflops"],
                     "peak": c["tensor"]["peak_tflops"], "unit": "TFLOP/s", "frac": c["tensor"]["frac"],
                     "peak_source": c["tensor"]["peak_source"], "traffic": None},
        "e2e": c["e2e"], "gpu_launches": c["gpu_launches"], "clocks": c["clocks"], "one_pass": rec["one_pass"],
    }), flush=True)


# ---- expert-parallel workload: FP8 E256 top-8 group-limited, experts sharded by rank

EP_E, EP_K, EP_H, EP_I, EP_T = 256, 8, 7168, 2048, 8192
EP_FLOPS_PER_STEP = (EP_T * EP_K + EP_T) * 2 * (3 * EP_H * EP_I)  # routed pairs + one shared expert per token


def run_ep(args):
    import datetime

    import torch
    import torch.distributed as dist

    import moe_b200 as M
    from moe_b200 import synth

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    assert EP_E % world == 0 and EP_T % world == 0
    epr, T = EP_E // world, EP_T // world
    prov = M.RoutedExpertsProvider()
    (g, u, d), (gs, us, ds) = synth.expert_stacks(epr, EP_H, EP_I, M.DTYPE_FP8_E4M3_B128, 0.02, seed=5000 + rank,
                                                  device=dev, with_scales=True)
    cfg = M.MoeConfig(num_experts=epr, num_experts_per_tok=EP_K, hidden_size=EP_H, moe_intermediate_size=EP_I)
    local_layer = prov.build(M.ExpertLoadContext(layer=0, device=local, config=cfg, wdtype=M.DTYPE_FP8_E4M3_B128,
                                                 gate=g, up=u, down=d, gate_scale=gs, up_scale=us, down_scale=ds,
                                                 max_tokens=T * world))
    del g, u, d, gs, us, ds
    (g, u, d), (gs, us, ds) = synth.expert_stacks(1, EP_H, EP_I, M.DTYPE_FP8_E4M3_B128, 0.02, seed=4999, device=dev,
                                                  with_scales=True)
    scfg = M.MoeConfig(num_experts=1, num_experts_per_tok=1, hidden_size=EP_H, moe_intermediate_size=EP_I)
    shared = prov.build(M.ExpertLoadContext(layer=0, device=local, config=scfg, wdtype=M.DTYPE_FP8_E4M3_B128,
                                            gate=g, up=u, down=d, gate_scale=gs, up_scale=us, down_scale=ds,
                                            max_tokens=T))
    del g, u, d, gs, us, ds
    torch.cuda.empty_cache()
    w_router = synth.router_weight(EP_E, EP_H, 0.02, seed=77, device=dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(900 + rank)
    bias = (torch.randn(EP_E, generator=gen, device=dev) * 0.01).float()
    x = torch.randn((T, EP_H), generator=gen, device=dev).to(torch.bfloat16)
    if world > 1 and args.ep_transport == "p2p":
        layer = M.PeerExpertParallelMoE(local_layer, rank, world, epr, max_tokens=T, shared=shared)
    else:
        layer = M.ExpertParallelMoE(local_layer, rank, world, epr, shared=shared)

    def step(xin):
        ids, w = M.route_tokens(xin, w_router, EP_K, M.ROUTER_SIGMOID_GROUP, bias=bias, n_group=8, topk_group=4,
                                routed_scale=2.5)
        return layer.forward(xin, w, ids)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v):
        if world > 1:
            t = torch.tensor([v], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            return float(t.item())
        return v

    for _ in range(max(3, args.warmup)):
        step(x)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            step(x)
        e1.record()
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    rows_out = None
    if getattr(layer, "last_counts", None):
        send_counts, recv_counts = layer.last_counts
        rows_out = sum(send_counts) - send_counts[rank]
    # end to end: this rank's activations copied in from pinned host memory and the output read back
    hx = x.cpu().pin_memory()
    hy = torch.empty_like(hx).pin_memory()
    dx = torch.empty_like(x)
    for _ in range(2):
        dx.copy_(hx, non_blocking=True)
        hy.copy_(step(dx), non_blocking=True)
    torch.cuda.synchronize()
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    for _ in range(args.steps):
        dx.copy_(hx, non_blocking=True)
        hy.copy_(step(dx), non_blocking=True)
    f1.record()
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(f0.elapsed_time(f1) / args.steps)
    if hasattr(layer, "check"):
        layer.check()
    local_layer.check()
    shared.check()
    try:
        peaks_j = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        tpeak, kind = float(peaks_j["bf16_tflops"]), "measured"
    except Exception:
        tpeak, kind = 1590.0, "fallback"
    tflops = EP_FLOPS_PER_STEP / (ms / 1e3) / 1e12
    if rank == 0:
        print(json.dumps({
            "metric": "MoE-layer tokens/s (expert parallel, DeepSeek-V3-shaped FP8 layer, 8192 tokens per step)",
            "value": EP_T / (ms / 1e3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": max(3, args.warmup), "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None,
            "dtype": "fp8 e4m3 (128x128 block scales) weights dequantised to f16 in tensor memory, tcgen05 f16 MMA",
            "data": "synthetic: seeded N(0,0.02) FP8 experts and router, N(0,1) bf16 activations",
            "config": {"workload": "BASELINE config 5: E256 (+1 shared) top-8 sigmoid group-limited (8 groups, "
                                   "top-4), H7168 I2048 FP8; 8192 tokens per step split over the ranks",
                       "experts_per_rank": epr, "tokens_per_rank": T, "parallelism": f"ep{world}",
                       "exchange": ("NVLink peer-memory kernels" if world > 1 and args.ep_transport == "p2p"
                                    else "NCCL all-to-all" if world > 1 else "none (one rank)"),
                       "l2": "inputs larger than L2 (11.3 GB of FP8 experts over the ranks)"},
            "roofline": {"kernel": "whole step (route, dispatch, NCCL all-to-all, grouped GEMM, return, combine)",
                         "bound": "tensor", "achieved": round(tflops, 1), "peak": tpeak * world,
                         "unit": "TFLOP/s", "frac": round(tflops / (tpeak * world), 4), "peak_source": kind,
                         "traffic": None, "rows_sent_off_rank_rank0": rows_out},
            "e2e": {"value": EP_T / (e2e_ms / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": EP_T * EP_H * 2,
                    "d2h_bytes_per_step": EP_T * EP_H * 2},
            # route, dispatch plan, pack, shared-expert forward (7), local forward (7), combine
            "gpu_launches": 17 * args.steps,
            "clocks": clk.summary(),
        }), flush=True)
    if hasattr(layer, "close"):
        layer.close()
    local_layer.close()
    shared.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


# ---- stack workload: 48 cached MoE layers, 32 decode sequences ------------------

def run_stack(args):
    import statistics as stats_mod

    import numpy as np
    import torch

    import moe_b200 as M
    from moe_b200 import synth

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    L, SLOTS, SEQS = args.layers, 32, 32
    cfg = M.MoeConfig(num_experts=E, num_experts_per_tok=K_TOP, hidden_size=H, moe_intermediate_size=I)
    prov = M.RoutedExpertsProvider()
    ncpu = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    layers, paged = [], []
    for li in range(L):
        g, u, d = synth.expert_stacks(E, H, I, M.DTYPE_Q8_0, 0.02, seed=3000 + li, device=dev)
        g, u, d = (t.cpu().numpy() for t in (g, u, d))
        router = synth.router_weight(E, H, 0.02, seed=6000 + li, device=dev).cpu().view(torch.int16).numpy().view(np.uint16)
        layer = prov.build(M.ExpertLoadContext(layer=li, device=local, config=cfg, wdtype=M.DTYPE_Q8_0, gate=g, up=u,
                                               down=d, router_weight=router, max_tokens=SEQS, cache_slots=SLOTS))
        cpu = M.CpuExperts(E, K_TOP, H, I, M.DTYPE_Q8_0, g, u, d, threads=ncpu)
        layer.cache_upload(range(SLOTS))  # the fill thread's first pass
        layers.append(layer)
        paged.append(M.PagedMoE(layer, cpu=cpu, pcie_frac=args.pcie_frac, max_tokens=SEQS, staging_slots=16,
                                lookahead=not args.no_lookahead))
        del g, u, d
    for a, b in zip(paged, paged[1:]):  # each layer's activation predicts the next layer's experts
        a.set_next(b)
    torch.cuda.synchronize()
    gen = torch.Generator(device=dev)
    gen.manual_seed(44)
    x0 = torch.randn((SEQS, H), generator=gen, device=dev).to(torch.bfloat16)

    def rmsnorm(x):  # the model's pre-MoE norm (plumbing): keeps the residual stream bounded
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-6)).to(torch.bfloat16)

    def step(x):
        for layer, pm in zip(layers, paged):
            xn = rmsnorm(x)
            ids, w = layer.route(xn)
            x = x + pm.forward(xn, w, ids)
        return x

    x = x0
    for _ in range(max(3, args.warmup)):  # the hidden state carries over from step to step
        x = step(x)
    torch.cuda.synchronize()
    base = [l.cache_stats() for l in layers]
    base_p = [dict(p.stats) for p in paged]
    times = []
    with ClockSampler(local) as clk:
        for _ in range(args.steps):
            t0 = time.perf_counter()
            x = step(x)
            torch.cuda.synchronize()
            times.append(time.perf_counter() - t0)
    for p in paged:
        p.check()
    up_bytes = sum(l.cache_stats()["upload_bytes"] - b["upload_bytes"] for l, b in zip(layers, base))
    pairs = sum(p.stats["pairs"] - b["pairs"] for p, b in zip(paged, base_p))
    hits = sum(p.stats["hits"] - b["hits"] for p, b in zip(paged, base_p))
    cpu_pairs = sum(p.stats["cpu_pairs"] - b["cpu_pairs"] for p, b in zip(paged, base_p))
    delta = {key: sum(p.stats[key] - b[key] for p, b in zip(paged, base_p))
             for key in ("staged_pairs", "staged_experts", "lookahead_passes", "lookahead_loads", "lookahead_swaps",
                         "lookahead_dropped", "predicted")}
    p50 = stats_mod.median(times) * 1e3
    print(json.dumps({
        "metric": "p50 TPOT (ms) of a 32-sequence decode step through a 48-layer MoE stack with a 25% expert cache",
        "value": p50, "unit": "ms", "n_gpus": 1, "steps": args.steps, "warmup": max(3, args.warmup),
        "ms_per_step": statistics.mean(times) * 1e3, "higher_is_better": False, "scaling": "weak",
        "vs_baseline": None, "dtype": "q8_0 weights, f16 tensor-core MMA on the GPU; f32 on the CPU",
        "data": "synthetic: seeded N(0,0.02) Q8_0 experts and routers, N(0,1) bf16 activations",
        "config": {"workload": f"BASELINE config 4 (MoE layers only, attention excluded): {L} Qwen3-30B-A3B-shaped "
                               "Q8_0 layers (E128 k8 H2048 I768), 32 of 128 experts per layer in GPU slots, the rest "
                               "in pinned host memory; 32 sequences per decode step, residual stream "
                               "x += moe(rmsnorm(x)) carried across steps",
                   "layers": L, "cache_slots": SLOTS, "sequences": SEQS, "cpu_threads": ncpu,
                   "miss_policy": f"streamed_misses(frac {args.pcie_frac}, cap 16) into 16 staging slots per layer, "
                                  "resident experts first; the rest on the CPU executor",
                   "lookahead": ("off" if args.no_lookahead else
                                 "each layer's activation predicts the next layer's experts on the lookahead thread "
                                 "(CPU router, union by votes, 1 swap per row)")},
        "tokens_per_s": SEQS / (p50 / 1e3), "hit_rate": hits / max(pairs, 1), "cpu_pair_share": cpu_pairs / max(pairs, 1),
        "staged_pair_share": delta["staged_pairs"] / max(pairs, 1), "paged_stats": delta,
        "h2d_gbs": up_bytes / sum(times) / 1e9, "p90_ms": sorted(times)[int(0.9 * (len(times) - 1))] * 1e3,
        "e2e": {"value": p50, "unit": "ms", "h2d_bytes_per_step": up_bytes // max(len(times), 1),
                "d2h_bytes_per_step": 0},
        "gpu_launches": None, "clocks": clk.summary(),
    }), flush=True)
    for p in paged:
        p.close()
    for l in layers:
        l.close()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=25)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--layers", type=int, default=48)
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--pcie-frac", type=float, default=1.0,
                    help="stack workload: share of each call's missed experts streamed into staging slots")
    ap.add_argument("--no-lookahead", action="store_true", help="stack workload: no next-layer prefetch")
    ap.add_argument("--no-prefill", action="store_true",
                    help="skip the nested config-3 prefill record of the default (decode) run")
    ap.add_argument("--workload", default="decode", choices=["decode", "prefill", "ep", "stack"],
                    help="decode: BASELINE config 2 (the headline); prefill: config 3; ep: config 5; "
                         "stack: config 4")
    ap.add_argument("--chunk", type=int, default=512,
                    help="prefill workload: tokens per grouped pass (4096 = the whole prompt in one pass)")
    ap.add_argument("--ep-transport", default="p2p", choices=["p2p", "nccl"],
                    help="ep workload at N > 1: NVLink peer-memory kernels (default) or NCCL all-to-alls")
    ap.add_argument("--batches", default=None,
                    help="comma-separated batch sizes replacing the ragged sweep (profiling runs only)")
    args = ap.parse_args()
    if args.batches:
        RAGGED[:] = [int(b) for b in args.batches.split(",")]
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "prefill":
        run_prefill(args)
    elif args.workload == "ep":
        run_ep(args)
    elif args.workload == "stack":
        run_stack(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
