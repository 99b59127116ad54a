"""Decode through an expert cache: the reference's split of one MoE layer call between resident GPU
slots, PCIe-streamed misses and the CPU.

Reference flow (naiwa-rs src/moe/decode.rs:224-378, stages/route.rs:19-158, stages/dma_miss.rs,
stages/cpu_miss.rs): the router's top-k reach the host thread through the top-k doorbell (no stream
sync), the route split marks each pair resident or missed, `streamed_misses` picks the missed
experts worth uploading now, the rest run on the CPU from the host stacks while the GPU computes the
resident pairs, and the CPU rows come back through the result doorbell and are added to the GPU's.

Per call, with the library's pieces:
  1. top-k ring (device -> host): ids and weights; activation ring (device -> host): x (bf16),
     both published on the compute stream right after the router;
  2. `RoutedExperts.cache_split` (a2) on the host copy of the ids;
  3. `policy.streamed_misses` over the missed pairs, `RoutedExperts.cache_upload` (a8) of those
     experts, protecting this call's hits;
  4. pairs still missing go to the CPU `Executor` (a11) with a selection mask;
  5. the GPU forward runs the resident pairs (the slot map skips the others);
  6. the result ring (host -> device) brings the CPU rows back; they are added to the output.
"""
from __future__ import annotations

import numpy as np

from . import policy
from .cpu import CpuExperts, Executor, add_f32_into_bf16
from .doorbell import Ring
from .layer import _torch


class PagedMoE:
    def __init__(self, layer, cpu: CpuExperts | None = None, pcie_frac: float = 1.0, stream_cap: int | None = None,
                 max_tokens: int | None = None, host_timeout_us: int = 5_000_000):
        torch = _torch()
        if not layer.cache_slots:
            raise ValueError("PagedMoE needs a layer built with cache_slots > 0")
        self.layer = layer
        self.cpu = cpu
        self.pcie_frac = float(pcie_frac)
        self.stream_cap = layer.cache_slots if stream_cap is None else int(stream_cap)
        self.T_max = int(max_tokens or layer.max_tokens)
        self.k = layer.top_k
        self.H = layer.hidden
        self.timeout = host_timeout_us
        dev = layer.device
        self.topk_ring = Ring(dev, 4, self.T_max * self.k * 8)
        self.act_ring = Ring(dev, 4, self.T_max * self.H * 2) if cpu is not None else None
        self.result_ring = Ring(dev, 4, self.T_max * self.H * 4) if cpu is not None else None
        self.executor = Executor(cpu, self.result_ring) if cpu is not None else None
        self.cpu_rows = torch.empty(self.T_max * self.H, dtype=torch.float32, device=f"cuda:{dev}")
        self.stats = {"calls": 0, "pairs": 0, "hits": 0, "streamed": 0, "cpu_pairs": 0}

    def forward(self, xs, topk_weights, topk_ids, stream=None):
        T = xs.shape[0]
        k = topk_ids.shape[1]
        if T > self.T_max or k != self.k:
            raise ValueError("PagedMoE.forward: T exceeds max_tokens or width != top_k")
        ids_d = topk_ids.to(_torch().int32).contiguous()
        w_d = topk_weights.to(_torch().float32).contiguous()
        seq = self.topk_ring.publish_from_device(ids_d, w_d, stream=stream)
        aseq = self.act_ring.publish_from_device(xs.contiguous(), stream=stream) if self.cpu is not None else 0
        buf = np.empty(T * k * 2, np.uint32)
        self.topk_ring.host_take(seq, buf, timeout_us=self.timeout)  # waits for the router, not the stream
        ids = buf[:T * k].reshape(T, k)
        w = buf[T * k:].view(np.float32).reshape(T, k)
        hit = self.layer.cache_split(ids)
        flat = ids.reshape(-1)
        miss_rows = [[(int(ids[t, j]), float(w[t, j])) for j in range(k) if hit[t * k + j] == 0] for t in range(T)]
        streamed = policy.streamed_misses(miss_rows, self.pcie_frac, self.stream_cap)
        if streamed:
            self.layer.cache_upload(streamed, protect=sorted(set(flat[hit == 1].tolist())), stream=stream)
        resident = self.layer.cache_resident()
        is_res = np.zeros(self.layer.num_experts + 1, bool)
        is_res[resident[resident >= 0]] = True
        live = flat != 0xFFFFFFFF
        now_res = np.where(live, is_res[np.where(live, flat, self.layer.num_experts)], False)
        cpu_sel = (live & ~now_res).astype(np.uint8)
        target = 0
        if self.cpu is not None:
            x_h = np.empty(T * self.H, np.uint16)
            self.act_ring.host_take(aseq, x_h, timeout_us=self.timeout)
            if cpu_sel.any():
                target = self.executor.submit(x_h.reshape(T, self.H), ids, w, cpu_sel)
        elif cpu_sel.any():
            raise RuntimeError("PagedMoE: missed experts with no CPU path and no slot to stream them into")
        y = self.layer.forward(xs, w_d, ids_d, stream=stream)
        if target:
            rows = self.cpu_rows[:T * self.H]
            self.result_ring.device_take(target, rows, stream=stream)
            add_f32_into_bf16(y, rows, stream=stream)
        s = self.stats
        s["calls"] += 1
        s["pairs"] += int(live.sum())
        s["hits"] += int((hit == 1).sum())
        s["streamed"] += len(streamed)
        s["cpu_pairs"] += int(cpu_sel.sum())
        return y

    __call__ = forward

    def prefill(self, xs, topk_weights, topk_ids, chunk: int | None = None, stream=None):
        """A prompt through the cached layer (PrefillStream::forward, prefill_stream.rs:1362-1694): chunks
        of at most `chunk` tokens (default: what the layer's scratch holds); per chunk, its distinct
        experts in waves of at most `slots` (resident ones first, so they need no upload); each wave
        uploads its experts, runs the forward on ids restricted to them (moe_select_ids) and the wave
        outputs are summed per token in f32 and rounded once (moe_ep_combine). All on the GPU."""
        import ctypes

        from ._lib import check, lib
        from .ep import ep_combine
        from .layer import _ptr, _stream

        torch = _torch()
        T, H = xs.shape
        k = topk_ids.shape[1]
        chunk = int(chunk or max(1, self.layer.max_tokens))
        ids_all = topk_ids.to(torch.int32).contiguous()
        w_all = topk_weights.to(torch.float32).contiguous()
        ids_host = ids_all.cpu().numpy().view(np.uint32)
        y = torch.empty_like(xs)
        S = self.layer.cache_slots
        for c0 in range(0, T, chunk):
            c1 = min(T, c0 + chunk)
            n = c1 - c0
            ids_c, w_c, x_c = ids_all[c0:c1], w_all[c0:c1], xs[c0:c1]
            flat = ids_host[c0:c1].reshape(-1)
            distinct = sorted(set(flat[flat != 0xFFFFFFFF].tolist()))
            res = set(int(e) for e in self.layer.cache_resident() if e >= 0)
            order = [e for e in distinct if e in res] + [e for e in distinct if e not in res]
            waves = [order[i:i + S] for i in range(0, len(order), S)] or [[]]
            outs = []
            for wave in waves:
                self.layer.cache_upload(wave, protect=wave, stream=stream)
                sel = torch.empty_like(ids_c)
                ev = np.ascontiguousarray(np.asarray(wave, dtype=np.uint32))
                check(lib().moe_select_ids(_ptr(ids_c), ids_c.numel(), self.layer.num_experts,
                                           ctypes.c_void_p(ev.ctypes.data if ev.size else None), ev.size, _ptr(sel),
                                           ctypes.c_void_p(_stream(stream))))
                outs.append(self.layer.forward(x_c, w_c, sel, stream=stream))
            rows = torch.arange(n, device=xs.device, dtype=torch.int32)
            token_rows = torch.stack([rows + i * n for i in range(len(outs))], dim=1).contiguous()
            y[c0:c1] = ep_combine(torch.cat(outs), token_rows, n, stream=stream)
        return y

    def check(self, stream=None):
        self.layer.check()
        self.topk_ring.check(stream)
        if self.cpu is not None:
            self.act_ring.check(stream)
            self.result_ring.check(stream)
            self.executor.drain()

    def close(self):
        if self.executor is not None:
            self.executor.close()
        for r in (self.topk_ring, self.act_ring, self.result_ring):
            if r is not None:
                r.close()
