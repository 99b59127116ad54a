"""Decode and prefill through an expert cache: the reference's CachedLayer call path (libmoe_b200's
moe_paged_*, csrc/paged.cu).

Reference flow (naiwa-rs src/moe/decode.rs:224-378, stages/route.rs:19-158, stages/dma_miss.rs,
stages/cpu_miss.rs, stages/preload.rs, staging.rs, rings.rs, prefill_stream.rs): the router's top-k
reach the host through the top-k doorbell (no stream sync); the route split marks each pair resident
or missed; `streamed_misses` picks the missed experts worth copying now into staging slots; the rest
run on the CPU from the host stacks while the GPU computes the resident pairs, then the staged ones;
the CPU rows come back through the result doorbell. Each call's activation feeds the next layer's
prediction on a background thread, which prefetches that layer's predicted experts. All of it runs
in the library; this class only holds the handle.
"""
from __future__ import annotations

import ctypes

from ._lib import check, lib
from .layer import _ptr, _stream, _torch


class PagedOpts(ctypes.Structure):
    _fields_ = [
        ("staging_slots", ctypes.c_int),
        ("pcie_frac", ctypes.c_float),
        ("stream_cap", ctypes.c_int),
        ("lookahead", ctypes.c_int),
        ("lookahead_swaps", ctypes.c_int),
        ("max_tokens", ctypes.c_int),
        ("host_timeout_us", ctypes.c_int64),
    ]


class PagedStats(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int64) for n in (
        "calls", "pairs", "hits", "staged_experts", "staged_pairs", "cpu_pairs", "lookahead_passes",
        "lookahead_loads", "lookahead_swaps", "lookahead_dropped", "lookahead_errors", "predicted", "prefill_calls",
        "prefill_waves", "prefill_uploads")]


class PagedMoE:
    """One cached layer's calls (a RoutedExperts built with cache_slots > 0).

    cpu: a CpuExperts for the misses that are not streamed (None: every miss must fit the staging
    slots). pcie_frac / stream_cap: the share and number of missed experts copied per call into the
    layer's staging slots. lookahead: predict the next layer's experts from each call's activation
    (set the next layer with `set_next`)."""

    def __init__(self, layer, cpu=None, pcie_frac: float = 1.0, stream_cap: int | None = None,
                 max_tokens: int | None = None, staging_slots: int = 16, lookahead: bool = True,
                 lookahead_swaps: int = 1, host_timeout_us: int = 5_000_000):
        if not layer.cache_slots:
            raise ValueError("PagedMoE needs a layer built with cache_slots > 0")
        self.layer = layer
        self.cpu = cpu
        o = PagedOpts()
        lib().moe_paged_default_opts(ctypes.byref(o))
        o.staging_slots = int(staging_slots)
        o.pcie_frac = float(pcie_frac)
        o.stream_cap = int(staging_slots if stream_cap is None else stream_cap)
        o.lookahead = 1 if lookahead else 0
        o.lookahead_swaps = int(lookahead_swaps)
        o.max_tokens = int(max_tokens or layer.max_tokens)
        o.host_timeout_us = int(host_timeout_us)
        self.T_max = o.max_tokens
        h = ctypes.c_void_p()
        check(lib().moe_paged_create(layer._h, cpu._h if cpu is not None else None, ctypes.byref(o), ctypes.byref(h)))
        self._h = h

    def set_next(self, nxt: "PagedMoE | None"):
        """The next MoE layer, whose experts this layer's calls predict and prefetch."""
        check(lib().moe_paged_set_next(self._h, nxt._h if nxt is not None else None))

    def forward(self, xs, topk_weights, topk_ids, out=None, stream=None):
        torch = _torch()
        T = xs.shape[0]
        ids = topk_ids if topk_ids.dtype == torch.int32 else topk_ids.to(torch.int32)
        w = topk_weights if topk_weights.dtype == torch.float32 else topk_weights.to(torch.float32)
        ids, w, xs = ids.contiguous(), w.contiguous(), xs.contiguous()
        y = out if out is not None else torch.empty_like(xs)
        check(lib().moe_paged_forward(self._h, _ptr(xs), T, _ptr(ids), _ptr(w), ids.shape[1], _ptr(y),
                                      ctypes.c_void_p(_stream(stream))))
        return y

    __call__ = forward

    def prefill(self, xs, topk_weights, topk_ids, out=None, stream=None):
        """A prompt through the cached layer (PrefillStream::forward, prefill_stream.rs:1362-1694)."""
        torch = _torch()
        T = xs.shape[0]
        ids = topk_ids.to(torch.int32).contiguous()
        w = topk_weights.to(torch.float32).contiguous()
        xs = xs.contiguous()
        y = out if out is not None else torch.empty_like(xs)
        check(lib().moe_paged_prefill(self._h, _ptr(xs), T, _ptr(ids), _ptr(w), ids.shape[1], _ptr(y),
                                      ctypes.c_void_p(_stream(stream))))
        return y

    def fill(self, stream=None):
        """Fill empty slots with the most-routed experts not resident (fill_candidate)."""
        check(lib().moe_paged_fill(self._h, ctypes.c_void_p(_stream(stream))))

    @property
    def stats(self) -> dict:
        s = PagedStats()
        check(lib().moe_paged_get_stats(self._h, ctypes.byref(s)))
        d = {n: int(getattr(s, n)) for n, _ in PagedStats._fields_}
        d["streamed"] = d["staged_experts"]
        return d

    @staticmethod
    def drain_lookahead():
        check(lib().moe_paged_drain_lookahead())

    def check(self, stream=None):
        check(lib().moe_paged_check(self._h, ctypes.c_void_p(_stream(stream))))

    def close(self):
        if getattr(self, "_h", None) is not None and self._h.value:
            lib().moe_paged_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
