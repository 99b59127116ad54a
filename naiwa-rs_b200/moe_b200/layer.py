"""Host-side mirror of the reference's routed-experts operator interface over libmoe_b200.so.

Reference (naiwa-rs, in its mistral.rs fork's `moe_offload` module):
  RoutedExpertsProvider::build(&self, ctx: ExpertLoadContext) -> Result<Option<Arc<dyn RoutedExperts>>>
      src/moe/provider.rs:316-615
  RoutedExperts::forward(&self, xs, topk_weights, topk_ids) -> Result<Tensor>
      src/moe/cached_layer.rs:524-664, src/moe/expert.rs:59-117

Argument meaning follows the reference: `xs` is [B, S, H] (or [T, H]) in the model dtype (bf16),
`topk_weights` [B*S, k] f32, `topk_ids` [B*S, k] u32/int; the result is a new tensor shaped like
`xs`. Errors raise MoeError (the reference's candle_core::Result bails). Tensors are torch CUDA
tensors; torch supplies device memory and the current stream, the kernels are the library's.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Any, Optional

import numpy as np

from . import _lib
from ._lib import LayerDesc, MoeError, check, lib


def _torch():
    import torch

    return torch


def _ptr(t) -> int:
    return 0 if t is None else int(t.data_ptr())


def _stream(stream=None) -> int:
    torch = _torch()
    if stream is None:
        stream = torch.cuda.current_stream()
    return int(stream.cuda_stream)


@dataclass
class MoeConfig:
    """The fields of the reference's ctx.config the operator reads (provider.rs:316-370)."""

    num_experts: int
    num_experts_per_tok: int
    hidden_size: int
    moe_intermediate_size: int
    router_mode: int = _lib.ROUTER_SOFTMAX_RENORM
    n_group: int = 1
    topk_group: int = 1
    routed_scaling_factor: float = 1.0


@dataclass
class ExpertLoadContext:
    """What the reference's provider receives per MoE block (provider.rs:316-370): the layer site,
    its device, the config, and the expert stacks (`expert_qtensors()` -> gate, up, down stacked
    [E, N, K] in GGML byte layout). Stacks may be host numpy uint8 arrays or CUDA uint8 tensors."""

    layer: int
    device: int
    config: MoeConfig
    wdtype: int
    gate: Any
    up: Any
    down: Any
    gate_scale: Any = None
    up_scale: Any = None
    down_scale: Any = None
    router_weight: Any = None  # [E, H] bf16 (torch tensor or numpy uint16)
    router_bias: Any = None    # [E] f32
    max_tokens: int = 256
    cache_slots: int = 0  # > 0: expert cache with this many device slots (CachedLayer)
    _keep: list = field(default_factory=list)


def _as_ptr(obj, keep: list, on_device: bool):
    """Raw pointer of a numpy array or torch tensor; numpy arrays are kept alive in `keep`."""
    if obj is None:
        return None
    if isinstance(obj, np.ndarray):
        if on_device:
            raise MoeError(_lib.MOE_ERR_INVALID, "mixed host and device inputs")
        a = np.ascontiguousarray(obj)
        keep.append(a)
        return a.ctypes.data
    torch = _torch()
    if isinstance(obj, torch.Tensor):
        if obj.is_cuda != on_device:
            raise MoeError(_lib.MOE_ERR_INVALID, "mixed host and device inputs")
        t = obj.contiguous()
        keep.append(t)
        return t.data_ptr()
    raise TypeError(type(obj))


class RoutedExperts:
    """One MoE layer's routed experts, resident on a B200 (the reference's CachedExperts with
    every expert in its cache). Created by RoutedExpertsProvider.build."""

    def __init__(self, ctx: ExpertLoadContext):
        torch = _torch()
        cfg = ctx.config
        self.layer = ctx.layer
        self.device = ctx.device
        self.config = cfg
        self.hidden = cfg.hidden_size
        self.top_k = cfg.num_experts_per_tok
        self.num_experts = cfg.num_experts
        self.wdtype = ctx.wdtype
        on_dev = isinstance(ctx.gate, torch.Tensor) and ctx.gate.is_cuda
        keep: list = []
        d = LayerDesc()
        d.num_experts = cfg.num_experts
        d.top_k = cfg.num_experts_per_tok
        d.hidden = cfg.hidden_size
        d.inter = cfg.moe_intermediate_size
        d.wdtype = ctx.wdtype
        d.gate = _as_ptr(ctx.gate, keep, on_dev)
        d.up = _as_ptr(ctx.up, keep, on_dev)
        d.down = _as_ptr(ctx.down, keep, on_dev)
        d.gate_scale = _as_ptr(ctx.gate_scale, keep, on_dev)
        d.up_scale = _as_ptr(ctx.up_scale, keep, on_dev)
        d.down_scale = _as_ptr(ctx.down_scale, keep, on_dev)
        d.weights_on_device = 1 if on_dev else 0
        d.router_weight = _as_ptr(ctx.router_weight, keep, on_dev)
        d.router_bias = _as_ptr(ctx.router_bias, keep, on_dev)
        d.router_mode = cfg.router_mode
        d.n_group = cfg.n_group
        d.topk_group = cfg.topk_group
        d.routed_scale = cfg.routed_scaling_factor
        d.device = ctx.device
        d.max_tokens = ctx.max_tokens
        d.cache_slots = int(ctx.cache_slots)
        handle = ctypes.c_void_p()
        if on_dev:
            torch.cuda.synchronize(ctx.device)
        check(lib().moe_layer_create(ctypes.byref(d), ctypes.byref(handle)))
        self._h = handle
        self.max_tokens = ctx.max_tokens
        self.cache_slots = int(ctx.cache_slots) if 0 < ctx.cache_slots < cfg.num_experts else 0

    # -- expert cache (cache_slots > 0) ---------------------------------------------------------
    def cache_split(self, ids) -> np.ndarray:
        """Route split of host ids ([T, k] or flat): 1 hit, 0 miss, 2 empty slot (route.rs:19-158)."""
        a = np.ascontiguousarray(np.asarray(ids).astype(np.uint32).reshape(-1))
        hit = np.empty(a.size, np.uint8)
        check(lib().moe_cache_split(self._h, ctypes.c_void_p(a.ctypes.data), a.size, ctypes.c_void_p(hit.ctypes.data)))
        return hit

    def cache_upload(self, experts, protect=(), stream=None) -> int:
        """Make `experts` resident (admit / LRU replace outside `protect`); returns how many came in."""
        e = np.ascontiguousarray(np.asarray(list(experts), dtype=np.uint32))
        pr = np.ascontiguousarray(np.asarray(list(protect), dtype=np.uint32))
        n = ctypes.c_int()
        check(lib().moe_cache_upload(self._h, ctypes.c_void_p(e.ctypes.data if e.size else None), e.size,
                                     ctypes.c_void_p(pr.ctypes.data if pr.size else None), pr.size,
                                     ctypes.c_void_p(_stream(stream)), ctypes.byref(n)))
        return int(n.value)

    def cache_resident(self) -> np.ndarray:
        """Each slot's expert (-1: empty)."""
        n = lib().moe_cache_slots(self._h, None)
        out = np.empty(n, np.int32)
        if n:
            lib().moe_cache_slots(self._h, ctypes.c_void_p(out.ctypes.data))
        return out

    def cache_stats(self) -> dict:
        v = [ctypes.c_int64() for _ in range(4)]
        hc = np.zeros(self.num_experts, np.uint64)
        check(lib().moe_cache_stats(self._h, *[ctypes.byref(x) for x in v], ctypes.c_void_p(hc.ctypes.data)))
        return {"hits": v[0].value, "misses": v[1].value, "uploads": v[2].value, "upload_bytes": v[3].value,
                "hit_counts": hc}

    # -- lifecycle ------------------------------------------------------------------------------
    def close(self):
        if getattr(self, "_h", None) is not None and self._h.value:
            lib().moe_layer_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def warmup(self, max_tokens: int):
        """Size scratch for `max_tokens` (the reference's provider warmup, provider.rs:192-303)."""
        check(lib().moe_layer_warmup(self._h, int(max_tokens)))
        self.max_tokens = max(self.max_tokens, int(max_tokens))

    def set_live_hint(self, live_fraction: float):
        """Expected share of live (non-empty) id slots per forward: steers the kernel-path choice only."""
        check(lib().moe_layer_set_live_hint(self._h, float(live_fraction)))

    def device_bytes(self) -> int:
        return int(lib().moe_layer_device_bytes(self._h))

    def check(self, stream=None):
        """Raise MoeError when a previous forward latched a device-side error (bad ids)."""
        check(lib().moe_layer_check(self._h, ctypes.c_void_p(_stream(stream))))

    # -- the operator -------------------------------------------------------------------------------
    def route(self, xs, out_ids=None, out_weights=None, stream=None):
        """Router + top-k for xs [.., H] bf16 -> (ids [T, k] int32 view of u32, weights [T, k] f32)."""
        torch = _torch()
        x2 = xs.reshape(-1, self.hidden)
        if x2.dtype != torch.bfloat16 or not x2.is_cuda:
            raise MoeError(_lib.MOE_ERR_INVALID, "route: xs must be a CUDA bf16 tensor")
        x2 = x2.contiguous()
        T = x2.shape[0]
        ids = out_ids if out_ids is not None else torch.empty((T, self.top_k), dtype=torch.int32, device=x2.device)
        w = out_weights if out_weights is not None else torch.empty((T, self.top_k), dtype=torch.float32,
                                                                    device=x2.device)
        check(lib().moe_route(self._h, _ptr(x2), T, _ptr(ids), _ptr(w), ctypes.c_void_p(_stream(stream))))
        return ids, w

    def forward_chunked(self, xs, topk_weights, topk_ids, out=None, stream=None):
        """forward over any number of tokens, in chunks the layer's scratch holds (prefill chunking,
        prefill_stream.rs:1362-1694)."""
        return self.forward(xs, topk_weights, topk_ids, out=out, stream=stream, _entry="moe_forward_chunked")

    def forward(self, xs, topk_weights, topk_ids, out=None, stream=None, _entry="moe_forward"):
        """sum_j topk_weights[t, j] * expert(topk_ids[t, j])(xs[t]) for every token, in xs's shape."""
        torch = _torch()
        shape = xs.shape
        x2 = xs.reshape(-1, self.hidden)
        if x2.dtype != torch.bfloat16 or not x2.is_cuda:
            raise MoeError(_lib.MOE_ERR_INVALID, "forward: xs must be a CUDA bf16 tensor")
        x2 = x2.contiguous()
        T = x2.shape[0]
        if T == 0:
            return (out if out is not None else torch.empty_like(x2)).reshape(shape)
        ids = topk_ids.reshape(T, -1)
        if ids.dtype not in (torch.int32, torch.uint32) or not ids.is_cuda:
            ids = ids.to(device=x2.device, dtype=torch.int32)
        ids = ids.contiguous()
        w = topk_weights.reshape(T, -1)
        if w.dtype != torch.float32 or not w.is_cuda:
            w = w.to(device=x2.device, dtype=torch.float32)
        w = w.contiguous()
        if w.shape != ids.shape:
            raise MoeError(_lib.MOE_ERR_INVALID, "forward: topk_weights and topk_ids shapes differ")
        width = ids.shape[1]
        y = out if out is not None else torch.empty_like(x2)
        check(getattr(lib(), _entry)(self._h, _ptr(x2), T, _ptr(ids), _ptr(w), width, _ptr(y),
                                     ctypes.c_void_p(_stream(stream))))
        return y.reshape(shape)

    __call__ = forward


class RoutedExpertsProvider:
    """Builds the per-layer operator (GpuCacheMoeProvider::build, provider.rs:316-615)."""

    def __init__(self):
        self.layers: dict[int, RoutedExperts] = {}

    def build(self, ctx: ExpertLoadContext) -> Optional[RoutedExperts]:
        layer = RoutedExperts(ctx)
        self.layers[ctx.layer] = layer
        return layer

    def warmup(self, max_tokens: int):
        for layer in self.layers.values():
            layer.warmup(max_tokens)

    def build_resident(self, ctx: ExpertLoadContext) -> RoutedExperts:
        """The reference's resident pool (resident.rs:92-182): the block's expert stacks requantised to
        Q2_0 on the layer's device (moe_requantize_q2_0) and kept resident, run by the same expert
        kernels. ctx holds BF16, Q8_0 or Q4_K stacks (host or CUDA); hidden and inter must be
        multiples of 128."""
        import dataclasses

        c = ctx.config
        E, H, I = c.num_experts, c.hidden_size, c.moe_intermediate_size
        stacks = [requantize_q2_0(s, ctx.wdtype, E, n, k, device=ctx.device)
                  for s, (n, k) in zip((ctx.gate, ctx.up, ctx.down), ((I, H), (I, H), (H, I)))]
        rctx = dataclasses.replace(ctx, wdtype=_lib.DTYPE_Q2_0, gate=stacks[0], up=stacks[1], down=stacks[2],
                                   gate_scale=None, up_scale=None, down_scale=None, _keep=[])
        return self.build(rctx)


# ---- stateless kernels ---------------------------------------------------------------------------

def requantize_q2_0(stack, src_dtype: int, E: int, N: int, K: int, device: int = 0, stream=None):
    """A stacked [E, N, K] projection (GGML bytes of src_dtype: BF16, Q8_0 or Q4_K; numpy uint8 or a
    CUDA uint8 tensor) requantised to Q2_0 on the device: a CUDA uint8 tensor of E*N*K/64*18 bytes
    (moe_requantize_q2_0, the reference's quantize_q2_0 scale-ladder search)."""
    torch = _torch()
    dev = torch.device("cuda", device)
    src = torch.from_numpy(np.ascontiguousarray(stack).reshape(-1)).to(dev) if isinstance(stack, np.ndarray) \
        else stack.reshape(-1).contiguous()
    out = torch.empty(E * N * K // 64 * 18, dtype=torch.uint8, device=dev)
    check(lib().moe_requantize_q2_0(int(src_dtype), _ptr(src), E, N, K, _ptr(out), ctypes.c_void_p(_stream(stream))))
    return out

def route_tokens(x, w_router, k: int, mode: int, bias=None, n_group: int = 1, topk_group: int = 1,
                 routed_scale: float = 1.0, stream=None):
    """Router logits + top-k without a layer: x [T, H] bf16, w_router [E, H] bf16 (CUDA)."""
    torch = _torch()
    T, H = x.shape
    E = w_router.shape[0]
    ids = torch.empty((T, k), dtype=torch.int32, device=x.device)
    w = torch.empty((T, k), dtype=torch.float32, device=x.device)
    ws_bytes = int(lib().moe_route_workspace_bytes(T, E))
    ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=x.device)
    check(lib().moe_route_tokens(_ptr(x.contiguous()), _ptr(w_router.contiguous()), _ptr(bias), T, H, E, k, mode,
                                 n_group, topk_group, float(routed_scale), _ptr(ids), _ptr(w), _ptr(ws), ws_bytes,
                                 ctypes.c_void_p(_stream(stream))))
    return ids, w


class Router:
    """The router of one MoE block on its own (the gate linear + top-k upstream of RoutedExperts.forward),
    for callers whose experts are not one local layer: an expert-parallel rank routes its tokens over
    all experts while holding only its share. Holds the gate, the bias and a workspace sized for
    max_tokens, so each call allocates nothing (and can be captured in a CUDA graph)."""

    def __init__(self, w_router, k: int, mode: int, max_tokens: int, bias=None, n_group: int = 1,
                 topk_group: int = 1, routed_scale: float = 1.0):
        torch = _torch()
        self.w = w_router.contiguous()
        self.E, self.H = self.w.shape
        self.k, self.mode, self.bias = int(k), int(mode), bias
        self.n_group, self.topk_group, self.scale = int(n_group), int(topk_group), float(routed_scale)
        self.max_tokens = int(max_tokens)
        self.ws_bytes = int(lib().moe_route_workspace_bytes(self.max_tokens, self.E))
        self.ws = torch.zeros(self.ws_bytes, dtype=torch.uint8, device=self.w.device)  # counters start at 0

    def route(self, x, out_ids=None, out_weights=None, stream=None):
        torch = _torch()
        T = x.shape[0]
        if T > self.max_tokens:
            raise MoeError(_lib.MOE_ERR_INVALID, "Router.route: T exceeds max_tokens")
        ids = out_ids if out_ids is not None else torch.empty((T, self.k), dtype=torch.int32, device=x.device)
        w = out_weights if out_weights is not None else torch.empty((T, self.k), dtype=torch.float32, device=x.device)
        check(lib().moe_route_tokens(_ptr(x), _ptr(self.w), _ptr(self.bias), T, self.H, self.E, self.k, self.mode,
                                     self.n_group, self.topk_group, self.scale, _ptr(ids), _ptr(w), _ptr(self.ws),
                                     self.ws_bytes, ctypes.c_void_p(_stream(stream))))
        return ids, w


def plan_pairs(ids, num_experts: int, stream=None):
    """Histogram + stable permutation of routed pairs -> (counts, offsets, perm, active, error_word)."""
    torch = _torch()
    flat = ids.reshape(-1).to(torch.int32).contiguous()
    n = flat.numel()
    dev = flat.device
    counts = torch.empty(num_experts, dtype=torch.int32, device=dev)
    offsets = torch.empty(num_experts + 1, dtype=torch.int32, device=dev)
    perm = torch.empty(max(n, 1), dtype=torch.int32, device=dev)
    active = torch.empty(num_experts, dtype=torch.int32, device=dev)
    n_active = torch.zeros(1, dtype=torch.int32, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    ws_bytes = int(lib().moe_plan_workspace_bytes(n, num_experts))
    ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=dev)
    check(lib().moe_plan_pairs(_ptr(flat), n, num_experts, _ptr(counts), _ptr(offsets), _ptr(perm), _ptr(active),
                               _ptr(n_active), _ptr(ws), ws_bytes, _ptr(err), ctypes.c_void_p(_stream(stream))))
    return counts, offsets, perm[:n], active, n_active, err
