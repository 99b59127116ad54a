"""ctypes binding of libmoe_b200.so (the C ABI declared in include/moe_b200.h).

The library is the product: every entry point here calls sm_100a kernels. If the shared library
is missing or fails to load, importing this module raises; there is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os

from . import _build

MOE_OK = 0
MOE_ERR_INVALID = 1
MOE_ERR_CUDA = 2
MOE_ERR_OOM = 3
MOE_ERR_TIMEOUT = 4
MOE_ERR_BAD_IDS = 5
MOE_ERR_UNSUPPORTED = 6
MOE_ERR_WORKER = 7

STATUS_NAMES = {
    0: "MOE_OK", 1: "MOE_ERR_INVALID", 2: "MOE_ERR_CUDA", 3: "MOE_ERR_OOM", 4: "MOE_ERR_TIMEOUT",
    5: "MOE_ERR_BAD_IDS", 6: "MOE_ERR_UNSUPPORTED", 7: "MOE_ERR_WORKER",
}

DTYPE_BF16, DTYPE_Q8_0, DTYPE_Q4_K, DTYPE_FP8_E4M3_B128, DTYPE_Q2_0 = 0, 1, 2, 3, 4
ROUTER_SOFTMAX, ROUTER_SOFTMAX_RENORM, ROUTER_SIGMOID_GROUP = 0, 1, 2


class MoeError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {msg}")
        self.status = status


class LayerDesc(ctypes.Structure):
    _fields_ = [
        ("num_experts", ctypes.c_int),
        ("top_k", ctypes.c_int),
        ("hidden", ctypes.c_int),
        ("inter", ctypes.c_int),
        ("wdtype", ctypes.c_int),
        ("gate", ctypes.c_void_p),
        ("up", ctypes.c_void_p),
        ("down", ctypes.c_void_p),
        ("gate_scale", ctypes.c_void_p),
        ("up_scale", ctypes.c_void_p),
        ("down_scale", ctypes.c_void_p),
        ("weights_on_device", ctypes.c_int),
        ("router_weight", ctypes.c_void_p),
        ("router_bias", ctypes.c_void_p),
        ("router_mode", ctypes.c_int),
        ("n_group", ctypes.c_int),
        ("topk_group", ctypes.c_int),
        ("routed_scale", ctypes.c_float),
        ("device", ctypes.c_int),
        ("max_tokens", ctypes.c_int),
        ("cache_slots", ctypes.c_int),
    ]


MOE_ID_NONE = 0xFFFFFFFF  # empty top-k slot: skipped by the plan (include/moe_b200.h)

LIB_PATH = _build.LIB
_lib = None


def lib():
    """Load libmoe_b200.so (building it first when the sources are newer). MOE_B200_LIB names
    another build of the same library to load instead (an alternate build of the same sources)."""
    global _lib
    if _lib is None:
        alt = os.environ.get("MOE_B200_LIB")
        if not alt and (not os.path.exists(LIB_PATH) or os.environ.get("MOE_B200_REBUILD") == "1"):
            _build.build()
        L = ctypes.CDLL(alt or LIB_PATH)
        P, i, f = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
        sigs = {
            "moe_layer_create": (i, [ctypes.POINTER(LayerDesc), ctypes.POINTER(ctypes.c_void_p)]),
            "moe_layer_warmup": (i, [P, i]),
            "moe_route": (i, [P, P, i, P, P, P]),
            "moe_requantize_q2_0": (i, [i, P, i, i, i, P, P]),
            "moe_forward": (i, [P, P, i, P, P, i, P, P]),
            "moe_forward_marked": (i, [P, P, i, P, P, i, P, P, ctypes.POINTER(ctypes.c_void_p)]),
            "moe_layer_destroy": (None, [P]),
            "moe_layer_device_bytes": (ctypes.c_int64, [P]),
            "moe_layer_check": (i, [P, P]),
            "moe_layer_set_live_hint": (i, [P, f]),
            "moe_last_error": (ctypes.c_size_t, [ctypes.c_char_p, ctypes.c_size_t]),
            "moe_route_tokens": (i, [P, P, P, i, i, i, i, i, i, i, f, P, P, P, ctypes.c_size_t, P]),
            "moe_route_workspace_bytes": (ctypes.c_size_t, [i, i]),
            "moe_route_tokens_noalloc": (i, [P, P, P, i, i, i, i, i, i, i, f, P, P, P]),
            "moe_plan_pairs": (i, [P, i, i, P, P, P, P, P, P, ctypes.c_size_t, P, P]),
            "moe_plan_workspace_bytes": (ctypes.c_size_t, [i, i]),
            "moe_ep_dispatch_plan": (i, [P, P, i, i, i, i, P, P, P, P, P, P, P, P]),
            "moe_ep_pack_rows": (i, [P, i, i, P, P, i, P, P]),
            "moe_ep_combine": (i, [P, P, i, i, i, P, P, P]),
            "moe_cache_split": (i, [P, P, i, P]),
            "moe_cache_upload": (i, [P, P, i, P, i, P, ctypes.POINTER(ctypes.c_int)]),
            "moe_cache_slots": (i, [P, P]),
            "moe_cache_stats": (i, [P, P, P, P, P, P]),
            "moe_policy_top_k_ids": (i, [P, i, i, P]),
            "moe_policy_union_by_votes": (i, [P, P, i, P]),
            "moe_policy_streamed_misses": (i, [P, P, P, i, f, i, P]),
            "moe_policy_lru_victim": (i, [P, P, P, i, P, i, P]),
            "moe_policy_fill_candidate": (i, [P, i, P, i]),
            "moe_cpu_experts_create": (i, [ctypes.POINTER(LayerDesc), i, ctypes.POINTER(ctypes.c_void_p)]),
            "moe_cpu_experts_destroy": (None, [P]),
            "moe_cpu_forward": (i, [P, P, P, P, i, i, P, P]),
            "moe_cpu_isa": (ctypes.c_char_p, []),
            "moe_executor_create": (i, [P, P, ctypes.POINTER(ctypes.c_void_p)]),
            "moe_executor_submit": (i, [P, P, P, P, i, i, P, ctypes.POINTER(ctypes.c_uint32)]),
            "moe_executor_drain": (i, [P]),
            "moe_executor_destroy": (None, [P]),
            "moe_add_f32_into_bf16": (i, [P, P, ctypes.c_int64, P]),
            "moe_select_ids": (i, [P, ctypes.c_int64, i, P, i, P, P]),
            "moe_forward_chunked": (i, [P, P, i, P, P, i, P, P]),
            "moe_ep_peer_create": (i, [i, i, i, i, i, i, ctypes.POINTER(ctypes.c_void_p)]),
            "moe_ep_peer_handle_bytes": (ctypes.c_size_t, []),
            "moe_ep_peer_export": (i, [P, P]),
            "moe_ep_peer_connect": (i, [P, P]),
            "moe_ep_peer_destroy": (None, [P]),
            "moe_ep_peer_recv_rows": (P, [P]),
            "moe_ep_peer_dispatch": (i, [P, P, i, P, P, P, P, ctypes.c_uint32, P]),
            "moe_ep_peer_receive": (i, [P, ctypes.c_uint32, P, P, P]),
            "moe_ep_peer_dispatch_routed": (i, [P, P, i, P, P, i, ctypes.c_uint32, P, P, P, P]),
            "moe_ep_peer_recv_ids": (P, [P]),
            "moe_ep_peer_recv_weights": (P, [P]),
            "moe_ep_peer_return": (i, [P, P, ctypes.c_uint32, P]),
            "moe_ep_peer_combine": (i, [P, ctypes.c_uint32, i, P, P, P, P, P]),
            "moe_ep_peer_check": (i, [P, P]),
            "moe_ep_peer_set_wait_limit": (i, [P, ctypes.c_int64]),
            "moe_ring_create": (i, [i, i, ctypes.c_size_t, ctypes.POINTER(ctypes.c_void_p)]),
            "moe_ring_destroy": (None, [P]),
            "moe_ring_slot_bytes": (ctypes.c_size_t, [P]),
            "moe_ring_publish_from_device": (i, [P, P, ctypes.c_size_t, P, ctypes.c_size_t, P,
                                                 ctypes.POINTER(ctypes.c_uint32)]),
            "moe_ring_host_take": (i, [P, ctypes.c_uint32, P, ctypes.c_size_t, ctypes.c_int64]),
            "moe_ring_host_publish": (i, [P, P, ctypes.c_size_t, ctypes.c_int64, ctypes.POINTER(ctypes.c_uint32)]),
            "moe_ring_device_take": (i, [P, ctypes.c_uint32, P, ctypes.c_size_t, P]),
            "moe_ring_check": (i, [P, P]),
            "moe_ring_counters": (None, [P, ctypes.POINTER(ctypes.c_uint32), ctypes.POINTER(ctypes.c_uint32)]),
            "moe_paged_default_opts": (None, [P]),
            "moe_paged_create": (i, [P, P, P, ctypes.POINTER(ctypes.c_void_p)]),
            "moe_paged_destroy": (None, [P]),
            "moe_paged_set_next": (i, [P, P]),
            "moe_paged_forward": (i, [P, P, i, P, P, i, P, P]),
            "moe_paged_prefill": (i, [P, P, i, P, P, i, P, P]),
            "moe_paged_fill": (i, [P, P]),
            "moe_paged_get_stats": (i, [P, P]),
            "moe_paged_drain_lookahead": (i, []),
            "moe_paged_check": (i, [P, P]),
            "moe_gguf_open": (i, [ctypes.c_char_p, ctypes.POINTER(ctypes.c_void_p)]),
            "moe_gguf_close": (None, [P]),
            "moe_gguf_tensor_count": (i, [P]),
            "moe_gguf_tensor_name": (ctypes.c_char_p, [P, i]),
            "moe_gguf_tensor": (i, [P, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int64),
                                    ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_void_p),
                                    ctypes.POINTER(ctypes.c_int64)]),
            "moe_gguf_get_int": (i, [P, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int64)]),
            "moe_gguf_get_str": (ctypes.c_size_t, [P, ctypes.c_char_p, ctypes.c_char_p, ctypes.c_size_t]),
            "moe_gguf_layer_desc": (i, [P, i, ctypes.POINTER(LayerDesc)]),
            "moe_version": (ctypes.c_char_p, []),
        }
        for name, (res, args) in sigs.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    lib().moe_last_error(buf, 1024)
    return buf.value.decode(errors="replace")


def check(status: int):
    if status != MOE_OK:
        raise MoeError(status, last_error())
