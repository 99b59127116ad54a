"""The expert cache's decision functions (libmoe_b200's moe_policy_*; host code, no CUDA).

Reference: naiwa-rs src/moe/cached_layer.rs — fill_candidate (:344-355), top_k_ids (:358-363),
union_by_votes (:367-379), streamed_misses (:385-398), lru_victim (:401-410).
"""
from __future__ import annotations

import ctypes

import numpy as np

from ._lib import lib


def _p(a):
    return ctypes.c_void_p(a.ctypes.data if a.size else None)


def top_k_ids(logits, k: int):
    a = np.ascontiguousarray(logits, dtype=np.float32)
    out = np.empty(max(k, 1), np.int32)
    n = lib().moe_policy_top_k_ids(_p(a), a.size, k, _p(out))
    return [int(v) for v in out[:n]]


def union_by_votes(rankings):
    arrs = [np.ascontiguousarray(r, dtype=np.int32) for r in rankings]
    ptrs = (ctypes.c_void_p * max(len(arrs), 1))(*[ctypes.c_void_p(a.ctypes.data if a.size else None) for a in arrs])
    lens = np.array([a.size for a in arrs] or [0], np.int32)
    out = np.empty(max(sum(a.size for a in arrs), 1), np.int32)
    n = lib().moe_policy_union_by_votes(ctypes.cast(ptrs, ctypes.c_void_p), _p(lens), len(arrs), _p(out))
    return [int(v) for v in out[:n]]


def streamed_misses(misses, frac: float, cap: int):
    """misses: per row, a list of (expert id, routed weight)."""
    ids = np.array([i for row in misses for i, _ in row] or [0], np.uint32)
    ws = np.array([w for row in misses for _, w in row] or [0.0], np.float32)
    lens = np.array([len(row) for row in misses] or [0], np.int32)
    out = np.empty(max(ids.size, 1), np.uint32)
    n = lib().moe_policy_streamed_misses(_p(ids), _p(ws), _p(lens), len(misses), float(frac), int(cap), _p(out))
    return [int(v) for v in out[:n]]


def lru_victim(slots, protect):
    """slots: list of (expert or None, published, last_use). Returns (expert, slot) or None."""
    se = np.array([-1 if e is None else e for e, _, _ in slots] or [0], np.int32)
    pub = np.array([1 if p else 0 for _, p, _ in slots] or [0], np.int32)
    lu = np.array([u for _, _, u in slots] or [0], np.uint64)
    pr = np.array(list(protect) or [0], np.int32)
    ex = ctypes.c_int32(-1)
    s = lib().moe_policy_lru_victim(_p(se), _p(pub), _p(lu), len(slots), _p(pr), len(protect), ctypes.byref(ex))
    return None if s < 0 else (int(ex.value), int(s))


def fill_candidate(slot_experts, hit_counts):
    se = np.array([-1 if e is None else e for e in slot_experts] or [0], np.int32)
    hc = np.ascontiguousarray(hit_counts, dtype=np.uint64)
    c = lib().moe_policy_fill_candidate(_p(se), len(slot_experts), _p(hc), hc.size)
    return None if c < 0 else int(c)
