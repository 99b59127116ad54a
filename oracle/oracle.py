"""ctypes front-end of the CPU oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY. Imported by tests/, __graft_entry__.smoke() and bench.py's
cpu_baseline leg, always as the checker or as the timed CPU baseline; the product library
(libmoe_b200.so and the moe_b200 package) never imports it.

Every wrapper takes and returns numpy arrays; the C functions it calls cite the reference
file:line they restate (oracle/moe_oracle.c).
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

DT_BF16, DT_Q8_0, DT_Q4_K, DT_FP8, DT_Q2_0 = 0, 1, 2, 3, 4


def build() -> str:
    """Compile liboracle.so with the Makefile beside this file (gcc only)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        srcs = [os.path.join(_HERE, f) for f in ("moe_oracle.c", "cpu_baseline.c", "moe_oracle.h", "Makefile")]
        if not os.path.exists(_LIB_PATH) or any(
                os.path.exists(f) and os.path.getmtime(f) > os.path.getmtime(_LIB_PATH) for f in srcs):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        P = ctypes.c_void_p
        i, i64, f = ctypes.c_int, ctypes.c_int64, ctypes.c_float
        sig = {
            "orc_f16_to_f32": (f, [ctypes.c_uint16]),
            "orc_f32_to_f16": (ctypes.c_uint16, [f]),
            "orc_bf16_to_f32": (f, [ctypes.c_uint16]),
            "orc_f32_to_bf16": (ctypes.c_uint16, [f]),
            "orc_fp8e4m3_to_f32": (f, [ctypes.c_uint8]),
            "orc_f32_to_fp8e4m3": (ctypes.c_uint8, [f]),
            "orc_exp": (f, [f]),
            "orc_sigmoid": (f, [f]),
            "orc_silu": (f, [f]),
            "orc_q8_0_quantize": (None, [P, i64, P]),
            "orc_q8_0_dequantize": (None, [P, i64, P]),
            "orc_q4_k_quantize": (None, [P, i64, P]),
            "orc_q2_0_quantize": (None, [P, i64, P]),
            "orc_q2_0_dequantize": (None, [P, i64, P]),
            "orc_q4_k_dequantize": (None, [P, i64, P]),
            "orc_fp8_b128_quantize": (None, [P, i, i, P, P]),
            "orc_fp8_b128_dequantize": (None, [P, P, i, i, P]),
            "orc_block_bytes": (i64, [i, i64]),
            "orc_expert_range": (i, [i, i, i, i, i, P, P]),
            "orc_top_k_ids": (i, [P, i, i, P]),
            "orc_union_by_votes": (i, [P, P, i, P]),
            "orc_streamed_misses": (i, [P, P, P, i, f, i, P]),
            "orc_lru_victim": (i, [P, P, P, i, P, i, P]),
            "orc_fill_candidate": (i, [P, i, P, i]),
            "orc_router_logits": (None, [P, P, i, i, i, P]),
            "orc_route": (i, [P, P, i, i, i, i, i, i, f, P, P]),
            "orc_permute": (i, [P, i, i, P, P, P, P, P]),
            "orc_moe_forward_f32": (None, [P, P, P, i, i, i, i, i, P, P, P, P]),
            "orc_moe_forward_ref": (i, [i, P, P, P, P, P, P, P, P, P, i, i, i, i, i, i, P]),
            "orc_fused_moe_decode_q8_0": (i, [P, P, P, P, P, P, i, i, i, i, i, i, P]),
            "orc_baseline_decode_q8_0": (i, [P, P, P, P, P, P, i, i, i, i, i, i, P]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(ctypes.c_void_p)


# ---- scalar formats ------------------------------------------------------------------------

def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16 bits (uint16), vectorised restatement of
    orc_f32_to_bf16."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    r[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return r


def bf16_to_f32(h: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(h, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def exp(x: float) -> float:
    return lib().orc_exp(float(x))


# ---- block formats -------------------------------------------------------------------------

def block_bytes(dtype: int, n_weights: int) -> int:
    return int(lib().orc_block_bytes(dtype, n_weights))


def quantize(dtype: int, w: np.ndarray):
    """Quantise a float array whose last dim is K into the GGML layout of `dtype`.
    Returns (bytes uint8 array, scales or None). FP8 needs a [..., N, K] array."""
    w = np.ascontiguousarray(w, dtype=np.float32)
    if dtype == DT_BF16:
        return f32_to_bf16(w).view(np.uint8).reshape(-1), None
    if dtype == DT_Q8_0:
        out = np.empty(w.size // 32 * 34, dtype=np.uint8)
        lib().orc_q8_0_quantize(_p(w), w.size, _p(out))
        return out, None
    if dtype == DT_Q4_K:
        out = np.empty(w.size // 256 * 144, dtype=np.uint8)
        lib().orc_q4_k_quantize(_p(w), w.size, _p(out))
        return out, None
    if dtype == DT_Q2_0:
        out = np.empty(w.size // 64 * 18, dtype=np.uint8)
        lib().orc_q2_0_quantize(_p(w), w.size, _p(out))
        return out, None
    if dtype == DT_FP8:
        n, k = w.shape[-2], w.shape[-1]
        lead = int(np.prod(w.shape[:-2])) if w.ndim > 2 else 1
        q = np.empty(w.size, dtype=np.uint8)
        sc = np.empty(lead * (n // 128) * (k // 128), dtype=np.float32)
        per, per_s = n * k, (n // 128) * (k // 128)
        for e in range(lead):
            src = np.ascontiguousarray(w.reshape(lead, n, k)[e])
            qe = np.empty(per, dtype=np.uint8)
            se = np.empty(per_s, dtype=np.float32)
            lib().orc_fp8_b128_quantize(_p(src), n, k, _p(qe), _p(se))
            q[e * per:(e + 1) * per] = qe
            sc[e * per_s:(e + 1) * per_s] = se
        return q, sc
    raise ValueError(dtype)


def dequantize(dtype: int, blob: np.ndarray, shape, scales=None) -> np.ndarray:
    n = int(np.prod(shape))
    out = np.empty(n, dtype=np.float32)
    blob = np.ascontiguousarray(blob)
    if dtype == DT_BF16:
        out[:] = bf16_to_f32(blob.view(np.uint16)[:n])
    elif dtype == DT_Q8_0:
        lib().orc_q8_0_dequantize(_p(blob), n, _p(out))
    elif dtype == DT_Q4_K:
        lib().orc_q4_k_dequantize(_p(blob), n, _p(out))
    elif dtype == DT_Q2_0:
        lib().orc_q2_0_dequantize(_p(blob), n, _p(out))
    elif dtype == DT_FP8:
        nn, kk = shape[-2], shape[-1]
        lead = n // (nn * kk)
        per, per_s = nn * kk, (nn // 128) * (kk // 128)
        sc = np.ascontiguousarray(scales, dtype=np.float32)
        for e in range(lead):
            q = np.ascontiguousarray(blob[e * per:(e + 1) * per])
            s = np.ascontiguousarray(sc[e * per_s:(e + 1) * per_s])
            o = np.empty(per, dtype=np.float32)
            lib().orc_fp8_b128_dequantize(_p(q), _p(s), nn, kk, _p(o))
            out[e * per:(e + 1) * per] = o
    else:
        raise ValueError(dtype)
    return out.reshape(shape)


def expert_range(dtype: int, E: int, N: int, K: int, e: int):
    b, en = ctypes.c_int64(), ctypes.c_int64()
    rc = lib().orc_expert_range(dtype, E, N, K, e, ctypes.byref(b), ctypes.byref(en))
    if rc != 0:
        raise IndexError(f"expert {e} out of range or K={K} not a block multiple")
    return b.value, en.value


# ---- cache policy ----------------------------------------------------------------------------

def top_k_ids(logits, k: int):
    a = np.ascontiguousarray(logits, dtype=np.float32)
    out = np.empty(max(k, 1), dtype=np.int32)
    n = lib().orc_top_k_ids(_p(a), a.size, k, _p(out))
    return [int(v) for v in out[:n]]


def union_by_votes(rankings):
    arrs = [np.ascontiguousarray(r, dtype=np.int32) for r in rankings]
    ptrs = (ctypes.c_void_p * len(arrs))(*[a.ctypes.data for a in arrs])
    lens = np.array([len(a) for a in arrs], dtype=np.int32)
    out = np.empty(max(1, int(lens.sum())), dtype=np.int32)
    n = lib().orc_union_by_votes(ctypes.cast(ptrs, ctypes.c_void_p), _p(lens), len(arrs), _p(out))
    return [int(v) for v in out[:n]]


def streamed_misses(misses, frac: float, cap: int):
    ids = np.array([i for row in misses for (i, _) in row] or [0], dtype=np.uint32)
    ws = np.array([w for row in misses for (_, w) in row] or [0.0], dtype=np.float32)
    lens = np.array([len(r) for r in misses] or [0], dtype=np.int32)
    out = np.empty(max(1, ids.size), dtype=np.uint32)
    n = lib().orc_streamed_misses(_p(ids), _p(ws), _p(lens), len(misses), frac, cap, _p(out))
    return [int(v) for v in out[:n]]


def lru_victim(slots, protect):
    """slots: list of (expert or None, published, last_use). Returns (expert, slot) or None."""
    ex = np.array([-1 if e is None else e for (e, _, _) in slots], dtype=np.int32)
    pub = np.array([1 if p else 0 for (_, p, _) in slots], dtype=np.int32)
    lu = np.array([u for (_, _, u) in slots], dtype=np.uint64)
    pr = np.array(list(protect) or [-2], dtype=np.int32)
    e = ctypes.c_int(-1)
    s = lib().orc_lru_victim(_p(ex), _p(pub), _p(lu), len(slots), _p(pr), len(protect), ctypes.byref(e))
    return None if s < 0 else (e.value, s)


def fill_candidate(slot_experts, hit_counts):
    ex = np.array([-1 if e is None else e for e in slot_experts] or [-1], dtype=np.int32)
    hc = np.array(list(hit_counts) or [0], dtype=np.uint64)
    r = lib().orc_fill_candidate(_p(ex), len(slot_experts), _p(hc), len(hit_counts))
    return None if r < 0 else r


# ---- router / permute / forward --------------------------------------------------------------

def router_logits(x_bf16: np.ndarray, w_bf16: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
    w = np.ascontiguousarray(w_bf16, dtype=np.uint16)
    T, H = x.shape
    E = w.shape[0]
    out = np.empty((T, E), dtype=np.float32)
    lib().orc_router_logits(_p(x), _p(w), T, H, E, _p(out))
    return out


def route(logits: np.ndarray, k: int, mode: int, bias=None, n_group=1, topk_group=1, routed_scale=1.0):
    l = np.ascontiguousarray(logits, dtype=np.float32)
    T, E = l.shape
    ids = np.empty((T, k), dtype=np.uint32)
    w = np.empty((T, k), dtype=np.float32)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float32)
    rc = lib().orc_route(_p(l), None if b is None else _p(b), T, E, k, mode, n_group, topk_group,
                         float(routed_scale), _p(ids), _p(w))
    if rc != 0:
        raise ValueError("orc_route: bad arguments")
    return ids, w


def permute(ids: np.ndarray, E: int):
    a = np.ascontiguousarray(ids, dtype=np.uint32).reshape(-1)
    n = a.size
    counts = np.empty(E, dtype=np.int32)
    offsets = np.empty(E + 1, dtype=np.int32)
    perm = np.empty(max(n, 1), dtype=np.int32)
    active = np.empty(E, dtype=np.int32)
    na = np.zeros(1, dtype=np.int32)
    rc = lib().orc_permute(_p(a), n, E, _p(counts), _p(offsets), _p(perm), _p(active), _p(na))
    if rc != 0:
        raise ValueError("orc_permute: id >= E")
    return counts, offsets, perm[: int(offsets[E])], active[: int(na[0])]


def moe_forward_f32(x, ids, w, gate, up, down):
    """Dequantised reference: gate/up [E, I, H], down [E, H, I] f32; x [T, H] f32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    ids = np.ascontiguousarray(ids, dtype=np.uint32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    gate = np.ascontiguousarray(gate, dtype=np.float32)
    up = np.ascontiguousarray(up, dtype=np.float32)
    down = np.ascontiguousarray(down, dtype=np.float32)
    T, H = x.shape
    k = ids.shape[1]
    E, I = gate.shape[0], gate.shape[1]
    y = np.empty((T, H), dtype=np.float32)
    lib().orc_moe_forward_f32(_p(x), _p(ids), _p(w), T, k, E, H, I, _p(gate), _p(up), _p(down), _p(y))
    return y


def moe_forward_ref(dtype: int, q, x, ids, w, E: int, H: int, I: int, scales=None, threads: int = 0):
    """moe_forward_f32 of the dequantised stacks, from the quantised stacks q = (gate, up, down) and,
    for FP8, their block scales, on `threads` host threads (0: all); x [T, H] f32."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    ids = np.ascontiguousarray(ids, dtype=np.uint32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    T, k = ids.shape
    qs = [np.ascontiguousarray(a).reshape(-1) for a in q]
    sc = [None] * 3 if scales is None else [np.ascontiguousarray(a, dtype=np.float32).reshape(-1) for a in scales]
    y = np.empty((T, H), dtype=np.float32)
    n = threads or (len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count() or 1)
    rc = lib().orc_moe_forward_ref(dtype, _p(qs[0]), _p(qs[1]), _p(qs[2]), None if sc[0] is None else _p(sc[0]),
                                   None if sc[1] is None else _p(sc[1]), None if sc[2] is None else _p(sc[2]),
                                   _p(x), _p(ids), _p(w), T, k, E, H, I, n, _p(y))
    if rc != 0:
        raise ValueError("orc_moe_forward_ref: bad arguments")
    return y


def fused_moe_decode_q8_0(gate_q, up_q, down_q, x, ids, w, E, H, I, threads):
    x = np.ascontiguousarray(x, dtype=np.float32)
    ids = np.ascontiguousarray(ids, dtype=np.uint32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    T, k = ids.shape
    y = np.empty((T, H), dtype=np.float32)
    rc = lib().orc_fused_moe_decode_q8_0(_p(gate_q), _p(up_q), _p(down_q), _p(x), _p(ids), _p(w), T, k, E, H, I,
                                         threads, _p(y))
    if rc != 0:
        raise ValueError("fused decode: bad arguments")
    return y


def baseline_decode_q8_0(gate_q, up_q, down_q, x, ids, w, E, H, I, threads):
    """The timed CPU baseline (cpu_baseline.c): fused_moe_decode_q8_0's result, vectorised, with each
    active expert's weights read once per call."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    ids = np.ascontiguousarray(ids, dtype=np.uint32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    T, k = ids.shape
    y = np.empty((T, H), dtype=np.float32)
    rc = lib().orc_baseline_decode_q8_0(_p(gate_q), _p(up_q), _p(down_q), _p(x), _p(ids), _p(w), T, k, E, H, I,
                                        threads, _p(y))
    if rc != 0:
        raise ValueError("baseline decode: bad arguments")
    return y


# ---- expert parallelism (no reference counterpart: the reference runs on one GPU) -----------------

ID_NONE = 0xFFFFFFFF


def ep_dispatch_plan(ids: np.ndarray, w: np.ndarray, experts_per_rank: int, world: int):
    """Restatement of the library's expert-parallel dispatch plan: every token is sent once to each
    rank owning one of its experts; rows ordered by rank, then token; slot j keeps its position
    (local id and weight where the expert lives on that rank, ID_NONE / 0 elsewhere).
    Returns rank_counts [world], token_rows [T, world] (-1: no row), send_token, send_ids, send_w."""
    ids = np.asarray(ids, dtype=np.uint32)
    w = np.asarray(w, dtype=np.float32)
    T, k = ids.shape
    limit = experts_per_rank * world
    valid = (ids != ID_NONE) & (ids < limit)
    dest = np.where(valid, ids.astype(np.int64) // max(experts_per_rank, 1), -1)
    has = np.zeros((T, world), dtype=bool)
    for j in range(k):
        m = dest[:, j] >= 0
        has[np.nonzero(m)[0], dest[m, j]] = True
    rank_counts = has.sum(0).astype(np.int32)
    starts = np.concatenate([[0], np.cumsum(rank_counts)[:-1]]).astype(np.int64)
    token_rows = np.full((T, world), -1, dtype=np.int32)
    n = int(rank_counts.sum())
    send_token = np.zeros(n, dtype=np.int32)
    send_ids = np.full((n, k), ID_NONE, dtype=np.uint32)
    send_w = np.zeros((n, k), dtype=np.float32)
    for r in range(world):
        toks = np.nonzero(has[:, r])[0]
        rows = starts[r] + np.arange(toks.size)
        token_rows[toks, r] = rows
        send_token[rows] = toks
        mine = dest[toks] == r
        send_ids[rows] = np.where(mine, ids[toks].astype(np.int64) - r * experts_per_rank, ID_NONE).astype(np.uint32)
        send_w[rows] = np.where(mine, w[toks], 0.0)
    return rank_counts, token_rows, send_token, send_ids, send_w


def ep_combine(y_back: np.ndarray, token_rows: np.ndarray, y_add=None) -> np.ndarray:
    """y[t] = y_add[t] + sum over ranks (in order) of y_back[token_rows[t, r]], f32."""
    T, world = token_rows.shape
    H = y_back.shape[1]
    y = np.zeros((T, H), dtype=np.float32) if y_add is None else np.asarray(y_add, dtype=np.float32).copy()
    for r in range(world):
        m = token_rows[:, r] >= 0
        y[m] += np.asarray(y_back, dtype=np.float32)[token_rows[m, r]]
    return y
