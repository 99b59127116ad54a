"""Routed experts on the host CPU and the executor that hands their results to the device.

Reference: CpuExperts::forward (naiwa-rs src/moe/expert.rs:59-117), the miss stage's fused decode
(src/moe/stages/cpu_miss.rs:21-54) and the result executor (src/executor.rs:116-166). The compute is
the library's (moe_cpu_forward, std::threads); results travel back through a doorbell Ring.
"""
from __future__ import annotations

import ctypes

import numpy as np

from ._lib import LayerDesc, check, lib
from .layer import _ptr, _stream


def _np_ptr(a):
    return ctypes.c_void_p(a.ctypes.data) if a is not None else None


def cpu_isa() -> str:
    """The instruction set of the CPU expert path's row dot products on this host (moe_cpu_isa)."""
    return lib().moe_cpu_isa().decode()


class CpuExperts:
    """Host copy of a layer's Q8_0 / BF16 stacks (numpy uint8, GGML layout) and the CPU expert path."""

    def __init__(self, num_experts: int, top_k: int, hidden: int, inter: int, wdtype: int, gate, up, down,
                 threads: int = 0):
        self._keep = [np.ascontiguousarray(a) for a in (gate, up, down)]
        d = LayerDesc()
        d.num_experts, d.top_k, d.hidden, d.inter, d.wdtype = num_experts, top_k, hidden, inter, wdtype
        d.gate, d.up, d.down = (a.ctypes.data for a in self._keep)
        d.max_tokens = 1
        h = ctypes.c_void_p()
        check(lib().moe_cpu_experts_create(ctypes.byref(d), int(threads), ctypes.byref(h)))
        self._h = h
        self._keep = None  # the library copied the stacks
        self.hidden = hidden

    def forward(self, x_bf16: np.ndarray, ids: np.ndarray, weights: np.ndarray, select=None) -> np.ndarray:
        """x_bf16 [T, H] uint16 (bf16 bits); ids/weights [T, width]; select [T*width] (nonzero: compute)."""
        x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        w = np.ascontiguousarray(weights, dtype=np.float32)
        T, width = ids.shape
        sel = None if select is None else np.ascontiguousarray(select, dtype=np.uint8)
        y = np.empty((T, self.hidden), np.float32)
        check(lib().moe_cpu_forward(self._h, _np_ptr(x), _np_ptr(ids), _np_ptr(w), T, width, _np_ptr(sel), _np_ptr(y)))
        return y

    def close(self):
        if getattr(self, "_h", None) is not None and self._h.value:
            lib().moe_cpu_experts_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Executor:
    """FIFO CPU jobs on a worker thread; each result lands in the next slot of `ring` (host -> device)."""

    def __init__(self, cpu: CpuExperts, ring):
        h = ctypes.c_void_p()
        check(lib().moe_executor_create(cpu._h, ring._h, ctypes.byref(h)))
        self._h = h
        self.cpu = cpu
        self.ring = ring

    def submit(self, x_bf16: np.ndarray, ids: np.ndarray, weights: np.ndarray, select=None) -> int:
        x = np.ascontiguousarray(x_bf16, dtype=np.uint16)
        ids = np.ascontiguousarray(ids, dtype=np.uint32)
        w = np.ascontiguousarray(weights, dtype=np.float32)
        T, width = ids.shape
        sel = None if select is None else np.ascontiguousarray(select, dtype=np.uint8)
        target = ctypes.c_uint32()
        check(lib().moe_executor_submit(self._h, _np_ptr(x), _np_ptr(ids), _np_ptr(w), T, width, _np_ptr(sel),
                                        ctypes.byref(target)))
        return int(target.value)

    def drain(self):
        check(lib().moe_executor_drain(self._h))

    def close(self):
        if getattr(self, "_h", None) is not None and self._h.value:
            lib().moe_executor_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def add_f32_into_bf16(y, add, stream=None):
    """y (bf16, CUDA) += add (f32, CUDA), rounded once."""
    check(lib().moe_add_f32_into_bf16(_ptr(y), _ptr(add), y.numel(), ctypes.c_void_p(_stream(stream))))
    return y
