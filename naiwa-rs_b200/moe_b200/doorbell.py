"""Host <-> device hand-off rings over mapped pinned memory (libmoe_b200's moe_ring_*).

Reference: naiwa-rs src/doorbell (doorbell.cu:15-149, mapped.rs:18-141, payload_ring.rs:14-81,
d2h/topk.rs:20-125, h2d/result.rs:27-123). A ring has `depth` slots; slot numbers start at 1.
Device waits are bounded (about a second) and report through `check()`; host waits take a timeout.
"""
from __future__ import annotations

import ctypes

from ._lib import check, lib
from .layer import _ptr, _stream


class Ring:
    def __init__(self, device: int, depth: int, slot_bytes: int):
        h = ctypes.c_void_p()
        check(lib().moe_ring_create(device, depth, slot_bytes, ctypes.byref(h)))
        self._h = h

    @property
    def slot_bytes(self) -> int:
        return int(lib().moe_ring_slot_bytes(self._h))

    def publish_from_device(self, src0, src1=None, stream=None) -> int:
        """Enqueue: copy device tensors src0 (++ src1) into the next slot; returns its number."""
        seq = ctypes.c_uint32()
        n0 = src0.numel() * src0.element_size()
        n1 = 0 if src1 is None else src1.numel() * src1.element_size()
        check(lib().moe_ring_publish_from_device(self._h, _ptr(src0), n0, _ptr(src1), n1,
                                                 ctypes.c_void_p(_stream(stream)), ctypes.byref(seq)))
        return int(seq.value)

    def host_take(self, target: int, dst, timeout_us: int = 5_000_000):
        """Wait for slot `target` on this thread and copy it into dst (a CPU tensor or numpy array)."""
        n = dst.nbytes if hasattr(dst, "nbytes") else dst.numel() * dst.element_size()
        ptr = dst.ctypes.data if hasattr(dst, "ctypes") else dst.data_ptr()
        check(lib().moe_ring_host_take(self._h, target, ctypes.c_void_p(ptr), n, timeout_us))
        return dst

    def host_publish(self, src, timeout_us: int = 5_000_000) -> int:
        """Copy a host buffer (numpy array or CPU tensor) into the next slot and publish it."""
        n = src.nbytes if hasattr(src, "nbytes") else src.numel() * src.element_size()
        ptr = src.ctypes.data if hasattr(src, "ctypes") else src.data_ptr()
        seq = ctypes.c_uint32()
        check(lib().moe_ring_host_publish(self._h, ctypes.c_void_p(ptr), n, timeout_us, ctypes.byref(seq)))
        return int(seq.value)

    def device_take(self, target: int, dst, stream=None):
        """Enqueue: wait (bounded) for slot `target` and copy it into the device tensor dst."""
        check(lib().moe_ring_device_take(self._h, target, _ptr(dst), dst.numel() * dst.element_size(),
                                         ctypes.c_void_p(_stream(stream))))
        return dst

    def check(self, stream=None):
        check(lib().moe_ring_check(self._h, ctypes.c_void_p(_stream(stream))))

    def counters(self):
        s, c = ctypes.c_uint32(), ctypes.c_uint32()
        lib().moe_ring_counters(self._h, ctypes.byref(s), ctypes.byref(c))
        return int(s.value), int(c.value)

    def close(self):
        if self._h:
            lib().moe_ring_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
