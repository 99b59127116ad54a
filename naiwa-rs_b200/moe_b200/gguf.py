"""GGUF model files as the source of a layer's expert stacks (moe_gguf_* in libmoe_b200.so).

The reference loads its model from GGUF shards (src/load.rs:414-450) and hands the provider each MoE
block's stacked expert tensors blk.{L}.ffn_{gate,up,down}_exps.weight ([E, N, K] GGML QTensors,
provider.rs:367; sliced per expert by expert.rs:123-145). `GGUFFile` maps such a file through the
library's native reader and builds the `ExpertLoadContext` of one layer with its stacks pointing
into the mapping (zero copy; the layer copies them into HBM at build time).
"""
from __future__ import annotations

import ctypes
from typing import Optional

import numpy as np

from ._lib import LayerDesc, MoeError, check, lib
from .layer import ExpertLoadContext, MoeConfig

GGML_F32, GGML_F16, GGML_Q8_0, GGML_Q4_K, GGML_BF16 = 0, 1, 8, 12, 30


def _view(ptr: int, nbytes: int) -> np.ndarray:
    """A uint8 numpy view of `nbytes` at `ptr` (no copy)."""
    return np.ctypeslib.as_array((ctypes.c_uint8 * nbytes).from_address(ptr))


class GGUFFile:
    def __init__(self, path: str):
        h = ctypes.c_void_p()
        check(lib().moe_gguf_open(path.encode(), ctypes.byref(h)))
        self._h = h
        self.path = path

    def close(self):
        if getattr(self, "_h", None) is not None and self._h.value:
            lib().moe_gguf_close(self._h)
            self._h = ctypes.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def tensor_names(self) -> list[str]:
        L = lib()
        return [L.moe_gguf_tensor_name(self._h, i).decode() for i in range(L.moe_gguf_tensor_count(self._h))]

    def tensor(self, name: str):
        """(ggml type, dims with dims[0] fastest, uint8 view of its bytes or None when its size is unknown)."""
        t, nd = ctypes.c_int(), ctypes.c_int()
        dims = (ctypes.c_int64 * 4)()
        data, nbytes = ctypes.c_void_p(), ctypes.c_int64()
        check(lib().moe_gguf_tensor(self._h, name.encode(), ctypes.byref(t), dims, ctypes.byref(nd),
                                    ctypes.byref(data), ctypes.byref(nbytes)))
        view = _view(data.value, nbytes.value) if nbytes.value >= 0 else None
        return t.value, tuple(int(d) for d in dims[:nd.value]), view

    def get_int(self, key: str) -> Optional[int]:
        v = ctypes.c_int64()
        return int(v.value) if lib().moe_gguf_get_int(self._h, key.encode(), ctypes.byref(v)) == 0 else None

    def get_str(self, key: str) -> Optional[str]:
        n = int(lib().moe_gguf_get_str(self._h, key.encode(), None, 0))
        if n == 0:
            return None
        buf = ctypes.create_string_buffer(n + 1)
        lib().moe_gguf_get_str(self._h, key.encode(), buf, n + 1)
        return buf.value.decode()

    def layer_context(self, layer: int, device: int, max_tokens: int = 256, top_k: Optional[int] = None,
                      router_mode: Optional[int] = None, cache_slots: int = 0, **config) -> ExpertLoadContext:
        """The ExpertLoadContext of MoE layer `layer`: shapes, weight format and (when the file has them)
        top-k and router from the file; `top_k` / `router_mode` / further MoeConfig fields override."""
        from . import _lib

        d = LayerDesc()
        d.top_k = 0
        check(lib().moe_gguf_layer_desc(self._h, int(layer), ctypes.byref(d)))
        k = top_k or d.top_k
        if k <= 0:
            raise MoeError(_lib.MOE_ERR_INVALID, "GGUFFile.layer_context: the file states no expert_used_count; "
                                                  "pass top_k")
        E, H, I = d.num_experts, d.hidden, d.inter
        per = {_lib.DTYPE_Q8_0: (32, 34), _lib.DTYPE_Q4_K: (256, 144), _lib.DTYPE_BF16: (1, 2)}[d.wdtype]
        gu_bytes = E * I * (H // per[0]) * per[1]
        dn_bytes = E * H * (I // per[0]) * per[1]
        router = None
        if d.router_weight:
            router = _view(d.router_weight, E * H * 2).view(np.uint16).reshape(E, H)
        cfg = MoeConfig(num_experts=E, num_experts_per_tok=k, hidden_size=H, moe_intermediate_size=I, **config)
        if router_mode is not None:
            cfg.router_mode = router_mode
        ctx = ExpertLoadContext(layer=int(layer), device=device, config=cfg, wdtype=d.wdtype,
                                gate=_view(d.gate, gu_bytes), up=_view(d.up, gu_bytes), down=_view(d.down, dn_bytes),
                                router_weight=router, max_tokens=max_tokens, cache_slots=cache_slots)
        ctx._keep.append(self)  # the mapping stays open while the context lives
        return ctx
