"""Seeded synthetic expert stacks for the BASELINE configs, generated on the device.

There are no checkpoints on the box, so benchmarks build random-init layers of the configured
shapes: weights ~ N(0, std) quantised into GGML byte layouts (the stacks a GGUF file would hold,
the bytes the reference slices in src/moe/expert.rs:123-145). torch only generates the numbers
and packs the bytes; the kernels that consume them are the library's.
"""
from __future__ import annotations

import torch

Q8_0_BLOCK_BYTES = 34


def q8_0_pack(w: torch.Tensor) -> torch.Tensor:
    """GGML Q8_0 of a float tensor whose last dim is a multiple of 32: per 32-block d = amax/127
    (stored f16), q = round-half-away(x/d) as int8. Returns uint8 [..., K/32*34]."""
    *lead, K = w.shape
    blocks = w.float().reshape(*lead, K // 32, 32)
    amax = blocks.abs().amax(-1, keepdim=True)
    d = amax / 127.0
    inv = torch.where(d != 0, 1.0 / d, torch.zeros_like(d))
    v = blocks * inv
    q = (torch.sign(v) * torch.floor(v.abs() + 0.5)).clamp_(-128, 127).to(torch.int8)
    out = torch.empty((*lead, K // 32, Q8_0_BLOCK_BYTES), dtype=torch.uint8, device=w.device)
    out[..., :2] = d.to(torch.float16).view(torch.uint8).reshape(*lead, K // 32, 2)
    out[..., 2:] = q.view(torch.uint8)
    return out.reshape(*lead, K // 32 * Q8_0_BLOCK_BYTES)


def bf16_pack(w: torch.Tensor) -> torch.Tensor:
    return w.to(torch.bfloat16).contiguous().view(torch.uint8).reshape(*w.shape[:-1], w.shape[-1] * 2)


def expert_stacks(E: int, H: int, I: int, wdtype: int, std: float, seed: int, device) -> tuple:
    """(gate [E, I, H], up [E, I, H], down [E, H, I]) packed in `wdtype`'s GGML layout (flat uint8)."""
    from ._lib import DTYPE_BF16, DTYPE_Q8_0

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    out = []
    for shape in ((E, I, H), (E, I, H), (E, H, I)):
        w = torch.randn(shape, generator=g, device=device, dtype=torch.float32).mul_(std)
        if wdtype == DTYPE_Q8_0:
            out.append(q8_0_pack(w).reshape(-1))
        elif wdtype == DTYPE_BF16:
            out.append(bf16_pack(w).reshape(-1))
        else:
            raise ValueError(f"synthetic stacks for dtype {wdtype} not built")
        del w
    return tuple(out)


def router_weight(E: int, H: int, std: float, seed: int, device) -> torch.Tensor:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return torch.randn((E, H), generator=g, device=device, dtype=torch.float32).mul_(std).to(torch.bfloat16)
