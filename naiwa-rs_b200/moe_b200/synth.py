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


def q4_k_pack(w: torch.Tensor) -> torch.Tensor:
    """GGML Q4_K of a float tensor whose last dim is a multiple of 256: per 32-weight sub-block a
    min/max fit (scale = (max - min)/15, min <= 0), 6-bit sub-scales/mins against the super-block's
    f16 d = max(scale)/63 and dmin = max(min)/63, 4-bit quants. Returns uint8 [..., K/256*144]."""
    *lead, K = w.shape
    x = w.float().reshape(*lead, K // 256, 8, 32)
    mn = x.amin(-1).clamp(max=0.0)
    mx = x.amax(-1)
    scale = (mx - mn) / 15.0
    minv = -mn
    d = (scale.amax(-1) / 63.0).to(torch.float16)
    dmin = (minv.amax(-1) / 63.0).to(torch.float16)
    df, dmf = d.float().unsqueeze(-1), dmin.float().unsqueeze(-1)
    sc = torch.where(df > 0, torch.round(scale / df.clamp(min=1e-30)), torch.zeros_like(scale)).clamp(0, 63).to(torch.int32)
    m = torch.where(dmf > 0, torch.round(minv / dmf.clamp(min=1e-30)), torch.zeros_like(minv)).clamp(0, 63).to(torch.int32)
    dj = (df * sc.float()).unsqueeze(-1)
    mj = (dmf * m.float()).unsqueeze(-1)
    q = torch.where(dj > 0, torch.round((x + mj) / dj.clamp(min=1e-30)), torch.zeros_like(x)).clamp(0, 15).to(torch.int32)
    out = torch.empty((*lead, K // 256, 144), dtype=torch.uint8, device=w.device)
    out[..., 0:2] = d.view(torch.uint8).reshape(*lead, K // 256, 2)
    out[..., 2:4] = dmin.view(torch.uint8).reshape(*lead, K // 256, 2)
    s0 = sc[..., :4] | ((sc[..., 4:] >> 4) << 6)
    s1 = m[..., :4] | ((m[..., 4:] >> 4) << 6)
    s2 = (sc[..., 4:] & 15) | ((m[..., 4:] & 15) << 4)
    out[..., 4:16] = torch.cat([s0, s1, s2], -1).to(torch.uint8)
    lo = q[..., 0::2, :]  # sub-blocks 2c   -> low nibbles
    hi = q[..., 1::2, :]  # sub-blocks 2c+1 -> high nibbles
    out[..., 16:] = (lo | (hi << 4)).reshape(*lead, K // 256, 128).to(torch.uint8)
    return out.reshape(*lead, K // 256 * 144)


def fp8_b128_pack(w: torch.Tensor):
    """FP8 e4m3 with one f32 scale per 128x128 block of the last two dims (amax/448). Returns
    (uint8 [..., N, K], f32 scales [..., N/128, K/128])."""
    *lead, N, K = w.shape
    blk = w.float().reshape(*lead, N // 128, 128, K // 128, 128)
    amax = blk.abs().amax(dim=(-3, -1), keepdim=True)
    scale = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
    q = (blk / scale).to(torch.float8_e4m3fn).reshape(*lead, N, K)
    return q.view(torch.uint8), scale.reshape(*lead, N // 128, K // 128).contiguous()


def bf16_pack(w: torch.Tensor) -> torch.Tensor:
    return w.to(torch.bfloat16).contiguous().view(torch.uint8).reshape(*w.shape[:-1], w.shape[-1] * 2)


def expert_stacks(E: int, H: int, I: int, wdtype: int, std: float, seed: int, device, with_scales: bool = False):
    """(gate [E, I, H], up [E, I, H], down [E, H, I]) packed in `wdtype`'s GGML layout (flat uint8).
    With with_scales, returns (stacks, scales) where scales are the FP8 block scales (or Nones)."""
    from ._lib import DTYPE_BF16, DTYPE_FP8_E4M3_B128, DTYPE_Q4_K, DTYPE_Q8_0

    g = torch.Generator(device=device)
    g.manual_seed(seed)
    out, scales = [], []
    for shape in ((E, I, H), (E, I, H), (E, H, I)):
        w = torch.randn(shape, generator=g, device=device, dtype=torch.float32).mul_(std)
        sc = None
        if wdtype == DTYPE_Q8_0:
            q = q8_0_pack(w)
        elif wdtype == DTYPE_BF16:
            q = bf16_pack(w)
        elif wdtype == DTYPE_Q4_K:
            q = torch.cat([q4_k_pack(w[e:e + 1]) for e in range(E)])  # per expert: bounded temporaries
        elif wdtype == DTYPE_FP8_E4M3_B128:
            q, sc = fp8_b128_pack(w)
            sc = sc.reshape(-1)
        else:
            raise ValueError(f"synthetic stacks for dtype {wdtype} not built")
        out.append(q.reshape(-1))
        scales.append(sc)
        del w
    return (tuple(out), tuple(scales)) if with_scales else tuple(out)


def router_weight(E: int, H: int, std: float, seed: int, device) -> torch.Tensor:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return torch.randn((E, H), generator=g, device=device, dtype=torch.float32).mul_(std).to(torch.bfloat16)
