"""MXFP8 weight packing: quantise once, at load time, on the device.

Format (OCP Microscaling Formats v1.0, MXFP8 with E4M3 elements):
blocks of 32 consecutive weights along the reduction axis (the last axis of
both ``w_gate_up [E, 2I, H]`` and ``w_down [E, H, I]``) share one E8M0 scale.
The shared exponent is ``floor(log2(max|w|)) - 8`` (8 = exponent of the
largest E4M3 normal, 448), elements are ``w / 2^exp`` rounded to nearest-even
E4M3 and saturated at +-448, and the scale byte stores ``exp + 127``.
An all-zero block gets the smallest scale (byte 0).

The kernels consume ``q`` (uint8 bit patterns, same shape as the weights) and
``scale`` (uint8, last axis / 32) directly; see include/warp_decode.h.
"""
from __future__ import annotations

import torch

BLOCK = 32
E4M3_MAX = 448.0


def quantize_mxfp8(w: torch.Tensor, chunk_rows: int = 4096):
    """Quantise along the last axis.  Returns (q uint8, scale uint8)."""
    if w.shape[-1] % BLOCK:
        raise ValueError("last axis must be a multiple of 32")
    shape = w.shape
    flat = w.reshape(-1, shape[-1])
    q = torch.empty(flat.shape, dtype=torch.uint8, device=w.device)
    s = torch.empty(flat.shape[0], shape[-1] // BLOCK, dtype=torch.uint8, device=w.device)
    for r0 in range(0, flat.shape[0], chunk_rows):
        blk = flat[r0:r0 + chunk_rows].float().reshape(-1, shape[-1] // BLOCK, BLOCK)
        amax = blk.abs().amax(dim=-1)
        # floor(log2(amax)) exactly: amax = m * 2^ex with m in [0.5, 1)
        _, ex = torch.frexp(amax)
        e = torch.where(amax > 0, ex.to(torch.int32) - 1 - 8, torch.full_like(ex, -127, dtype=torch.int32))
        e = e.clamp(-127, 127)
        scaled = torch.ldexp(blk, (-e).to(torch.float32)[..., None])
        scaled = scaled.clamp(-E4M3_MAX, E4M3_MAX)
        q[r0:r0 + chunk_rows] = scaled.to(torch.float8_e4m3fn).view(torch.uint8).reshape(-1, shape[-1])
        s[r0:r0 + chunk_rows] = (e + 127).to(torch.uint8)
    return q.reshape(shape), s.reshape(*shape[:-1], shape[-1] // BLOCK)


def dequantize_mxfp8(q: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """float32 weights: e4m3(q) * 2^(scale - 127) per block of 32."""
    vals = q.view(torch.float8_e4m3fn).float()
    shape = vals.shape
    blk = vals.reshape(*shape[:-1], shape[-1] // BLOCK, BLOCK)
    out = torch.ldexp(blk, (scale.to(torch.float32) - 127.0)[..., None])
    return out.reshape(shape)
