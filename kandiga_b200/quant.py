"""MLX-layout affine group quantization on the GPU (torch).

Restates the documented affine scheme of mlx.core.quantize (called by the
reference at scripts/repack_experts_3bit.py:91-94 and scripts/convert_3bit.py:58):
per group of 64 columns, bias = min, scale = (max - min) / (2^bits - 1)
(scale 1 for a constant group), both rounded to the 16-bit storage dtype, then
q = clip(round_half_even((w - bias) / scale), 0, 2^bits - 1).

Packing is the MLX byte layout: 3-bit codes LSB-first in 3-byte packs of 8
(uint8 [rows, cols*3/8], the bytes of MLX's uint32 [rows, cols*3/32]); 4-bit
nibbles LSB-first in uint32 [rows, cols/8].  Used to build synthetic tables on
the device; real checkpoints arrive already packed (BKEX files).
"""
from __future__ import annotations

import torch


def _to_sb(x: torch.Tensor, sb_dtype: str) -> torch.Tensor:
    dt = torch.float16 if sb_dtype == "f16" else torch.bfloat16
    return x.to(dt)


def quantize_affine(w: torch.Tensor, bits: int, group_size: int = 64, sb_dtype: str = "f16"):
    """w [rows, cols] float -> (packed, scales, biases); scales/biases are
    float16 or bfloat16 tensors [rows, cols/group_size]."""
    assert bits in (3, 4) and w.dim() == 2 and w.shape[1] % group_size == 0
    rows, cols = w.shape
    g = w.float().reshape(rows, cols // group_size, group_size)
    mn = g.amin(-1)
    mx = g.amax(-1)
    nb = float((1 << bits) - 1)
    scale = (mx - mn) / nb
    scale = torch.where(scale == 0, torch.ones_like(scale), scale)
    s16 = _to_sb(scale, sb_dtype)
    b16 = _to_sb(mn, sb_dtype)
    s32 = s16.float()
    s32 = torch.where(s32 == 0, torch.ones_like(s32), s32)
    q = torch.clamp(torch.round((g - b16.float()[..., None]) / s32[..., None]), 0, nb)
    q = q.to(torch.int64).reshape(rows, cols)
    return pack_codes(q, bits), s16, b16


def pack_codes(q: torch.Tensor, bits: int) -> torch.Tensor:
    rows, cols = q.shape
    q8 = q.to(torch.int64).reshape(rows, cols // 8, 8)
    shifts = torch.arange(8, device=q.device, dtype=torch.int64) * bits
    word = (q8 << shifts).sum(-1)  # fields do not overlap, so sum == or
    if bits == 4:
        # uint32 bit pattern carried in an int32 tensor
        return torch.where(word >= 2 ** 31, word - 2 ** 32, word).to(torch.int32)
    out = torch.stack([word & 0xFF, (word >> 8) & 0xFF, (word >> 16) & 0xFF], -1).to(torch.uint8)
    return out.reshape(rows, cols * 3 // 8)


def unpack_codes(packed: torch.Tensor, bits: int, cols: int) -> torch.Tensor:
    rows = packed.shape[0]
    if bits == 4:
        w = packed.reshape(rows, cols // 8).view(torch.int32).to(torch.int64) & 0xFFFFFFFF
        shifts = torch.arange(8, device=packed.device, dtype=torch.int64) * 4
        return ((w[..., None] >> shifts) & 15).reshape(rows, cols)
    b = packed.reshape(rows, cols // 8, 3).to(torch.int64)
    w = b[..., 0] | (b[..., 1] << 8) | (b[..., 2] << 16)
    shifts = torch.arange(8, device=packed.device, dtype=torch.int64) * 3
    return ((w[..., None] >> shifts) & 7).reshape(rows, cols)


def dequantize_affine(packed, scales, biases, bits: int, cols: int, group_size: int = 64) -> torch.Tensor:
    q = unpack_codes(packed, bits, cols).float()
    rows = q.shape[0]
    s = scales.float().reshape(rows, cols // group_size, 1)
    b = biases.float().reshape(rows, cols // group_size, 1)
    return (q.reshape(rows, cols // group_size, group_size) * s + b).reshape(rows, cols)
