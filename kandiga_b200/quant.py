"""MLX-layout affine group quantization on the GPU (torch).

Restates the published affine quantizer of mlx.core.quantize (called by the
reference at scripts/repack_experts_3bit.py:91-94 and scripts/convert_3bit.py:58).
Per group of 64 columns, in fp32: scale = max((max - min) / (2^bits - 1), 1e-7),
negated unless |min| > |max|; edge = the end of larger magnitude; q0 =
round_half_even(edge / scale); where q0 != 0, scale = edge / q0 and bias = edge
(else bias 0), so that edge, and zero, are exactly representable; codes
q = clip(round_half_even((w - bias) / scale), 0, 2^bits - 1) from those fp32
values, then scale and bias rounded to the 16-bit storage dtype (mode "edge").
Mode "minmax" is the older formula: bias = min, scale = (max - min) /
(2^bits - 1) (1 for a constant group), both rounded first, codes from the
rounded values.

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


def quantize_affine(w: torch.Tensor, bits: int, group_size: int = 64, sb_dtype: str = "f16", mode: str = "edge"):
    """w [rows, cols] float -> (packed, scales, biases); scales/biases are
    float16 or bfloat16 tensors [rows, cols/group_size]."""
    assert bits in (3, 4) and w.dim() == 2 and w.shape[1] % group_size == 0 and mode in ("edge", "minmax")
    rows, cols = w.shape
    g = w.float().reshape(rows, cols // group_size, group_size)
    mn = g.amin(-1)
    mx = g.amax(-1)
    nb = float((1 << bits) - 1)
    if mode == "edge":
        scale = torch.clamp_min((mx - mn) / nb, 1e-7)
        side = mn.abs() > mx.abs()
        scale = torch.where(side, scale, -scale)
        edge = torch.where(side, mn, mx)
        q0 = torch.round(edge / scale)
        nz = q0 != 0
        scale = torch.where(nz, edge / torch.where(nz, q0, torch.ones_like(q0)), scale)
        bias = torch.where(nz, edge, torch.zeros_like(edge))
        q = torch.clamp(torch.round((g - bias[..., None]) / scale[..., None]), 0, nb)
        return pack_codes(q.to(torch.int64).reshape(rows, cols), bits), _to_sb(scale, sb_dtype), _to_sb(bias, sb_dtype)
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
