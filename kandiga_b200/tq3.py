"""TQ3_1S dense layers on the GPU.

Python mirror of kandiga/tq3 (quantize.py, engine.py, fused_kernel.py):

* ``quantize_tensor(weights) -> (bytes, shape, num_blocks)`` -- the TQ3_1S
  quantizer (kandiga/tq3/quantize.py:390-461): per 32-weight block,
  r = WHT(S . w) / sqrt(32); per half of 16: mean, RMS, a grid search over
  nine scale multipliers and six least-squares refinements on the 3-bit
  Lloyd-Max codebook; 20-byte blocks (fp16 d0 d1 m0 m1, 12 bytes of indices).
  Offline: runs in float64 torch (CPU or GPU), the precision the reference
  reaches under numpy 2 promotion.
* ``dequantize_tensor(data, shape, num_blocks)`` -- reconstruction on the GPU
  (kq_tq3_dequant), numpy fp32 out as in kandiga/tq3/quantize.py:483-516.
* ``TQ3Linear`` -- same constructor, ``forward``/``__call__``, ``save``/``load``
  (the "TQ31" file, kandiga/tq3/engine.py:83-116), ``from_linear``,
  ``memory_bytes``, ``compression_ratio``; ``forward`` runs kq_tq3_gemv on the
  block stream resident in HBM instead of dequantizing the whole matrix.
* ``tq3_gemv(x, layer)`` -- the fused GEMV entry point.
"""
from __future__ import annotations

import ctypes
import os
import struct
from typing import Optional, Tuple

import numpy as np
import torch

from . import _native as N

# kandiga/tq3/quantize.py:29-47
CENTROIDS = (-1.996684, -1.291398, -0.740341, -0.247508, 0.230106, 0.725222, 1.277503, 1.988943)
BOUNDARIES = (-1.644041, -1.015870, -0.493924, -0.008701, 0.477664, 1.001362, 1.633223)
SIGNS = (+1, -1, +1, -1, +1, +1, -1, +1, -1, -1, +1, -1, +1, +1, -1, +1,
         -1, -1, +1, -1, +1, -1, -1, +1, -1, +1, +1, -1, +1, -1, -1, +1)
BLOCK_BYTES = 20
_MULTS = (0.60, 0.70, 0.80, 0.90, 1.00, 1.10, 1.20, 1.35, 1.50)
_DT = {torch.float16: N.DT_F16, torch.bfloat16: N.DT_BF16, torch.float32: N.DT_F32}


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _butterfly32(a: torch.Tensor) -> torch.Tensor:
    """Unnormalised Walsh-Hadamard butterfly over the last axis (32), stages 1, 2, 4, 8, 16."""
    out = a.clone()
    step = 1
    while step < 32:
        v = out.reshape(*out.shape[:-1], 32 // (2 * step), 2, step)
        lo, hi = v[..., 0, :].clone(), v[..., 1, :].clone()
        v[..., 0, :] = lo + hi
        v[..., 1, :] = lo - hi
        out = v.reshape(out.shape)
        step *= 2
    return out


_EDGES = tuple(float(np.float32(b)) for b in BOUNDARIES)  # the stored fp32 boundaries


def _index(v: torch.Tensor) -> torch.Tensor:
    idx = torch.zeros(v.shape, dtype=torch.int64, device=v.device)
    for b, edge in enumerate(_EDGES):
        idx[v > edge] = b + 1
    return idx


def _refine(halves, rms, means, cent):
    """Scale per half-block: best of the multiplier grid, then six least-squares steps."""
    centered = halves - means[:, None]
    best_s = rms.clone()
    best_e = torch.full_like(rms, float("inf"))

    def err(s):
        idx = _index(centered * (1.0 / s)[:, None])
        return ((halves - (cent[idx] * s[:, None] + means[:, None])) ** 2).sum(1)

    for mult in _MULTS:
        s = torch.clamp(rms * mult, min=1e-10)
        e = err(s)
        better = e < best_e
        best_e = torch.where(better, e, best_e)
        best_s = torch.where(better, s, best_s)
    s = best_s.clone()
    for _ in range(6):
        idx = _index(centered * (1.0 / torch.clamp(s, min=1e-10))[:, None])
        c = cent[idx]
        num = (centered * c).sum(1)
        den = (c ** 2).sum(1)
        ns = torch.where(den > 1e-12, num / torch.where(den > 1e-12, den, torch.ones_like(den)), s)
        ns = torch.clamp(ns, min=1e-10)
        e = ((halves - (c * ns[:, None] + means[:, None])) ** 2).sum(1)
        better = e < best_e
        best_e = torch.where(better, e, best_e)
        best_s = torch.where(better, ns, best_s)
        s = ns
    return best_s


def _pack(idx: torch.Tensor) -> torch.Tensor:
    """[n, 32] indices -> [n, 12] bytes: four little-endian 24-bit groups of eight."""
    g = idx.reshape(-1, 4, 8)
    word = torch.zeros(g.shape[:2], dtype=torch.int64, device=idx.device)
    for r in range(8):
        word |= g[:, :, r] << (3 * r)
    return torch.stack([word & 0xFF, (word >> 8) & 0xFF, (word >> 16) & 0xFF], -1).reshape(-1, 12).to(torch.uint8)


def quantize_tensor(weights, device=None) -> tuple:
    """weights (numpy or torch, any shape) -> (block bytes, shape, num_blocks)."""
    w = torch.as_tensor(np.asarray(weights, np.float32) if not torch.is_tensor(weights) else weights)
    shape = tuple(w.shape)
    dev = torch.device(device) if device is not None else w.device
    flat = w.reshape(-1).to(dev, torch.float32)
    pad = (32 - flat.numel() % 32) % 32
    if pad:
        flat = torch.cat([flat, torch.zeros(pad, dtype=torch.float32, device=dev)])
    nb = flat.numel() // 32
    signs = torch.tensor(SIGNS, dtype=torch.float32, device=dev)
    rot = _butterfly32(flat.reshape(nb, 32) * signs).double() / float(np.sqrt(32.0))
    h0, h1 = rot[:, :16], rot[:, 16:]
    m0, m1 = h0.mean(1), h1.mean(1)
    r0 = torch.sqrt(((h0 - m0[:, None]) ** 2).mean(1))
    r1 = torch.sqrt(((h1 - m1[:, None]) ** 2).mean(1))
    r0 = torch.where(r0 < 1e-10, torch.ones_like(r0), r0)
    r1 = torch.where(r1 < 1e-10, torch.ones_like(r1), r1)
    cent = torch.tensor(np.array(CENTROIDS, np.float32).astype(np.float64), device=dev)  # fp32 codebook values
    d0 = _refine(h0, r0, m0, cent)
    d1 = _refine(h1, r1, m1, cent)
    idx = torch.cat([_index((h0 - m0[:, None]) / torch.clamp(d0, min=1e-10)[:, None]),
                     _index((h1 - m1[:, None]) / torch.clamp(d1, min=1e-10)[:, None])], 1)
    lim = 65504.0
    hdr = torch.stack([d0.clamp(-lim, lim), d1.clamp(-lim, lim), m0.clamp(-lim, lim), m1.clamp(-lim, lim)], 1)
    hdr = hdr.cpu().numpy().astype(np.float16)
    blocks = np.concatenate([hdr.view(np.uint8).reshape(nb, 8), _pack(idx).cpu().numpy()], 1)
    return blocks.tobytes(), shape, nb


class TQ3Matrix:
    """A TQ3_1S block stream resident in HBM (kq_tq3_mat)."""

    def __init__(self, data: bytes, rows: int, cols: int, block_bytes: int = BLOCK_BYTES):
        self.lib = N.load()
        self.rows, self.cols, self.block_bytes = rows, cols, block_bytes
        buf = np.frombuffer(data, np.uint8)
        h = ctypes.c_void_p()
        N.check(self.lib.kq_tq3_create(rows, cols, block_bytes, buf.ctypes.data_as(ctypes.c_void_p), buf.nbytes,
                                       ctypes.byref(h)), "kq_tq3_create")
        self.h = h

    def __del__(self):
        h = getattr(self, "h", None)
        if h:
            try:
                self.lib.kq_tq3_destroy(h)
            except Exception:
                pass
            self.h = None

    def gemv(self, x: torch.Tensor, bias: Optional[torch.Tensor] = None, out_dtype=torch.float32):
        if not x.is_cuda or x.shape[-1] != self.cols:
            raise ValueError(f"x must be a CUDA tensor [..., {self.cols}]")
        lead = x.shape[:-1]
        dt = x.dtype if x.dtype in _DT else torch.float32
        xf = x.to(dt).reshape(-1, self.cols).contiguous()
        y = torch.empty(xf.shape[0], self.rows, dtype=out_dtype, device=x.device)
        b = bias.to(torch.float32).contiguous() if bias is not None else None
        N.check(self.lib.kq_tq3_gemv(self.h, ctypes.c_void_p(xf.data_ptr()), _DT[dt], xf.shape[0],
                                     ctypes.c_void_p(b.data_ptr()) if b is not None else None,
                                     ctypes.c_void_p(y.data_ptr()), _DT[out_dtype], _stream()), "kq_tq3_gemv")
        return y.reshape(*lead, self.rows)

    def dequant(self) -> torch.Tensor:
        w = torch.empty(self.rows, self.cols, dtype=torch.float32, device="cuda")
        N.check(self.lib.kq_tq3_dequant(self.h, ctypes.c_void_p(w.data_ptr()), _stream()), "kq_tq3_dequant")
        return w


def dequantize_tensor(blocks_data: bytes, shape: tuple, num_blocks: int) -> np.ndarray:
    """Reconstructed weights (numpy fp32, `shape`), computed on the GPU."""
    bb = len(blocks_data) // num_blocks
    m = TQ3Matrix(blocks_data, 1, num_blocks * 32, bb)
    w = m.dequant().reshape(-1)[: int(np.prod(shape))].cpu().numpy()
    return w.reshape(shape)


class TQ3Linear:
    """Linear layer with TQ3_1S weights [out_features, in_features] (in % 32 == 0)."""

    def __init__(self, weight_data: bytes, shape: Tuple[int, ...], num_blocks: int,
                 bias: Optional[np.ndarray] = None):
        self.weight_data = weight_data
        self.shape = tuple(shape)
        self.num_blocks = num_blocks
        self.bias = bias
        self._mat = None
        self._bias_dev = None

    def _ensure(self):
        if self._mat is None:
            if len(self.shape) != 2 or self.shape[1] % 32:
                raise ValueError("TQ3Linear on the GPU needs a 2-D weight with in_features % 32 == 0")
            bb = len(self.weight_data) // self.num_blocks
            self._mat = TQ3Matrix(self.weight_data, self.shape[0], self.shape[1], bb)
            if self.bias is not None:
                self._bias_dev = torch.as_tensor(np.asarray(self.bias, np.float32)).cuda()
        return self._mat

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """x @ W^T + bias (fp32 out), x a CUDA tensor [..., in_features]."""
        return self._ensure().gemv(x, self._bias_dev)

    def __call__(self, x):
        return self.forward(x)

    def save(self, path: str):
        os.makedirs(os.path.dirname(path) or ".", exist_ok=True)
        with open(path, "wb") as f:
            f.write(b"TQ31")
            f.write(struct.pack("<I", len(self.shape)))
            for s in self.shape:
                f.write(struct.pack("<I", s))
            f.write(struct.pack("<I", self.num_blocks))
            f.write(struct.pack("<B", 1 if self.bias is not None else 0))
            if self.bias is not None:
                f.write(np.asarray(self.bias).astype(np.float16).tobytes())
            f.write(self.weight_data)

    @classmethod
    def load(cls, path: str) -> "TQ3Linear":
        with open(path, "rb") as f:
            magic = f.read(4)
            if magic != b"TQ31":
                raise ValueError(f"Invalid TQ3 file: {magic}")
            ndims = struct.unpack("<I", f.read(4))[0]
            shape = tuple(struct.unpack("<I", f.read(4))[0] for _ in range(ndims))
            num_blocks = struct.unpack("<I", f.read(4))[0]
            has_bias = struct.unpack("<B", f.read(1))[0]
            bias = None
            if has_bias:
                bias = np.frombuffer(f.read(shape[0] * 2), dtype=np.float16).astype(np.float32)
            weight_data = f.read()
        return cls(weight_data, shape, num_blocks, bias)

    @classmethod
    def from_linear(cls, weight, bias: Optional[np.ndarray] = None) -> "TQ3Linear":
        data, shape, num_blocks = quantize_tensor(weight)
        return cls(data, shape, num_blocks, bias)

    @property
    def memory_bytes(self) -> int:
        return len(self.weight_data) + (np.asarray(self.bias).nbytes if self.bias is not None else 0)

    @property
    def compression_ratio(self) -> float:
        original = 2
        for s in self.shape:
            original *= s
        return original / self.memory_bytes


def tq3_gemv(x: torch.Tensor, layer: TQ3Linear) -> torch.Tensor:
    """Fused TQ3 GEMV y = x @ W^T (kandiga/tq3/fused_kernel.py:289-341)."""
    return layer.forward(x)
