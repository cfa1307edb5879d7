"""CPU oracle for the quantized routed-expert path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
legs may import this module, and only as the checker.  The product package
(kandiga_b200) never imports it.

Contents (each restates a reference function; paths are relative to the kandiga
project root):

* C oracle via ctypes (oracle/kq_oracle.c): unpack, affine matvec, expert MLP,
  MoE layer, router top-K, combine.  Pinned bit-for-bit against the
  reference's own scalar C (oracle/_ref, built by oracle/build_ref.py).
* ``quantize_affine``: MLX's affine group quantizer (group 64; the edge
  selection that makes zero exactly representable, and the older min/max
  formula as a mode), restating the published algorithm of mlx.core.quantize
  as called at scripts/repack_experts_3bit.py:91-94 and scripts/convert_3bit.py:52-70.
  MLX is not installed here: quantizer parity is UNPINNED.  Kernel parity does
  not depend on it (kernels and oracle consume the same codes/scales/biases).
* ``TurboQuantRef``: kandiga/kv_compress.py:30-118 op for op in numpy float32.
  Pinned against fixtures made by running the reference module itself on a
  numpy-backed stand-in for mlx.core (tests/golden/make_golden.py).
* TQ3: kandiga/tq3/quantize.py:52-118,390-516 restated with vectorised numpy.
  Pinned against fixtures made by importing the reference module.
* BKEX: kandiga/_pack_experts.py:95-132 header, parsed the way
  kandiga/metal/kandiga_cpu_expert_lg.m:67-117 parses it.
"""
from __future__ import annotations

import ctypes
import math
import os
import struct

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None
_REF = {}

_f32p = ctypes.POINTER(ctypes.c_float)
_i32p = ctypes.POINTER(ctypes.c_int32)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_u8p = ctypes.POINTER(ctypes.c_uint8)


def _p(a, t=ctypes.c_void_p):
    return a.ctypes.data_as(t)


def lib():
    """Load (building if needed) the C oracle."""
    global _LIB
    if _LIB is None:
        from oracle.build import build
        path = build()
        L = ctypes.CDLL(path)
        L.kqo_code3.argtypes = [_u8p, ctypes.c_int]
        L.kqo_code3.restype = ctypes.c_int
        L.kqo_unpack3.argtypes = [_u8p, ctypes.c_int, _u8p]
        L.kqo_unpack4.argtypes = [ctypes.c_void_p, ctypes.c_int, _u8p]
        L.kqo_pack3.argtypes = [_u8p, ctypes.c_int, _u8p]
        L.kqo_pack4.argtypes = [_u8p, ctypes.c_int, ctypes.c_void_p]
        L.kqo_matvec.argtypes = [ctypes.c_int, ctypes.c_void_p, _u16p, _u16p, ctypes.c_int, _f32p,
                                 _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.kqo_moe_layer.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                    ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_int64),
                                    ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p),
                                    ctypes.POINTER(ctypes.c_int64), _f32p, _i32p, ctypes.c_int,
                                    ctypes.c_int, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                    ctypes.c_int]
        L.kqo_router_topk.argtypes = [_f32p, ctypes.c_int, ctypes.c_int, ctypes.c_int, _i32p, _f32p]
        L.kqo_combine.argtypes = [_f32p, _f32p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                  ctypes.c_int, ctypes.c_int, ctypes.c_int, _f32p]
        L.kqo_f32_to_f16.argtypes = [_f32p, _u16p, ctypes.c_long]
        _LIB = L
    return _LIB


def ref_lib(variant: str = "small"):
    """The reference's own scalar C (compiled by oracle/build_ref.py), or None if not built."""
    if variant in _REF:
        return _REF[variant]
    name = {"small": "libref_expert.so", "lg": "libref_expert_lg.so"}[variant]
    path = os.path.join(HERE, "_ref", name)
    if not os.path.exists(path):
        _REF[variant] = None
        return None
    L = ctypes.CDLL(path)
    if variant == "small":
        L.ref_expert_size.argtypes = [ctypes.c_int]
        L.ref_matvec3.argtypes = [ctypes.c_void_p, _u16p, _u16p, _f32p, _f32p, ctypes.c_int, ctypes.c_int]
        L.ref_matvec4.argtypes = [ctypes.c_void_p, _u16p, _u16p, _f32p, _f32p, ctypes.c_int, ctypes.c_int]
        L.ref_expert.argtypes = [ctypes.c_int, ctypes.c_void_p, _f32p, _f32p]
        L.ref_moe_layer.argtypes = [ctypes.c_int, ctypes.c_void_p, _f32p, _i32p, ctypes.c_int,
                                    ctypes.c_int, _f32p, ctypes.c_int]
    else:
        L.ref_lg_expert.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                    ctypes.POINTER(ctypes.c_size_t), ctypes.c_void_p, _f32p, _f32p]
    _REF[variant] = L
    return L


# ---------------------------------------------------------------------------
# 16-bit float helpers
# ---------------------------------------------------------------------------

def bf16_bits_to_f32(u16: np.ndarray) -> np.ndarray:
    return (u16.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(f: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns."""
    u = np.ascontiguousarray(f, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return rounded.astype(np.uint16)


def sb_to_f32(u16: np.ndarray, sb_dtype: str) -> np.ndarray:
    if sb_dtype == "bf16":
        return bf16_bits_to_f32(u16)
    return u16.view(np.float16).astype(np.float32)


def f32_to_sb(f: np.ndarray, sb_dtype: str) -> np.ndarray:
    if sb_dtype == "bf16":
        return f32_to_bf16_bits(f)
    return np.asarray(f, dtype=np.float32).astype(np.float16).view(np.uint16)


# ---------------------------------------------------------------------------
# MLX-layout affine quantizer (parity unpinned: MLX is not installed)
# ---------------------------------------------------------------------------

def quantize_affine(w: np.ndarray, bits: int, gs: int = 64, sb_dtype: str = "f16", mode: str = "edge"):
    """w [rows, cols] fp32 -> (packed, scales_u16, biases_u16), MLX layout.

    mode "edge" restates the published affine quantizer of MLX
    (mlx.core.quantize, mode "affine"; the call sites are
    scripts/repack_experts_3bit.py:91-94 and scripts/convert_3bit.py:52-70).
    Per group of `gs` columns, in fp32:
      scale = max((max - min) / (2^bits - 1), 1e-7), negated unless |min| > |max|;
      edge  = min if |min| > |max| else max;
      q0    = round_half_even(edge / scale);
      scale = edge / q0 and bias = edge when q0 != 0 (else scale kept, bias 0),
    so the edge of larger magnitude, and zero with it, are exactly
    representable; codes q = clip(round_half_even((w - bias) / scale), 0,
    2^bits - 1) use those fp32 values, and the scale and bias are then rounded
    to the storage dtype.  Scales are negative for groups whose max has the
    larger magnitude.
    mode "minmax": the older formula (bias = min, scale = (max - min) /
    (2^bits - 1), 1 for a constant group; both rounded to the storage dtype
    first, and q from the rounded values).
    packed is uint8 [rows, cols*3/8] for 3-bit and uint32 [rows, cols/8] for 4-bit.
    """
    rows, cols = w.shape
    assert cols % gs == 0 and mode in ("edge", "minmax")
    g = w.reshape(rows, cols // gs, gs).astype(np.float32)
    mn = g.min(-1)
    mx = g.max(-1)
    nb = np.float32((1 << bits) - 1)
    if mode == "edge":
        with np.errstate(divide="ignore", invalid="ignore"):
            scale = np.maximum((mx - mn) / nb, np.float32(1e-7)).astype(np.float32)
            side = np.abs(mn) > np.abs(mx)
            scale = np.where(side, scale, -scale).astype(np.float32)
            edge = np.where(side, mn, mx).astype(np.float32)
            q0 = np.round(edge / scale).astype(np.float32)
            nz = q0 != 0
            scale = np.where(nz, edge / np.where(nz, q0, np.float32(1)), scale).astype(np.float32)
            bias = np.where(nz, edge, np.float32(0)).astype(np.float32)
            q = np.clip(np.round((g - bias[..., None]) / scale[..., None]), 0, nb).astype(np.uint8)
        return pack_codes(q.reshape(rows, cols), bits), f32_to_sb(scale, sb_dtype), f32_to_sb(bias, sb_dtype)
    scale = (mx - mn) / nb
    scale = np.where(scale == 0, np.float32(1.0), scale).astype(np.float32)
    s16 = f32_to_sb(scale, sb_dtype)
    b16 = f32_to_sb(mn, sb_dtype)
    s32 = sb_to_f32(s16, sb_dtype)
    b32 = sb_to_f32(b16, sb_dtype)
    s32 = np.where(s32 == 0, np.float32(1.0), s32)
    q = np.clip(np.round((g - b32[..., None]) / s32[..., None]), 0, nb).astype(np.uint8)
    q = q.reshape(rows, cols)
    return pack_codes(q, bits), s16, b16


def pack_codes(q: np.ndarray, bits: int) -> np.ndarray:
    """codes uint8 [rows, cols] -> MLX packed layout (vectorised)."""
    rows, cols = q.shape
    q = q.astype(np.uint32)
    if bits == 4:
        q8 = q.reshape(rows, cols // 8, 8)
        word = np.zeros((rows, cols // 8), dtype=np.uint32)
        for t in range(8):
            word |= q8[:, :, t] << np.uint32(4 * t)
        return word
    q8 = q.reshape(rows, cols // 8, 8)
    word = np.zeros((rows, cols // 8), dtype=np.uint32)
    for t in range(8):
        word |= q8[:, :, t] << np.uint32(3 * t)
    out = np.empty((rows, cols // 8, 3), dtype=np.uint8)
    out[:, :, 0] = word & 0xFF
    out[:, :, 1] = (word >> 8) & 0xFF
    out[:, :, 2] = (word >> 16) & 0xFF
    return out.reshape(rows, cols * 3 // 8)


def unpack_codes(packed: np.ndarray, bits: int, cols: int) -> np.ndarray:
    """MLX packed layout -> codes uint8 [rows, cols] (vectorised)."""
    rows = packed.shape[0]
    if bits == 4:
        w = packed.reshape(rows, cols // 8).astype(np.uint32)
        return np.stack([(w >> np.uint32(4 * t)) & 0xF for t in range(8)], -1).reshape(rows, cols).astype(np.uint8)
    b = packed.reshape(rows, cols // 8, 3).astype(np.uint32)
    w = b[:, :, 0] | (b[:, :, 1] << 8) | (b[:, :, 2] << 16)
    return np.stack([(w >> np.uint32(3 * t)) & 7 for t in range(8)], -1).reshape(rows, cols).astype(np.uint8)


def dequantize_affine(packed, scales, biases, bits, cols, gs=64, sb_dtype="f16") -> np.ndarray:
    q = unpack_codes(packed, bits, cols).astype(np.float32)
    rows = q.shape[0]
    s = sb_to_f32(scales, sb_dtype).reshape(rows, cols // gs, 1)
    b = sb_to_f32(biases, sb_dtype).reshape(rows, cols // gs, 1)
    return (q.reshape(rows, cols // gs, gs) * s + b).reshape(rows, cols)


# ---------------------------------------------------------------------------
# C oracle wrappers
# ---------------------------------------------------------------------------

def matvec(bits, packed, scales, biases, x, sb_dtype="f16", gs=64):
    """fp32 out[r] in the reference scalar order (C oracle)."""
    out_dim = packed.shape[0]
    in_dim = x.shape[0]
    out = np.zeros(out_dim, np.float32)
    x = np.ascontiguousarray(x, np.float32)
    lib().kqo_matvec(bits, _p(np.ascontiguousarray(packed)), _p(np.ascontiguousarray(scales), _u16p),
                     _p(np.ascontiguousarray(biases), _u16p), 1 if sb_dtype == "f16" else 0,
                     _p(x, _f32p), _p(out, _f32p), out_dim, in_dim, gs)
    return out


class ExpertLayer:
    """A stacked MoE layer in MLX layout: for m in (gate, up, down):
    w[m] [E, rows, packed_cols], s[m]/b[m] [E, rows, groups] (uint16 bits)."""

    def __init__(self, bits, hidden, inter, w, s, b, sb_dtype="f16", act="silu", gs=64, variant=None):
        self.bits, self.hidden, self.inter, self.gs = bits, hidden, inter, gs
        # accumulation order of the reference library the layer would run in:
        # "small" (kandiga_cpu_expert.m) or "lg" (kandiga_cpu_expert_lg.m, GELU models)
        self.variant = variant or ("lg" if act == "gelu" else "small")
        self.w = [np.ascontiguousarray(a) for a in w]
        self.s = [np.ascontiguousarray(a) for a in s]
        self.b = [np.ascontiguousarray(a) for a in b]
        self.sb_dtype, self.act = sb_dtype, act
        self.num_experts = self.w[0].shape[0]

    @classmethod
    def random(cls, bits, hidden, inter, num_experts, seed=0, sb_dtype="f16", act="silu", std=0.02,
               variant=None):
        rng = np.random.RandomState(seed)
        w, s, b = [], [], []
        for rows, cols in ((inter, hidden), (inter, hidden), (hidden, inter)):
            ws, ss, bs = [], [], []
            for _ in range(num_experts):
                W = (rng.randn(rows, cols) * std).astype(np.float32)
                p, sc, bi = quantize_affine(W, bits, 64, sb_dtype)
                ws.append(p); ss.append(sc); bs.append(bi)
            w.append(np.stack(ws)); s.append(np.stack(ss)); b.append(np.stack(bs))
        return cls(bits, hidden, inter, w, s, b, sb_dtype, act, variant=variant)

    def expert_blob(self, e: int) -> bytes:
        """The nine tensors of expert e concatenated in BKEX order."""
        parts = []
        for m in range(3):
            parts += [self.w[m][e].tobytes(), self.s[m][e].tobytes(), self.b[m][e].tobytes()]
        return b"".join(parts)

    def layer_blob(self) -> bytes:
        return b"".join(self.expert_blob(e) for e in range(self.num_experts))

    def expert_size(self) -> int:
        return sum(self.w[m][0].nbytes + self.s[m][0].nbytes + self.b[m][0].nbytes for m in range(3))

    def tensor_offsets(self):
        offs, o = [], 0
        for m in range(3):
            for a in (self.w[m], self.s[m], self.b[m]):
                offs.append(o)
                o += a[0].nbytes
        return offs

    def moe(self, x: np.ndarray, idx: np.ndarray, threads: int = 0) -> np.ndarray:
        """x [T, H] fp32, idx [T, K] -> per-(t,k) expert outputs [T, K, H] fp32 (C oracle)."""
        x = np.ascontiguousarray(x, np.float32)
        idx = np.ascontiguousarray(idx, np.int32)
        T, K = idx.shape
        out = np.zeros((T, K, self.hidden), np.float32)
        wp = (ctypes.c_void_p * 3)(*[a.ctypes.data for a in self.w])
        sp = (ctypes.c_void_p * 3)(*[a.ctypes.data for a in self.s])
        bp = (ctypes.c_void_p * 3)(*[a.ctypes.data for a in self.b])
        ws = (ctypes.c_int64 * 3)(*[a[0].nbytes for a in self.w])
        ss = (ctypes.c_int64 * 3)(*[a[0].size for a in self.s])
        lib().kqo_moe_layer(self.bits, 1 if self.variant == "lg" else 0, 1 if self.sb_dtype == "f16" else 0,
                            1 if self.act == "gelu" else 0, wp, ws, sp, bp, ss, _p(x, _f32p),
                            _p(idx, _i32p), T, K, _p(out, _f32p), self.hidden, self.inter, self.gs,
                            threads or (os.cpu_count() or 1))
        return out

    def dequant_fp32_moe(self, x: np.ndarray, idx: np.ndarray) -> np.ndarray:
        """The "fp32 dequant reference": dequantize, then fp32 matmuls
        (the semantics of kandiga/engine.py:295-304)."""
        T, K = idx.shape
        out = np.zeros((T, K, self.hidden), np.float32)
        cache = {}
        for t in range(T):
            for k in range(K):
                e = int(idx[t, k])
                if e not in cache:
                    cache[e] = [dequantize_affine(self.w[m][e], self.s[m][e], self.b[m][e], self.bits,
                                                  (self.hidden if m < 2 else self.inter), self.gs,
                                                  self.sb_dtype) for m in range(3)]
                G, U, D = cache[e]
                g = G @ x[t]
                u = U @ x[t]
                if self.act == "gelu":
                    a = 0.5 * g * (1 + np.tanh(0.7978845608 * (g + 0.044715 * g ** 3))) * u
                else:
                    a = g / (1 + np.exp(-g)) * u
                out[t, k] = D @ a.astype(np.float32)
        return out


def router_topk(logits: np.ndarray, K: int):
    logits = np.ascontiguousarray(logits, np.float32)
    T, E = logits.shape
    idx = np.zeros((T, K), np.int32)
    w = np.zeros((T, K), np.float32)
    lib().kqo_router_topk(_p(logits, _f32p), T, E, K, _p(idx, _i32p), _p(w, _f32p))
    return idx, w


def combine(y, w, res=None, shared=None, gate=None):
    y = np.ascontiguousarray(y, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    T, K, H = y.shape
    out = np.zeros((T, H), np.float32)
    r = None if res is None else np.ascontiguousarray(res, np.float32)
    sh = None if shared is None else np.ascontiguousarray(shared, np.float32)
    g = None if gate is None else np.ascontiguousarray(gate, np.float32)
    lib().kqo_combine(_p(y, _f32p), _p(w, _f32p), None if r is None else r.ctypes.data,
                      None if sh is None else sh.ctypes.data, None if g is None else g.ctypes.data,
                      T, K, H, _p(out, _f32p))
    return out


def shared_gate(x: np.ndarray, packed, scales, biases, bits, sb_dtype="f16", gs=64) -> np.ndarray:
    """sigmoid(w_gate . x) per token, w_gate one quantized row
    (kandiga/metal/moe_block.metal:335-404: sum of fma(q, s, b) * x in fp32)."""
    H = x.shape[-1]
    w = dequantize_affine(packed, scales, biases, bits, H, gs, sb_dtype).reshape(H).astype(np.float32)
    logit = (x.astype(np.float32) * w[None, :]).sum(-1, dtype=np.float32)
    return (1.0 / (1.0 + np.exp(-logit))).astype(np.float32)


def rms_norm(x_f16: np.ndarray, w: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    """fp16(x * (1 / sqrt(mean(x^2) + eps)) * w) in fp32 arithmetic
    (kandiga/metal/moe_block.metal:134-178); x fp16 [H], w the norm weight as fp32."""
    x = np.asarray(x_f16, np.float16).astype(np.float32)
    ss = np.float32((x * x).sum(dtype=np.float32))
    scale = np.float32(1.0) / np.sqrt(np.float32(ss / np.float32(x.shape[-1])) + np.float32(eps))
    return ((x * scale) * np.asarray(w, np.float32)).astype(np.float16)


def group_by_expert(idx: np.ndarray):
    """Stable grouping of the T*K assignments by expert id
    (kandiga/engine.py:407-418: mergesort argsort, boundaries via diff)."""
    T, K = idx.shape
    flat_tok = np.repeat(np.arange(T, dtype=np.int32), K)
    flat_k = np.tile(np.arange(K, dtype=np.int32), T)
    flat_exp = idx.reshape(-1).astype(np.int32)
    order = np.argsort(flat_exp, kind="mergesort")
    s_tok, s_k, s_exp = flat_tok[order], flat_k[order], flat_exp[order]
    changes = np.concatenate([[0], np.where(np.diff(s_exp))[0] + 1, [len(s_exp)]]).astype(np.int32)
    unique = s_exp[changes[:-1]]
    return s_tok, s_exp, s_k, changes, unique


# ---------------------------------------------------------------------------
# BKEX container (kandiga/_pack_experts.py:95-132)
# ---------------------------------------------------------------------------

BKEX_HEADER = 4096
BKEX_NAMES = ["gate_proj.weight", "gate_proj.scales", "gate_proj.biases",
              "up_proj.weight", "up_proj.scales", "up_proj.biases",
              "down_proj.weight", "down_proj.scales", "down_proj.biases"]


def bkex_header(num_experts: int, tensors) -> bytes:
    """tensors: list of (name, shape, dtype_code 0=uint32/1=bf16, nbytes) in blob order."""
    buf = bytearray(BKEX_HEADER)
    expert_size = sum(t[3] for t in tensors)
    buf[0:4] = b"BKEX"
    struct.pack_into("<IIQI", buf, 4, 1, num_experts, expert_size, len(tensors))
    pos, off = 24, 0
    for name, shape, dt, nbytes in tensors:
        nb = name.encode("ascii")
        buf[pos] = len(nb)
        buf[pos + 1:pos + 1 + len(nb)] = nb
        pos += 25
        d0 = shape[0] if len(shape) > 0 else 0
        d1 = shape[1] if len(shape) > 1 else 0
        struct.pack_into("<IIIIB", buf, pos, off, nbytes, d0, d1, dt)
        pos += 17
        off += nbytes
    return bytes(buf)


def bkex_parse(header: bytes):
    if header[:4] != b"BKEX":
        raise ValueError("bad BKEX magic")
    version, ne, esz, nt = struct.unpack_from("<IIQI", header, 4)
    pos, tensors = 24, []
    for _ in range(nt):
        nl = header[pos]
        name = header[pos + 1:pos + 1 + min(nl, 24)].decode("ascii")
        off, nbytes, d0, d1, dt = struct.unpack_from("<IIIIB", header, pos + 25)
        tensors.append(dict(name=name, offset=off, nbytes=nbytes, d0=d0, d1=d1, dtype=dt))
        pos += 42
    return dict(version=version, num_experts=ne, expert_size=esz, tensors=tensors)


def bkex_tensors_for(layer: ExpertLayer):
    """Descriptor list for an ExpertLayer in BKEX order (MLX stores the 3-bit
    weight as uint32 [rows, cols*3/32])."""
    out = []
    for m, (rows, cols) in enumerate(((layer.inter, layer.hidden), (layer.inter, layer.hidden),
                                      (layer.hidden, layer.inter))):
        wcols = cols * layer.bits // 32
        out.append((BKEX_NAMES[3 * m], (rows, wcols), 0, rows * wcols * 4))
        out.append((BKEX_NAMES[3 * m + 1], (rows, cols // layer.gs), 1, rows * cols // layer.gs * 2))
        out.append((BKEX_NAMES[3 * m + 2], (rows, cols // layer.gs), 1, rows * cols // layer.gs * 2))
    return out


# ---------------------------------------------------------------------------
# TurboQuant (kandiga/kv_compress.py:30-118), numpy float32
# ---------------------------------------------------------------------------

class TurboQuantRef:
    def __init__(self, head_dim: int, num_heads: int, seed: int = 42):
        self.head_dim, self.num_heads = head_dim, num_heads
        rng = np.random.RandomState(seed)
        m = rng.randn(head_dim, head_dim).astype(np.float32)
        q, _ = np.linalg.qr(m)
        self.rotation = q.astype(np.float32)
        qjl = rng.choice([-1.0, 1.0], size=(head_dim, head_dim)).astype(np.float32)
        qjl /= math.sqrt(head_dim)
        self.qjl_proj = qjl

    def quantize(self, x: np.ndarray):
        """x [..., D] fp32 -> (codes int8, scale fp32 [...], zero fp32 [...], signs int8)."""
        rot = np.matmul(x.astype(np.float32), self.rotation)
        mn = rot.min(-1, keepdims=True)
        mx = rot.max(-1, keepdims=True)
        scale = (mx - mn) / np.float32(7.0)
        scale = np.where(scale == 0, np.float32(1.0), scale).astype(np.float32)
        q = np.clip(np.round((rot - mn) / scale), 0, 7).astype(np.int8)
        deq = q.astype(np.float32) * scale + mn
        res = rot - deq
        proj = np.matmul(res, self.qjl_proj)
        signs = (proj > 0).astype(np.int8)
        return q, scale[..., 0], mn[..., 0], signs

    def dequantize(self, q, scale, zero, signs) -> np.ndarray:
        s = scale[..., None].astype(np.float32)
        z = zero[..., None].astype(np.float32)
        deq = q.astype(np.float32) * s + z
        corr = s / np.float32(4.0)
        corrected = deq + np.where(signs.astype(bool), corr, -corr)
        return np.matmul(corrected, self.rotation.T).astype(np.float16)

    def attend(self, q: np.ndarray, k_codes, k_scale, k_zero, k_signs, v: np.ndarray) -> np.ndarray:
        """Single-query attention over a compressed key cache.
        q [H, D]; cache tensors [H, S, ...]; v [H, S, D] (fp16 or fp32 values).
        Keys are the reference dequantization (fp16, as `.keys` returns)."""
        kh = self.dequantize(k_codes, k_scale, k_zero, k_signs).astype(np.float32)
        D = q.shape[-1]
        scores = np.einsum("hd,hsd->hs", q.astype(np.float32), kh) / np.float32(math.sqrt(D))
        p = np.exp(scores - scores.max(-1, keepdims=True))
        p /= p.sum(-1, keepdims=True)
        return np.einsum("hs,hsd->hd", p, v.astype(np.float32)), scores  # scores: the scaled logits


# ---------------------------------------------------------------------------
# TQ3_1S (kandiga/tq3/quantize.py), vectorised numpy
# ---------------------------------------------------------------------------

TQ3_CENTROIDS = np.array([-1.996684, -1.291398, -0.740341, -0.247508,
                          0.230106, 0.725222, 1.277503, 1.988943], dtype=np.float32)
TQ3_BOUNDARIES = np.array([-1.644041, -1.015870, -0.493924, -0.008701,
                           0.477664, 1.001362, 1.633223], dtype=np.float32)
TQ3_SIGNS = np.array([+1, -1, +1, -1, +1, +1, -1, +1, -1, -1, +1, -1, +1, +1, -1, +1,
                      -1, -1, +1, -1, +1, -1, -1, +1, -1, +1, +1, -1, +1, -1, -1, +1],
                     dtype=np.float32)


def _butterfly32(a: np.ndarray) -> np.ndarray:
    """Unnormalised Walsh-Hadamard butterfly on the last axis (length 32), in the
    reference's stage order (step 1, 2, 4, 8, 16)."""
    out = a.astype(np.float32).copy()
    step = 1
    while step < 32:
        v = out.reshape(*out.shape[:-1], 32 // (2 * step), 2, step)
        a0 = v[..., 0, :].copy()
        b0 = v[..., 1, :].copy()
        v[..., 0, :] = a0 + b0
        v[..., 1, :] = a0 - b0
        out = v.reshape(*out.shape)
        step *= 2
    return out


def tq3_wht_forward(x: np.ndarray) -> np.ndarray:
    return _butterfly32(x * TQ3_SIGNS) / np.float32(np.sqrt(32.0))


def tq3_wht_inverse(x: np.ndarray) -> np.ndarray:
    return _butterfly32(x) * TQ3_SIGNS / np.float32(np.sqrt(32.0))


def _tq3_index(v: np.ndarray) -> np.ndarray:
    idx = np.zeros(v.shape, np.uint8)
    for b in range(7):
        idx[v > TQ3_BOUNDARIES[b]] = b + 1
    return idx


def _tq3_refine(halves: np.ndarray, rms: np.ndarray, means: np.ndarray) -> np.ndarray:
    """Grid search over scale multipliers, then 6 least-squares refinements
    (kandiga/tq3/quantize.py:187-240), vectorised over half-blocks.  Inputs
    are float64, as they are in the reference under numpy 2 promotion rules."""
    n = halves.shape[0]
    centered = halves - means[:, None]
    best_s = rms.copy()
    best_e = np.full(n, np.inf)
    for mult in np.array([0.60, 0.70, 0.80, 0.90, 1.00, 1.10, 1.20, 1.35, 1.50]):
        s = np.maximum(rms * mult, 1e-10)
        idx = _tq3_index(centered * (1.0 / s)[:, None])
        deq = TQ3_CENTROIDS[idx] * s[:, None] + means[:, None]
        e = np.sum((halves - deq) ** 2, axis=1)
        better = e < best_e
        best_e[better] = e[better]
        best_s[better] = s[better]
    s = best_s.copy()
    for _ in range(6):
        idx = _tq3_index(centered * (1.0 / np.maximum(s, 1e-10))[:, None])
        c = TQ3_CENTROIDS[idx]
        num = np.sum(centered * c, axis=1)
        den = np.sum(c ** 2, axis=1)
        with np.errstate(divide="ignore", invalid="ignore"):
            ns = np.where(den > 1e-12, num / den, s)
        ns = np.maximum(ns, 1e-10)
        deq = c * ns[:, None] + means[:, None]
        e = np.sum((halves - deq) ** 2, axis=1)
        better = e < best_e
        best_e[better] = e[better]
        best_s[better] = ns[better]
        s = ns
    return best_s


def tq3_quantize(weights: np.ndarray):
    """-> (bytes of 20-byte blocks, shape, num_blocks): d0 d1 m0 m1 fp16 + 12 B codes.
    The butterfly runs in float32 and the 1/sqrt(32) step promotes to float64,
    as in kandiga/tq3/quantize.py:367-379 under numpy 2."""
    flat = weights.reshape(-1).astype(np.float32)
    pad = (32 - flat.size % 32) % 32
    if pad:
        flat = np.concatenate([flat, np.zeros(pad, np.float32)])
    nb = flat.size // 32
    rot = _butterfly32(flat.reshape(nb, 32) * TQ3_SIGNS) / np.sqrt(32.0)
    h0, h1 = rot[:, :16], rot[:, 16:]
    m0, m1 = np.mean(h0, axis=1), np.mean(h1, axis=1)
    r0 = np.sqrt(np.mean((h0 - m0[:, None]) ** 2, axis=1))
    r1 = np.sqrt(np.mean((h1 - m1[:, None]) ** 2, axis=1))
    r0[r0 < 1e-10] = 1.0
    r1[r1 < 1e-10] = 1.0
    d0 = _tq3_refine(h0, r0, m0)
    d1 = _tq3_refine(h1, r1, m1)
    idx = np.zeros((nb, 32), np.uint8)
    idx[:, :16] = _tq3_index((h0 - m0[:, None]) / np.maximum(d0, 1e-10)[:, None])
    idx[:, 16:] = _tq3_index((h1 - m1[:, None]) / np.maximum(d1, 1e-10)[:, None])
    lim = 65504.0
    hdr = np.stack([np.clip(d0, -lim, lim), np.clip(d1, -lim, lim),
                    np.clip(m0, -lim, lim), np.clip(m1, -lim, lim)], 1).astype(np.float16)
    codes = tq3_pack_indices(idx)
    blocks = np.concatenate([hdr.view(np.uint8).reshape(nb, 8), codes], 1)
    return blocks.tobytes(), weights.shape, nb


def tq3_pack_indices(idx: np.ndarray) -> np.ndarray:
    """[N, 32] indices -> [N, 12] bytes: four 24-bit little-endian groups of 8."""
    n = idx.shape[0]
    g = idx.reshape(n, 4, 8).astype(np.uint32)
    word = np.zeros((n, 4), np.uint32)
    for r in range(8):
        word |= g[:, :, r] << np.uint32(3 * r)
    out = np.stack([word & 0xFF, (word >> 8) & 0xFF, (word >> 16) & 0xFF], -1).astype(np.uint8)
    return out.reshape(n, 12)


def tq3_unpack_indices(codes: np.ndarray) -> np.ndarray:
    n = codes.shape[0]
    b = codes.reshape(n, 4, 3).astype(np.uint32)
    word = b[:, :, 0] | (b[:, :, 1] << 8) | (b[:, :, 2] << 16)
    return np.stack([(word >> np.uint32(3 * r)) & 7 for r in range(8)], -1).reshape(n, 32).astype(np.uint8)


def tq3_dequantize(data: bytes, shape, num_blocks: int) -> np.ndarray:
    blocks = np.frombuffer(data, np.uint8).reshape(num_blocks, -1)
    if blocks.shape[1] == 16:
        hdr = blocks[:, :4].copy().view(np.float16).astype(np.float32)
        d0, d1 = hdr[:, 0], hdr[:, 1]
        m0 = m1 = np.zeros(num_blocks, np.float32)
        idx = tq3_unpack_indices(blocks[:, 4:16])
    else:
        hdr = blocks[:, :8].copy().view(np.float16).astype(np.float32)
        d0, d1, m0, m1 = hdr[:, 0], hdr[:, 1], hdr[:, 2], hdr[:, 3]
        idx = tq3_unpack_indices(blocks[:, 8:20])
    c = TQ3_CENTROIDS[idx]
    rot = np.empty((num_blocks, 32), np.float32)
    rot[:, :16] = c[:, :16] * d0[:, None] + m0[:, None]
    rot[:, 16:] = c[:, 16:] * d1[:, None] + m1[:, None]
    flat = tq3_wht_inverse(rot).reshape(-1)
    n = int(np.prod(shape))
    return flat[:n].reshape(shape)
