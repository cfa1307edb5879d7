"""Routed-expert engine on the HBM table (torch tensors in, torch tensors out).

Python mirror of the reference's expert dispatch (kandiga/engine.py):

* ``ExpertLib``   -- same methods and argument meaning as ``_CPUExpertLib``
  (kandiga/engine.py:79-214): init(packed_dir, num_layers), expert_mlp_f16,
  expert_mlp_bf16, destroy, num_layers; numpy arrays in and out.  It binds the
  reference-compatible ``bakan_cpu_expert_*`` symbols of libkq.so, so the BKEX
  layer files are read once into HBM and every call runs the sm_100a kernels.
* ``ExpertTable`` -- the device-pointer path: a kq_table built from MLX-layout
  tensors already on the GPU, with ``moe()`` for the routed MLP (router top-K,
  gate/up, SwiGLU, down, weighted combine).
* ``SwitchGLU``   -- ``_CPUSwitchGLU.__call__(x, indices) -> [..., K, H]``
  (kandiga/engine.py:670-739): unweighted per-expert outputs, fp16.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np
import torch

from . import _native as N

_DT = {torch.float16: N.DT_F16, torch.bfloat16: N.DT_BF16, torch.float32: N.DT_F32}


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def mlx_matrix(w, s, b) -> N.kq_mlx_matrix:
    """kq_mlx_matrix for (stacked) MLX tensors; a leading expert dim sets the strides."""
    m = N.kq_mlx_matrix()
    m.weight, m.scales, m.biases = w.data_ptr(), s.data_ptr(), b.data_ptr()
    if w.dim() == 3:
        m.weight_stride = w[0].numel() * w.element_size()
        m.sb_stride = s[0].numel() * s.element_size()
    else:
        m.weight_stride = m.sb_stride = 0
    return m


class ExpertTable:
    """All routed experts of `num_layers` MoE layers, resident in HBM.

    bits 3|4, group 64, per-group scale/bias in fp16 ('f16') or bf16 ('bf16').
    """

    def __init__(self, num_layers, num_experts, hidden, inter, bits=3, sb_dtype="f16",
                 activation="silu", _handle=None):
        self.lib = N.load()
        if _handle is None:
            d = N.kq_table_desc(num_layers, num_experts, hidden, inter, bits, 64,
                                N.DT_F16 if sb_dtype == "f16" else N.DT_BF16,
                                N.ACT_GELU_TANH if activation == "gelu" else N.ACT_SILU)
            h = ctypes.c_void_p()
            N.check(self.lib.kq_table_create(ctypes.byref(d), ctypes.byref(h)), "kq_table_create")
            self._owned = True
        else:  # a table owned by another object (the HBM pool of a SpillTable)
            h = ctypes.c_void_p(_handle)
            self._owned = False
        self.handle = h
        self.num_layers, self.num_experts, self.hidden, self.inter = num_layers, num_experts, hidden, inter
        self.bits, self.sb_dtype, self.activation = bits, sb_dtype, activation
        self._ws = None
        self._ws_key = None

    def __del__(self):
        try:
            if getattr(self, "handle", None) and getattr(self, "_owned", True):
                self.lib.kq_table_destroy(self.handle)
                self.handle = None
        except Exception:
            pass

    @property
    def bytes(self) -> int:
        return int(self.lib.kq_table_bytes(self.handle))

    @property
    def expert_bytes(self) -> int:
        return int(self.lib.kq_table_expert_bytes(self.handle))

    def load_mlx(self, layer, gate, up, down, expert_begin=0):
        """gate/up/down: (weight, scales, biases) CUDA tensors stacked [E, rows, ...]."""
        n = gate[0].shape[0]
        mg, mu, md = mlx_matrix(*gate), mlx_matrix(*up), mlx_matrix(*down)
        N.check(self.lib.kq_table_load_mlx(self.handle, layer, expert_begin, n, ctypes.byref(mg),
                                           ctypes.byref(mu), ctypes.byref(md), _stream()),
                "kq_table_load_mlx")

    def load_bkex(self, layer, file_bytes: bytes):
        buf = ctypes.create_string_buffer(file_bytes, len(file_bytes))
        N.check(self.lib.kq_table_load_bkex(self.handle, layer, buf, len(file_bytes), _stream()),
                "kq_table_load_bkex")

    def unpack_mlx(self, layer, expert, matrix):
        """-> (weight bytes uint8, scales int16-bits, biases) of one matrix in MLX layout."""
        rows, cols = ((self.inter, self.hidden) if matrix < 2 else (self.hidden, self.inter))
        wb = rows * cols * self.bits // 8
        dev = torch.device("cuda")
        w = torch.empty(wb, dtype=torch.uint8, device=dev)
        s = torch.empty(rows * cols // 64, dtype=torch.int16, device=dev)
        b = torch.empty_like(s)
        N.check(self.lib.kq_table_unpack_mlx(self.handle, layer, expert, matrix, _ptr(w), _ptr(s), _ptr(b),
                                             _stream()), "kq_table_unpack_mlx")
        return w.reshape(rows, -1), s.reshape(rows, -1), b.reshape(rows, -1)

    def workspace(self, T, K, prefill=False):
        fn = self.lib.kq_moe_prefill_workspace_size if prefill else self.lib.kq_moe_workspace_size
        need = int(fn(self.handle, T, K))
        if self._ws is None or self._ws.numel() < need:
            self._ws = torch.zeros(max(need, 1), dtype=torch.uint8, device="cuda")
        return self._ws

    def status(self) -> int:
        if self._ws is None:
            return 0
        st = ctypes.c_uint32(0)
        N.check(self.lib.kq_status_read(_ptr(self._ws), ctypes.byref(st), _stream()), "kq_status_read")
        return st.value

    # token count from which the grouped tensor-core path (kq_moe_prefill) is used
    PREFILL_MIN_TOKENS = 16

    def moe(self, layer, x, *, logits=None, idx=None, weights=None, top_k=8, per_k=False, combine=True,
            residual=None, out_dtype=None, out=None, out_per_k=None, path="auto"):
        """Routed MLP of layer `layer` for x [T, H] (fp16/bf16/fp32 CUDA tensor).

        Routing: pass `logits` [T, E] fp32 (router top-K runs on the GPU and
        idx/weights are returned), or `idx` [T, K] int32 (+ `weights` [T, K]
        fp32 when combining).  path: "decode" (every (token, k) pair runs its
        expert), "prefill" (grouped by expert on the tensor cores) or "auto".
        Returns dict(out=[T, H] or None, per_k=[T, K, H] or None, idx, weights)."""
        T = x.shape[0]
        K = idx.shape[1] if idx is not None else top_k
        out_dtype = out_dtype or (x.dtype if x.dtype != torch.float32 else torch.float32)
        dev = x.device
        if logits is not None:
            if idx is None:
                idx = torch.empty(T, K, dtype=torch.int32, device=dev)
            if weights is None:
                weights = torch.empty(T, K, dtype=torch.float32, device=dev)
        if combine and out is None:
            out = torch.empty(T, self.hidden, dtype=out_dtype, device=dev)
        if per_k and out_per_k is None:
            out_per_k = torch.empty(T, K, self.hidden, dtype=out_dtype, device=dev)
        if residual is not None and (residual.dtype != out_dtype or residual.shape != (T, self.hidden)):
            raise ValueError("residual must be [T, hidden] in out_dtype")
        if path == "auto":
            path = "prefill" if (T >= self.PREFILL_MIN_TOKENS and self.hidden % 512 == 0 and
                                 self.inter % 512 == 0) else "decode"
        ws = self.workspace(T, K, prefill=(path == "prefill"))
        fn = self.lib.kq_moe_prefill if path == "prefill" else self.lib.kq_moe_decode
        rc = fn(self.handle, layer, _ptr(x), _DT[x.dtype], T, _ptr(logits), _ptr(idx), _ptr(weights), K,
                _ptr(out_per_k) if per_k else None, _ptr(out) if combine else None, _DT[out_dtype],
                _ptr(residual), _ptr(ws), ws.numel(), _stream())
        N.check(rc, f"kq_moe_{path}")
        return dict(out=out if combine else None, per_k=out_per_k if per_k else None, idx=idx,
                    weights=weights)


    def decode_batch(self, x, *, layers=None, layer=0, logits=None, idx=None, weights=None, top_k=8,
                     per_k=False, combine=True, residual=None, norm_w=None, eps=1e-6, out_dtype=None, out=None,
                     out_per_k=None):
        """n independent single-token items in one launch (kq_moe_decode_batch):
        item j = row j of x through layer layers[j] (int32 CUDA tensor [n]; None:
        all through `layer`), routed by row j of `logits` or given by `idx` /
        `weights`.  Same outputs as moe(); items must not depend on each other."""
        n = x.shape[0]
        K = idx.shape[1] if idx is not None else top_k
        out_dtype = out_dtype or (x.dtype if x.dtype != torch.float32 else torch.float32)
        dev = x.device
        if logits is not None:
            if idx is None:
                idx = torch.empty(n, K, dtype=torch.int32, device=dev)
            if weights is None:
                weights = torch.empty(n, K, dtype=torch.float32, device=dev)
        if combine and out is None:
            out = torch.empty(n, self.hidden, dtype=out_dtype, device=dev)
        if per_k and out_per_k is None:
            out_per_k = torch.empty(n, K, self.hidden, dtype=out_dtype, device=dev)
        need = int(self.lib.kq_moe_decode_batch_workspace_size(self.handle, K))
        if getattr(self, "_bws", None) is None or self._bws.numel() < need:
            self._bws = torch.zeros(max(need, 1), dtype=torch.uint8, device=dev)
        rc = self.lib.kq_moe_decode_batch(self.handle, n, _ptr(layers), layer, _ptr(x), _DT[x.dtype],
                                          _ptr(logits), _ptr(idx), _ptr(weights), K,
                                          _ptr(out_per_k) if per_k else None, _ptr(out) if combine else None,
                                          _DT[out_dtype], _ptr(residual), _ptr(norm_w), eps, _ptr(self._bws),
                                          self._bws.numel(), _stream())
        N.check(rc, "kq_moe_decode_batch")
        return dict(out=out if combine else None, per_k=out_per_k if per_k else None, idx=idx,
                    weights=weights)

    def batch_status(self) -> int:
        """device status word of decode_batch (read and cleared)"""
        if getattr(self, "_bws", None) is None:
            return 0
        st = ctypes.c_uint32(0)
        N.check(self.lib.kq_status_read(_ptr(self._bws), ctypes.byref(st), _stream()), "kq_status_read")
        return st.value

    def moe_block(self, layer, x, logits, top_k, shared_gate, shared_id=None, gate_bits=4, gate_sb="f16",
                  residual=None, out_dtype=None, path="auto"):
        """MoE block with a shared expert (kandiga/metal/moe_block.metal:134-584):
        out = [res] + sum_k w_k expert_k(x) + sigmoid(w_gate . x) shared(x).

        The shared expert is expert `shared_id` of this layer (default: the last
        one; `logits` cover the routed experts before it).  shared_gate =
        (weight, scales, biases): the gate row [1, H] in MLX layout.
        Returns dict(out, idx [T, K+1], weights [T, K+1], gate [T])."""
        T, E = logits.shape
        sid = self.num_experts - 1 if shared_id is None else shared_id
        dev = x.device
        idx, w = router_topk(logits, top_k)
        idx2 = torch.empty(T, top_k + 1, dtype=torch.int32, device=dev)
        w2 = torch.empty(T, top_k + 1, dtype=torch.float32, device=dev)
        gate = torch.empty(T, dtype=torch.float32, device=dev)
        gw, gs, gb = shared_gate
        N.check(self.lib.kq_shared_gate(_ptr(x), _DT[x.dtype], T, self.hidden, _ptr(gw), _ptr(gs), _ptr(gb),
                                        gate_bits, N.DT_F16 if gate_sb == "f16" else N.DT_BF16, _ptr(idx), _ptr(w),
                                        top_k, sid, _ptr(idx2), _ptr(w2), _ptr(gate), _stream()), "kq_shared_gate")
        r = self.moe(layer, x, idx=idx2, weights=w2, combine=True, residual=residual, out_dtype=out_dtype,
                     path=path)
        return dict(out=r["out"], idx=idx2, weights=w2, gate=gate)


def router_topk(logits: torch.Tensor, k: int):
    """softmax -> top-k (strict '>', lowest index on ties) -> renormalised weights."""
    lib = N.load()
    T, E = logits.shape
    idx = torch.empty(T, k, dtype=torch.int32, device=logits.device)
    w = torch.empty(T, k, dtype=torch.float32, device=logits.device)
    N.check(lib.kq_router_topk(_ptr(logits.contiguous()), T, E, k, _ptr(idx), _ptr(w), _stream()),
            "kq_router_topk")
    return idx, w


class SwitchGLU:
    """Drop-in for ``_CPUSwitchGLU`` (kandiga/engine.py:327-739) on CUDA tensors:
    ``__call__(x [..., H], indices [..., K]) -> [..., K, H]`` fp16, unweighted
    (the caller applies scores and sums, as mlx-lm's SparseMoeBlock does)."""

    def __init__(self, table: ExpertTable, layer_idx: int, hidden_size: int = 2048, top_k: int = 8):
        self.table, self._layer_idx, self._hidden_size, self._top_k = table, layer_idx, hidden_size, top_k

    def __call__(self, x: torch.Tensor, indices: torch.Tensor) -> torch.Tensor:
        K = indices.shape[-1]
        xf = x.reshape(-1, self._hidden_size)
        if xf.dtype not in (torch.float16, torch.bfloat16):
            xf = xf.to(torch.float16)
        idx = indices.reshape(-1, K).to(torch.int32).contiguous()
        r = self.table.moe(self._layer_idx, xf.contiguous(), idx=idx, per_k=True, combine=False,
                           out_dtype=torch.float16)
        return r["per_k"].reshape(*indices.shape, self._hidden_size)


class ExpertLib:
    """Same interface as the reference's ``_CPUExpertLib`` (kandiga/engine.py:79-214),
    bound to libkq.so's reference-compatible symbols."""

    def __init__(self, large: bool = False):
        self._lib = N.load()
        self._large = large

    def init(self, packed_dir: str, num_layers: int):
        engine = self._lib.bakan_cpu_expert_init(packed_dir.encode(), num_layers)
        if engine is None:
            raise RuntimeError(f"Failed to initialize CPU expert engine from {packed_dir}")
        return engine

    def expert_mlp_f16(self, engine, layer_idx, x_f16, expert_indices, num_experts, hidden_size=2048):
        output = np.empty((num_experts, hidden_size), dtype=np.float16)
        idx = np.ascontiguousarray(np.asarray(expert_indices).astype(np.int32))
        x = np.ascontiguousarray(x_f16, dtype=np.float16)
        ret = self._lib.bakan_cpu_expert_mlp_f16(engine, layer_idx, x.ctypes.data_as(ctypes.c_void_p),
                                                 idx.ctypes.data_as(N.c_i32p), num_experts,
                                                 output.ctypes.data_as(ctypes.c_void_p))
        if ret != 0:
            raise RuntimeError(f"CPU expert MLP failed for layer {layer_idx}")
        return output

    def expert_mlp_bf16(self, engine, layer_idx, x_bf16, expert_indices, num_experts, hidden_size=2048):
        output = np.empty((num_experts, hidden_size), dtype=np.float16)
        idx = np.ascontiguousarray(np.asarray(expert_indices).astype(np.int32))
        x = np.ascontiguousarray(x_bf16)  # uint16 bit patterns, as MLX hands them over
        ret = self._lib.bakan_cpu_expert_mlp_bf16(engine, layer_idx, x.ctypes.data_as(ctypes.c_void_p),
                                                  idx.ctypes.data_as(N.c_i32p), num_experts,
                                                  output.ctypes.data_as(ctypes.c_void_p))
        if ret != 0:
            raise RuntimeError(f"CPU expert MLP (bf16) failed for layer {layer_idx}")
        return output

    def destroy(self, engine):
        if engine is not None:
            self._lib.bakan_cpu_expert_destroy(engine)

    def num_layers(self, engine) -> int:
        return self._lib.bakan_cpu_expert_num_layers(engine)


class QuantizedLinear:
    """Dense MLX-affine quantized matrix in HBM (the shared / dense-layer GEMV).

    pair=True holds two matrices (gate, up) and returns act(gate x) * (up x)."""

    def __init__(self, rows, cols, bits=3, sb_dtype="f16", pair=False):
        self.lib = N.load()
        h = ctypes.c_void_p()
        N.check(self.lib.kq_qmat_create(rows, cols, bits, N.DT_F16 if sb_dtype == "f16" else N.DT_BF16,
                                        1 if pair else 0, ctypes.byref(h)), "kq_qmat_create")
        self.handle, self.rows, self.cols, self.bits, self.pair = h, rows, cols, bits, pair

    def __del__(self):
        try:
            if getattr(self, "handle", None):
                self.lib.kq_qmat_destroy(self.handle)
                self.handle = None
        except Exception:
            pass

    def load_mlx(self, a, b=None):
        ma = mlx_matrix(*a)
        mb = mlx_matrix(*b) if b is not None else None
        N.check(self.lib.kq_qmat_load_mlx(self.handle, ctypes.byref(ma), ctypes.byref(mb) if mb else None,
                                          _stream()), "kq_qmat_load_mlx")

    def unpack_mlx(self, which=0):
        dev = torch.device("cuda")
        w = torch.empty(self.rows * self.cols * self.bits // 8, dtype=torch.uint8, device=dev)
        s = torch.empty(self.rows * self.cols // 64, dtype=torch.int16, device=dev)
        b = torch.empty_like(s)
        N.check(self.lib.kq_qmat_unpack_mlx(self.handle, which, _ptr(w), _ptr(s), _ptr(b), _stream()),
                "kq_qmat_unpack_mlx")
        return w.reshape(self.rows, -1), s.reshape(self.rows, -1), b.reshape(self.rows, -1)

    def __call__(self, x, norm_weight=None, eps=1e-6, activation="silu", out_dtype=None, out=None):
        T = x.shape[0]
        out_dtype = out_dtype or x.dtype
        if out is None:
            out = torch.empty(T, self.rows, dtype=out_dtype, device=x.device)
        N.check(self.lib.kq_dense_gemv(self.handle, _ptr(x), _DT[x.dtype], T, _ptr(norm_weight), eps,
                                       N.ACT_GELU_TANH if activation == "gelu" else N.ACT_SILU, _ptr(out),
                                       _DT[out_dtype], _stream()), "kq_dense_gemv")
        return out
