"""Routed experts of a model larger than HBM: host-pinned table, HBM slot pool.

The reference runs such models (397B-class) by streaming expert weights from
the SSD on every call and warming the OS page cache ahead of use with a
cross-layer predictor: the next layer's router applied to this layer's input,
top-K per token, union over tokens (``_CPUSwitchGLU._predict_and_prefetch``,
kandiga/engine.py:577-616; the multi-layer variant 618-668).

``SpillTable`` keeps the whole table in pinned host memory and `slots`
experts per layer in HBM (libkq ``kq_spill_*``).  ``fetch`` maps expert ids to
slot ids on the GPU and copies the experts that are not resident; the routed
kernels then run on the pool unchanged.  ``prefetch`` does the same ahead of
use on a second stream, and ``moe`` makes the current stream wait for it.
For a call that names more distinct experts than there are slots (a long
prefill), ``moe`` splits the tokens into runs that fit, reading the routing
on the host once.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from . import _native as N
from .experts import ExpertTable, _ptr, _stream, router_topk


def token_runs(idx: np.ndarray, num_experts: int, slots: int):
    """Split tokens (rows of idx [T, K]) into contiguous runs [(a, b), ...],
    each as long as its distinct valid expert ids fit in `slots`.  Ids outside
    [0, num_experts) take no slot (the kernels zero their rows)."""
    runs, start, seen = [], 0, set()
    for t in range(idx.shape[0]):
        row = set(int(e) for e in idx[t] if 0 <= e < num_experts)
        if len(row) > slots:
            raise ValueError(f"token {t} names {len(row)} distinct experts, more than {slots} slots")
        if len(seen | row) > slots:
            runs.append((start, t))
            start, seen = t, set()
        seen |= row
    if idx.shape[0] > start or not runs:
        runs.append((start, idx.shape[0]))
    return runs


class SpillTable:
    """All routed experts of `num_layers` MoE layers in pinned host memory,
    `slots` of each layer resident in HBM at a time (least recently used
    slots are refilled)."""

    def __init__(self, num_layers, num_experts, hidden, inter, slots, bits=3, sb_dtype="f16",
                 activation="silu"):
        self.lib = N.load()
        d = N.kq_table_desc(num_layers, num_experts, hidden, inter, bits, 64,
                            N.DT_F16 if sb_dtype == "f16" else N.DT_BF16,
                            N.ACT_GELU_TANH if activation == "gelu" else N.ACT_SILU)
        h = ctypes.c_void_p()
        N.check(self.lib.kq_spill_create(ctypes.byref(d), slots, ctypes.byref(h)), "kq_spill_create")
        self.handle = h
        self.num_layers, self.num_experts, self.hidden, self.inter = num_layers, num_experts, hidden, inter
        self.slots, self.bits, self.sb_dtype, self.activation = slots, bits, sb_dtype, activation
        self.pool = ExpertTable(num_layers, slots, hidden, inter, bits, sb_dtype, activation,
                                _handle=self.lib.kq_spill_pool(h))
        self.prefetch_stream = torch.cuda.Stream()
        self._pending = {}  # layer -> event recorded after its prefetch

    def __del__(self):
        try:
            if getattr(self, "handle", None):
                torch.cuda.synchronize()
                self.pool = None
                self.lib.kq_spill_destroy(self.handle)
                self.handle = None
        except Exception:
            pass

    @property
    def host_bytes(self) -> int:
        return int(self.lib.kq_spill_host_bytes(self.handle))

    @property
    def expert_bytes(self) -> int:
        return self.pool.expert_bytes

    # ---- loading -----------------------------------------------------------
    def store_layer(self, layer, table: ExpertTable, src_layer=0):
        """Copy layer `src_layer` of an HBM table of the same shape into the host store."""
        self._pending.pop(layer, None)
        N.check(self.lib.kq_spill_store_layer(self.handle, layer, table.handle, src_layer, _stream()),
                "kq_spill_store_layer")

    def _staging(self):
        return ExpertTable(1, self.num_experts, self.hidden, self.inter, self.bits, self.sb_dtype,
                           self.activation)

    def load_mlx(self, layer, gate, up, down):
        """gate/up/down: (weight, scales, biases) CUDA tensors stacked [E, rows, ...] (all experts)."""
        st = self._staging()
        st.load_mlx(0, gate, up, down)
        self.store_layer(layer, st, 0)

    def load_bkex(self, layer, file_bytes: bytes):
        st = self._staging()
        st.load_bkex(0, file_bytes)
        self.store_layer(layer, st, 0)

    # ---- residency ---------------------------------------------------------
    def _wait_prefetch(self, layer):
        ev = self._pending.pop(layer, None)
        if ev is not None:
            torch.cuda.current_stream().wait_event(ev)

    def fetch(self, layer, ids: torch.Tensor) -> torch.Tensor:
        """Expert ids (int32 CUDA tensor, any shape) -> slot ids of the pool, same shape."""
        self._wait_prefetch(layer)
        ids = ids.to(torch.int32).contiguous()
        slot = torch.empty_like(ids)
        N.check(self.lib.kq_spill_fetch(self.handle, layer, _ptr(ids), ids.numel(), _ptr(slot), _stream()),
                "kq_spill_fetch")
        return slot

    def prefetch(self, layer, ids: torch.Tensor):
        """Bring experts of `layer` into HBM on the prefetch stream, after the
        work already queued on the current stream; the next fetch/moe of
        `layer` waits for it."""
        if layer < 0 or layer >= self.num_layers:
            return
        ids = ids.to(torch.int32).contiguous()
        cur = torch.cuda.current_stream()
        ps = self.prefetch_stream
        ps.wait_stream(cur)
        prev = self._pending.pop(layer, None)
        if prev is not None:
            ps.wait_event(prev)
        N.check(self.lib.kq_spill_prefetch(self.handle, layer, _ptr(ids), ids.numel(),
                                           ctypes.c_void_p(ps.cuda_stream)), "kq_spill_prefetch")
        ids.record_stream(ps)
        ev = torch.cuda.Event()
        ev.record(ps)
        self._pending[layer] = ev

    def predict(self, x: torch.Tensor, next_router, top_k=8) -> torch.Tensor:
        """Experts the next layer is expected to route x to: its router on this
        layer's input, top-K per token (kandiga/engine.py:584-601).
        next_router: [E, H] weight tensor or a callable x -> fp32 logits [T, E]."""
        xf = x.reshape(-1, x.shape[-1])
        if callable(next_router):
            logits = next_router(xf)
        else:
            logits = xf.float() @ next_router.float().t()
        idx, _ = router_topk(logits.float().contiguous(), top_k)
        return idx

    def predict_and_prefetch(self, layer, x, next_router, top_k=8):
        """``_predict_and_prefetch`` (kandiga/engine.py:577-616): predict layer
        `layer` + 1 from x and prefetch it."""
        if next_router is None or layer + 1 >= self.num_layers:
            return None
        ids = self.predict(x, next_router, top_k)
        self.prefetch(layer + 1, ids)
        return ids

    def stats(self, reset=False) -> dict:
        out = (ctypes.c_uint64 * 4)()
        N.check(self.lib.kq_spill_stats(self.handle, out, 1 if reset else 0, _stream()), "kq_spill_stats")
        return dict(hits=int(out[0]), misses=int(out[1]), bytes=int(out[2]), status=int(out[3]))

    def residency(self, layer):
        """-> (slot_of [E] int32, owner [slots] int32) numpy arrays."""
        slot_of = np.empty(self.num_experts, dtype=np.int32)
        owner = np.empty(self.slots, dtype=np.int32)
        N.check(self.lib.kq_spill_residency(self.handle, layer, slot_of.ctypes.data_as(ctypes.c_void_p),
                                            owner.ctypes.data_as(ctypes.c_void_p), _stream()),
                "kq_spill_residency")
        return slot_of, owner

    # ---- routed MLP ----------------------------------------------------------
    def moe(self, layer, x, *, logits=None, idx=None, weights=None, top_k=8, per_k=False, combine=True,
            residual=None, out_dtype=None, out=None, out_per_k=None, path="auto"):
        """``ExpertTable.moe`` on the spilled table: same arguments and
        results (idx holds expert ids).  Calls naming at most `slots` experts
        (every decode step with T * K <= slots) run with no host round trip."""
        T = x.shape[0]
        if logits is not None and idx is None:
            idx, weights = router_topk(logits, top_k)
        K = idx.shape[1]
        out_dtype = out_dtype or (x.dtype if x.dtype != torch.float32 else torch.float32)
        if combine and out is None:
            out = torch.empty(T, self.hidden, dtype=out_dtype, device=x.device)
        if per_k and out_per_k is None:
            out_per_k = torch.empty(T, K, self.hidden, dtype=out_dtype, device=x.device)
        if T * K <= self.slots:
            runs = [(0, T)]
        else:
            runs = token_runs(idx.cpu().numpy(), self.num_experts, self.slots)
        for a, b in runs:
            slot = self.fetch(layer, idx[a:b])
            self.pool.moe(layer, x[a:b], idx=slot, weights=None if weights is None else weights[a:b],
                          per_k=per_k, combine=combine,
                          residual=None if residual is None else residual[a:b], out_dtype=out_dtype,
                          out=None if out is None else out[a:b],
                          out_per_k=None if out_per_k is None else out_per_k[a:b], path=path)
        return dict(out=out if combine else None, per_k=out_per_k if per_k else None, idx=idx,
                    weights=weights)

    def status(self) -> int:
        """Device status of the pool's routed kernels (ExpertTable.status)."""
        return self.pool.status()
