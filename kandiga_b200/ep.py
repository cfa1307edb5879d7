"""Expert-parallel MoE layers across the GPUs of one node (one process per GPU).

The routed experts of a layer are partitioned over the ranks (each rank's
kq_table holds only its own experts); tokens are data-parallel (each rank owns
its own tokens).  Per layer and rank:

1. route the local tokens (kq_router_topk: softmax, top-K, renormalise);
2. count the (token, k) assignments per destination rank, exchange the counts
   (all-to-all of G int64);
3. all-to-all-v of the assigned token rows (fp16/bf16) and of their expert ids
   local to the destination;
4. every rank runs its experts on the rows it received, grouped by expert
   (kq_moe_prefill / kq_moe_decode with one assignment per row);
5. all-to-all-v of the expert outputs back to the token owners;
6. weighted combine with the residual and the gated shared expert, computed
   on the owner (kq_combine).

Two exchanges implement these steps:

* ``ExpertParallelMoE``: NCCL (or gloo) all-to-all-v through torch.distributed,
  one row per (token, k) assignment, split sizes read on the host.  Router,
  expert compute and combine are pluggable, so the same exchange code runs with
  the GPU kernels or, in CPU tests, with a restatement of them.
* ``PeerExpertParallelMoE``: the libkq exchange over peer memory (kq_ep_*):
  one row per (token, destination rank), counts kept on the device, the
  destination returns the weighted sum of its experts; no host
  synchronisation, so a whole multi-layer step is one CUDA graph.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Callable, Optional

import numpy as np
import torch
import torch.distributed as dist

from . import _native as N

_DT = {torch.float16: N.DT_F16, torch.bfloat16: N.DT_BF16, torch.float32: N.DT_F32}


@dataclass
class ExpertPlacement:
    """owner[e]: rank holding routed expert e; local[e]: its index in that rank's table."""
    owner: np.ndarray
    local: np.ndarray
    world: int

    @classmethod
    def contiguous(cls, num_experts: int, world: int) -> "ExpertPlacement":
        per = (num_experts + world - 1) // world
        e = np.arange(num_experts)
        return cls((e // per).astype(np.int64), (e % per).astype(np.int64), world)

    @classmethod
    def balanced(cls, load: np.ndarray, world: int) -> "ExpertPlacement":
        """Greedy bin packing by expected load (largest first onto the least loaded
        rank with room), equal expert counts per rank (the expected routing
        frequencies are static across a run)."""
        E = len(load)
        cap = (E + world - 1) // world
        owner = np.zeros(E, np.int64)
        local = np.zeros(E, np.int64)
        tot = np.zeros(world)
        used = np.zeros(world, np.int64)
        for e in np.argsort(-np.asarray(load, np.float64), kind="stable"):
            cand = [r for r in range(world) if used[r] < cap]
            r = min(cand, key=lambda q: (tot[q], q))
            owner[e], local[e] = r, used[r]
            used[r] += 1
            tot[r] += load[e]
        return cls(owner, local, world)

    def experts_of(self, rank: int) -> np.ndarray:
        """Global ids of `rank`'s experts in local order."""
        ids = np.nonzero(self.owner == rank)[0]
        return ids[np.argsort(self.local[ids], kind="stable")]


def zipf_bias(num_experts: int, s: float = 1.1, seed: int = 0) -> np.ndarray:
    """Router-logit bias b_e = -s ln(rank_e + 1) with a seeded permutation of ranks."""
    rank = np.random.RandomState(seed).permutation(num_experts)
    return (-s * np.log(rank + 1.0)).astype(np.float32)


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def gpu_router(logits: torch.Tensor, k: int):
    from .experts import router_topk
    return router_topk(logits, k)


def gpu_combine(per_k, weights, residual=None, shared=None, gate=None, out_dtype=None):
    """kq_combine: [res] + sum_k w_k y_k + gate * shared."""
    T, K, H = per_k.shape
    out_dtype = out_dtype or per_k.dtype
    out = torch.empty(T, H, dtype=out_dtype, device=per_k.device)
    lib = N.load()
    p = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None  # noqa: E731
    N.check(lib.kq_combine(p(per_k), _DT[per_k.dtype], p(weights), T, K, H, p(residual), p(shared),
                           _DT[shared.dtype] if shared is not None else 0, p(gate), p(out), _DT[out_dtype],
                           _stream()), "kq_combine")
    return out


def table_local_moe(table):
    """One-rank path: the whole routed MLP of the layer on this rank's table
    (grouped by expert inside kq_moe_prefill / kq_moe_decode), combined over K in fp32."""
    def run(layer: int, x: torch.Tensor, idx: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        return table.moe(layer, x, idx=idx, weights=w, combine=True, out_dtype=torch.float32)["out"]
    return run


def table_compute(table):
    """Expert compute on this rank's kq_table: one assignment per received row."""
    def run(layer: int, rows: torch.Tensor, local_ids: torch.Tensor) -> torch.Tensor:
        R = rows.shape[0]
        if R == 0:
            return torch.empty(0, rows.shape[1], dtype=rows.dtype, device=rows.device)
        r = table.moe(layer, rows, idx=local_ids.to(torch.int32).reshape(R, 1).contiguous(), per_k=True,
                      combine=False, out_dtype=rows.dtype)
        return r["per_k"].reshape(R, -1)
    return run


class ExpertParallelMoE:
    """Expert-parallel routed MoE for the tokens this rank owns."""

    def __init__(self, placement: ExpertPlacement, rank: int, top_k: int,
                 compute: Callable, router: Callable = gpu_router, combine: Callable = gpu_combine,
                 group=None, local_moe: Optional[Callable] = None):
        """compute(layer, rows, local_ids) -> rows' expert outputs (one assignment a row);
        local_moe(layer, x, idx, w) -> [T, H] routed sum, used instead of the exchange when
        there is one rank (no permutation of the T*K rows)."""
        self.pl, self.rank, self.k, self.group = placement, rank, top_k, group
        self.compute, self.router, self.combine = compute, router, combine
        self.local_moe = local_moe
        self._owner = None
        self._local = None

    def _maps(self, dev):
        if self._owner is None or self._owner.device != dev:
            self._owner = torch.from_numpy(self.pl.owner).to(dev)
            self._local = torch.from_numpy(self.pl.local).to(dev)
        return self._owner, self._local

    def forward(self, layer: int, x: torch.Tensor, logits: torch.Tensor, residual=None, shared=None, gate=None,
                out_dtype=None, return_parts: bool = False):
        """x [T, H] this rank's tokens, logits [T, E] over the routed experts.
        shared [T, H] / gate [T]: the shared expert's output and gate (or None).
        Returns out [T, H] (and a dict of intermediate tensors if return_parts)."""
        G, K = self.pl.world, self.k
        T, H = x.shape
        dev = x.device
        owner, local = self._maps(dev)
        idx, w = self.router(logits, K)
        if G == 1 and self.local_moe is not None and not return_parts:
            local_idx = local[idx.to(torch.int64)].to(torch.int32).contiguous()
            routed = self.local_moe(layer, x, local_idx, w)
            ones = torch.ones(T, 1, dtype=torch.float32, device=dev)
            return self.combine(routed.reshape(T, 1, H), ones, residual=residual, shared=shared, gate=gate,
                                out_dtype=out_dtype)
        flat = idx.reshape(-1).to(torch.int64)
        dest = owner[flat]
        order = torch.argsort(dest, stable=True)
        tok = torch.div(order, K, rounding_mode="floor")
        send_x = x.index_select(0, tok).contiguous()
        send_ids = local[flat].index_select(0, order).to(torch.int32).contiguous()
        if G == 1:  # one rank: no exchange
            s_split = r_split = [T * K]
            y_back = self.compute(layer, send_x, send_ids).to(x.dtype).contiguous()
        else:
            send_counts = torch.bincount(dest, minlength=G).to(torch.int64)
            recv_counts = torch.empty_like(send_counts)
            dist.all_to_all_single(recv_counts, send_counts, group=self.group)
            s_split, r_split = send_counts.tolist(), recv_counts.tolist()
            R = int(sum(r_split))
            recv_x = torch.empty(R, H, dtype=x.dtype, device=dev)
            recv_ids = torch.empty(R, dtype=torch.int32, device=dev)
            dist.all_to_all_single(recv_x, send_x, r_split, s_split, group=self.group)
            dist.all_to_all_single(recv_ids, send_ids, r_split, s_split, group=self.group)
            y_recv = self.compute(layer, recv_x, recv_ids).to(x.dtype).contiguous()
            y_back = torch.empty(T * K, H, dtype=x.dtype, device=dev)
            dist.all_to_all_single(y_back, y_recv, s_split, r_split, group=self.group)
        per_k = torch.empty_like(y_back)
        per_k.index_copy_(0, order, y_back)
        per_k = per_k.reshape(T, K, H)
        out = self.combine(per_k, w, residual=residual, shared=shared, gate=gate, out_dtype=out_dtype)
        if return_parts:
            return out, dict(idx=idx, weights=w, per_k=per_k, send=s_split, recv=r_split)
        return out


# ---- exchange over peer memory (kq_ep) --------------------------------------------------------------

class PeerExchange:
    """This rank's exchange buffer (kq_ep_create): every rank of the group holds
    one of the same layout and peers store into it directly (CUDA IPC mapping).

    max_tokens: most tokens any rank passes to one layer call; dtype: the token
    rows' type (fp16 / bf16), also the type partial sums travel back in."""

    def __init__(self, rank: int, world: int, max_tokens: int, hidden: int, top_k: int,
                 dtype=torch.float16, wait_ns: Optional[int] = None):
        self.lib = N.load()
        self.rank, self.world, self.max_tokens, self.hidden, self.top_k = rank, world, max_tokens, hidden, top_k
        self.dtype = dtype
        h = ctypes.c_void_p()
        N.check(self.lib.kq_ep_create(rank, world, max_tokens, hidden, top_k, _DT[dtype], ctypes.byref(h)),
                "kq_ep_create")
        self.handle = h
        if wait_ns is not None:
            N.check(self.lib.kq_ep_set_wait_ns(h, int(wait_ns)), "kq_ep_set_wait_ns")

    def ipc_handle(self) -> bytes:
        buf = ctypes.create_string_buffer(N.EP_HANDLE_BYTES)
        N.check(self.lib.kq_ep_ipc_handle(self.handle, buf), "kq_ep_ipc_handle")
        return buf.raw

    def connect(self, group=None, gather: Optional[Callable] = None):
        """Exchange the IPC handles over the process group (all ranks call this),
        map the peers' buffers, then wait for every rank to have mapped.
        gather(own_handle) -> every rank's handle in rank order replaces the
        process-group exchange (and the barrier)."""
        mine = self.ipc_handle()
        if gather is None:
            handles = [None] * self.world
            dist.all_gather_object(handles, mine, group=group)
        else:
            handles = gather(mine)
        if len(handles) != self.world or any(len(h) != N.EP_HANDLE_BYTES for h in handles):
            raise N.KQError("kq_ep_connect: malformed handle list")
        N.check(self.lib.kq_ep_connect(self.handle, b"".join(handles)), "kq_ep_connect")
        if gather is None:
            dist.barrier(group=group)

    @staticmethod
    def connect_local(exchanges):
        """Join contexts of this process on one device as ranks 0..n-1 (one-GPU emulation)."""
        arr = (ctypes.c_void_p * len(exchanges))(*[e.handle.value for e in exchanges])
        N.check(exchanges[0].lib.kq_ep_connect_local(arr, len(exchanges)), "kq_ep_connect_local")

    def status(self):
        """(KQ_DEV_* bits, (site, source, value seen, CTA) of the first wait that gave up)."""
        st = ctypes.c_uint32(0)
        site = (ctypes.c_uint32 * 4)()
        N.check(self.lib.kq_ep_status(self.handle, ctypes.byref(st), site, _stream()), "kq_ep_status")
        return st.value, tuple(site)

    def clear_status(self):
        N.check(self.lib.kq_ep_clear_status(self.handle, _stream()), "kq_ep_clear_status")

    def calls(self) -> int:
        v = ctypes.c_uint32(0)
        N.check(self.lib.kq_ep_calls(self.handle, ctypes.byref(v)), "kq_ep_calls")
        return v.value

    def close(self):
        if getattr(self, "handle", None) is not None and self.handle.value:
            self.lib.kq_ep_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class PeerExpertParallelMoE:
    """Expert-parallel routed MoE through kq_ep: rows cross NVLink as stores into
    the owners' buffers, counts never leave the device, and a layer is five
    launches plus the grouped expert MLP (graph-capturable; no host sync).

    placements: one ExpertPlacement for every layer, or a list indexed by layer.
    table: this rank's ExpertTable whose layer l holds placements[l].experts_of(rank)
    in local order (extra experts after them, e.g. a shared expert, are allowed).
    shared_id: local id of a shared expert held by every rank, run as one more
    slot of each token's row on its own rank (the exchange then has top_k + 1
    slots); forward() takes its per-token gate as `shared_gate`."""

    def __init__(self, placements, rank: int, top_k: int, table, exchange: PeerExchange,
                 shared_id: Optional[int] = None):
        self.rank, self.k, self.table, self.ex = rank, top_k, table, exchange
        self.shared_id = shared_id
        if exchange.top_k != top_k + (0 if shared_id is None else 1):
            raise ValueError("the exchange's slots must be top_k (+ 1 with a shared expert)")
        self.lib = N.load()
        self._pl = placements
        self._maps = {}
        need = int(self.lib.kq_ep_moe_workspace_size(exchange.handle, table.handle))
        self.ws = torch.zeros(max(need, 1), dtype=torch.uint8, device="cuda")

    def placement(self, layer: int) -> ExpertPlacement:
        return self._pl[layer] if isinstance(self._pl, (list, tuple)) else self._pl

    def maps(self, layer: int, dev):
        key = layer if isinstance(self._pl, (list, tuple)) else 0
        m = self._maps.get(key)
        if m is None:
            pl = self.placement(layer)
            m = (torch.from_numpy(pl.owner.astype(np.int32)).to(dev),
                 torch.from_numpy(pl.local.astype(np.int32)).to(dev), len(pl.owner))
            self._maps[key] = m
        return m

    def route(self, logits=None, idx=None, weights=None):
        if logits is not None:
            return gpu_router(logits, self.k)
        return idx.to(torch.int32).contiguous(), weights.to(torch.float32).contiguous()

    # the five steps (forward issues them in order; the one-GPU emulation interleaves ranks)
    def dispatch(self, layer, x, idx, w, shared_gate=None):
        owner, local, E = self.maps(layer, x.device)
        if x.dtype != self.ex.dtype:
            raise ValueError("x must be in the exchange dtype")
        if (shared_gate is None) != (self.shared_id is None):
            raise ValueError("shared_gate goes with a shared_id")
        N.check(self.lib.kq_ep_dispatch(self.ex.handle, _ptr(x), _ptr(idx), _ptr(w), x.shape[0], self.k, _ptr(owner),
                                        _ptr(local), E, self.shared_id if self.shared_id is not None else -1,
                                        _ptr(shared_gate), _stream()), "kq_ep_dispatch")

    def receive(self):
        N.check(self.lib.kq_ep_receive(self.ex.handle, None, None, None, None, _stream()), "kq_ep_receive")

    def compute(self, layer):
        N.check(self.lib.kq_ep_compute(self.ex.handle, self.table.handle, layer, _ptr(self.ws), self.ws.numel(),
                                       _stream()), "kq_ep_compute")

    def send_back(self):
        N.check(self.lib.kq_ep_return(self.ex.handle, _stream()), "kq_ep_return")

    def combine(self, T, residual=None, shared=None, gate=None, out_dtype=torch.float16, out=None):
        if out is None:
            out = torch.empty(T, self.ex.hidden, dtype=out_dtype, device="cuda")
        N.check(self.lib.kq_ep_combine(self.ex.handle, T, _ptr(residual),
                                       _DT[residual.dtype] if residual is not None else 0, _ptr(shared),
                                       _DT[shared.dtype] if shared is not None else 0, _ptr(gate), _ptr(out),
                                       _DT[out.dtype], _stream()), "kq_ep_combine")
        return out

    def forward(self, layer, x, logits=None, idx=None, weights=None, residual=None, shared=None, gate=None,
                out_dtype=None, out=None, shared_gate=None):
        """out [T, H] = residual + routed MoE of x (+ shared_gate * shared expert of x
        when the object has a shared_id) + gate * shared, for this rank's tokens."""
        T = x.shape[0]
        idx, w = self.route(logits, idx, weights)
        out_dtype = out_dtype or x.dtype
        if out is None:
            out = torch.empty(T, self.ex.hidden, dtype=out_dtype, device=x.device)
        owner, local, E = self.maps(layer, x.device)
        if (shared_gate is None) != (self.shared_id is None):
            raise ValueError("shared_gate goes with a shared_id")
        N.check(self.lib.kq_ep_moe(self.ex.handle, self.table.handle, layer, _ptr(x), T, _ptr(idx), _ptr(w), self.k,
                                   E, _ptr(owner), _ptr(local),
                                   self.shared_id if self.shared_id is not None else -1, _ptr(shared_gate),
                                   _ptr(residual),
                                   _DT[residual.dtype] if residual is not None else 0, _ptr(shared),
                                   _DT[shared.dtype] if shared is not None else 0, _ptr(gate), _ptr(out),
                                   _DT[out.dtype], _ptr(self.ws), self.ws.numel(), _stream()), "kq_ep_moe")
        return out


def emulate_ranks(moes, layer, xs, routes, residuals=None, shareds=None, gates=None, out_dtype=torch.float32,
                  shared_gates=None):
    """Run one layer of n emulated ranks (PeerExpertParallelMoE objects joined by
    PeerExchange.connect_local) on one GPU and one stream: every dispatch, then
    every receive + compute, then every return, then every combine, so each
    wait finds its flags already set.  routes[r] = (idx, weights)."""
    n = len(moes)
    for r in range(n):
        moes[r].dispatch(layer, xs[r], *routes[r], shared_gate=None if shared_gates is None else shared_gates[r])
    for r in range(n):
        moes[r].receive()
        moes[r].compute(layer)
    for r in range(n):
        moes[r].send_back()
    return [moes[r].combine(xs[r].shape[0], residual=None if residuals is None else residuals[r],
                            shared=None if shareds is None else shareds[r],
                            gate=None if gates is None else gates[r], out_dtype=out_dtype) for r in range(n)]
