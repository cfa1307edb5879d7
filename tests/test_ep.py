"""Expert-parallel exchange logic on CPU: world-size 2 and 3 gloo ranks run
ExpertParallelMoE with the oracle as the expert compute and compare every
per-expert output and the combined rows with a single-process run over the
whole layer (the expert MLP of one (token, expert) pair is the same
computation on either side, so per-expert outputs are bit-identical)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from kandiga_b200.ep import ExpertParallelMoE, ExpertPlacement, zipf_bias
from oracle import oracle as O

E, H, I, K, BITS = 8, 256, 128, 2, 4


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def make_layer():
    return O.ExpertLayer.random(BITS, H, I, E, seed=5, sb_dtype="f16")


def sub_layer(layer, ids):
    return O.ExpertLayer(BITS, H, I, [m[ids] for m in layer.w], [m[ids] for m in layer.s], [m[ids] for m in layer.b],
                         "f16", "silu")


def cpu_router(logits, k):
    idx, w = O.router_topk(logits.numpy(), k)
    return torch.from_numpy(idx), torch.from_numpy(w)


def cpu_combine(per_k, w, residual=None, shared=None, gate=None, out_dtype=None):
    out = (per_k.float() * w[..., None]).sum(1)
    if shared is not None:
        out = out + (gate[:, None] if gate is not None else 1.0) * shared.float()
    if residual is not None:
        out = out + residual.float()
    return out


def tokens_of(rank):
    rng = np.random.RandomState(100 + rank)
    T = 5 + rank
    x = rng.randn(T, H).astype(np.float32)
    logits = (rng.randn(T, E) + zipf_bias(E, 1.1, 3)).astype(np.float32)
    res = rng.randn(T, H).astype(np.float32)
    return x, logits, res


def worker(rank, world, port, mode, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        layer = make_layer()
        if mode == "balanced":
            load = np.exp(zipf_bias(E, 1.1, 3))
            pl = ExpertPlacement.balanced(load, world)
        else:
            pl = ExpertPlacement.contiguous(E, world)
        mine = sub_layer(layer, pl.experts_of(rank))

        def compute(lay, rows, ids):
            if rows.shape[0] == 0:
                return rows.clone()
            y = mine.moe(rows.numpy().astype(np.float32), ids.numpy().reshape(-1, 1).astype(np.int32))
            return torch.from_numpy(y.reshape(rows.shape[0], H))

        ep = ExpertParallelMoE(pl, rank, K, compute, router=cpu_router, combine=cpu_combine)
        x, logits, res = tokens_of(rank)
        out, parts = ep.forward(0, torch.from_numpy(x), torch.from_numpy(logits), residual=torch.from_numpy(res),
                                return_parts=True)
        q.put((rank, out.numpy(), parts["per_k"].numpy(), parts["idx"].numpy(), parts["send"], parts["recv"]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,mode", [(2, "contiguous"), (2, "balanced"), (3, "balanced")])
def test_ep_matches_single_process(world, mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = {}
    for _ in range(world):
        r, out, per_k, idx, send, recv = q.get(timeout=120)
        got[r] = (out, per_k, idx, send, recv)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    layer = make_layer()
    total_send = np.zeros((world, world), np.int64)
    for r in range(world):
        out, per_k, idx, send, recv = got[r]
        x, logits, res = tokens_of(r)
        idx_ref, w_ref = O.router_topk(logits, K)
        assert np.array_equal(idx, idx_ref)
        y = layer.moe(x, idx_ref)
        assert np.array_equal(per_k, y)
        want = (y * w_ref[..., None]).sum(1) + res
        np.testing.assert_allclose(out, want, rtol=1e-6, atol=1e-6)
        total_send[r] = send
    for r in range(world):
        assert got[r][4] == [int(total_send[s, r]) for s in range(world)]


def test_balanced_placement_properties():
    load = np.exp(zipf_bias(256, 1.1, 0))
    pl = ExpertPlacement.balanced(load, 8)
    assert np.array_equal(np.bincount(pl.owner, minlength=8), np.full(8, 32))
    per = np.array([load[pl.owner == r].sum() for r in range(8)])
    assert per.max() <= per.min() + load.max() + 1e-9  # greedy largest-first bound
    rr = ExpertPlacement.contiguous(256, 8)
    per_c = np.array([load[rr.owner == r].sum() for r in range(8)])
    assert per.max() <= per_c.max()
    for r in range(8):
        ids = pl.experts_of(r)
        assert np.array_equal(pl.local[ids], np.arange(len(ids)))


class _FakeEpLib:
    """Stand-in for the five libkq calls PeerExchange makes on the host side
    (the real ones allocate and map device memory)."""

    def __init__(self, rank):
        self.rank = rank
        self.connected = None

    def kq_ep_create(self, rank, world, max_tokens, hidden, top_k, dtype, out):
        out._obj.value = 1000 + rank
        return 0

    def kq_ep_ipc_handle(self, h, buf):
        import ctypes
        ctypes.memmove(buf, bytes([h.value - 1000]) * 64, 64)
        return 0

    def kq_ep_connect(self, h, blob):
        self.connected = bytes(blob)
        return 0

    def kq_ep_destroy(self, h):
        pass


def peer_worker(rank, world, port, q):
    import kandiga_b200._native as N
    from kandiga_b200 import ep as EP
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        fake = _FakeEpLib(rank)
        N.load = lambda *a, **k: fake  # the exchange object binds whatever load() returns
        ex = EP.PeerExchange(rank, world, 16, 1024, 4)
        ex.connect()
        q.put((rank, fake.connected))
        ex.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_peer_exchange_handles_in_rank_order(world):
    """PeerExchange.connect gathers every rank's 64-byte IPC handle over the
    process group and passes them to kq_ep_connect in rank order."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=peer_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = b"".join(bytes([r]) * 64 for r in range(world))
    assert all(got[r] == want for r in range(world))


def test_peer_moe_checks_slot_count():
    """The exchange's slots must be top_k, or top_k + 1 with a shared expert."""
    from kandiga_b200 import ep as EP

    class Ex:
        top_k = 8
        handle = None

    with pytest.raises(ValueError):
        EP.PeerExpertParallelMoE(EP.ExpertPlacement.contiguous(8, 1), 0, 8, None, Ex(), shared_id=8)
