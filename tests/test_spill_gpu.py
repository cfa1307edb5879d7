"""GPU tests of the expert spill (kq_spill_*): host-pinned table, HBM slot pool.

* residency decisions against a Python model of the documented policy
  (hits keep their slot; misses in expert-id order take the least recently
  used slots not named by the call, ties to the lowest slot);
* routed-MLP results on the spilled table bit-identical to the resident
  table's (the same kernels read the same bytes from a different slot), and
  within 2e-3 relative L2 of the oracle;
* prefetch on the second stream, CUDA-graph capture, status bits."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu
RTOL_L2 = 2e-3


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


def to_dev(layer: O.ExpertLayer):
    out = []
    for m in range(3):
        w = torch.from_numpy(layer.w[m].view(np.uint8).reshape(layer.num_experts, layer.w[m].shape[1], -1)).cuda()
        s = torch.from_numpy(layer.s[m].view(np.int16)).cuda()
        b = torch.from_numpy(layer.b[m].view(np.int16)).cuda()
        out.append((w, s, b))
    return out


LAYERS = {}


def get_layers(n, bits=3, H=2048, I=512, E=32, sb="f16"):
    key = (n, bits, H, I, E, sb)
    if key not in LAYERS:
        LAYERS[key] = [O.ExpertLayer.random(bits, H, I, E, seed=100 + l, sb_dtype=sb) for l in range(n)]
    return LAYERS[key]


def build(layers, slots):
    """(resident ExpertTable, SpillTable) holding the same layers."""
    from kandiga_b200.experts import ExpertTable
    from kandiga_b200.spill import SpillTable
    L0 = layers[0]
    res = ExpertTable(len(layers), L0.num_experts, L0.hidden, L0.inter, L0.bits, L0.sb_dtype, L0.act)
    sp = SpillTable(len(layers), L0.num_experts, L0.hidden, L0.inter, slots, L0.bits, L0.sb_dtype, L0.act)
    for l, layer in enumerate(layers):
        g, u, d = to_dev(layer)
        res.load_mlx(l, g, u, d)
        sp.load_mlx(l, g, u, d)
    torch.cuda.synchronize()
    return res, sp


class PolicyModel:
    """The residency policy of kq_spill_fetch / kq_spill_prefetch, one layer."""

    def __init__(self, E, S):
        self.E, self.S = E, S
        self.slot_of = np.full(E, -1, np.int32)
        self.owner = np.full(S, -1, np.int32)
        self.stamp = np.zeros(S, np.int64)
        self.clock = 0
        self.hits = self.misses = 0
        self.status = 0

    def call(self, ids, fetch=True):
        t = self.clock + 1
        valid = [int(e) for e in ids if 0 <= e < self.E]
        if len(valid) != len(ids):
            self.status |= 1
        req = sorted(set(valid))
        miss = []
        for e in req:
            s = self.slot_of[e]
            if s >= 0:
                self.stamp[s] = t
                self.hits += 1
            else:
                miss.append(e)
        cand = sorted((s for s in range(self.S) if self.stamp[s] != t), key=lambda s: (self.stamp[s], s))
        served = min(len(miss), len(cand))
        for r in range(served):
            s, e = cand[r], miss[r]
            old = self.owner[s]
            if old >= 0:
                self.slot_of[old] = -1
            self.owner[s] = e
            self.slot_of[e] = s
            self.stamp[s] = t
        if fetch and served < len(miss):
            self.status |= 8
        self.misses += served
        self.clock = t
        return np.array([self.slot_of[e] if 0 <= e < self.E else -1 for e in ids], np.int32)


def test_spill_policy_matches_model(gpu):
    from kandiga_b200.spill import SpillTable
    E, S, L = 64, 12, 2
    sp = SpillTable(L, E, 512, 512, S, 3)
    models = [PolicyModel(E, S) for _ in range(L)]
    rng = np.random.RandomState(5)
    for step in range(60):
        layer = step % L if step < 40 else rng.randint(L)
        n = int(rng.choice([1, 4, 8, 8, 16, 20]))
        hot = rng.rand() < 0.5
        ids = (rng.choice(16, n) if hot else rng.randint(0, E, n)).astype(np.int32)
        fetch = rng.rand() < 0.8
        want = models[layer].call(ids, fetch)
        dev = torch.from_numpy(ids).cuda()
        if fetch:
            got = sp.fetch(layer, dev).cpu().numpy()
            assert np.array_equal(got, want), (step, ids, got, want)
        else:
            sp.prefetch(layer, dev)
            torch.cuda.current_stream().wait_stream(sp.prefetch_stream)
        slot_of, owner = sp.residency(layer)
        assert np.array_equal(slot_of, models[layer].slot_of), step
        assert np.array_equal(owner, models[layer].owner), step
    st = sp.stats()
    assert st["hits"] == sum(m.hits for m in models)
    assert st["misses"] == sum(m.misses for m in models)
    assert st["bytes"] == st["misses"] * sp.expert_bytes
    assert st["status"] == (models[0].status | models[1].status)


def test_spill_decode_bit_identical_to_resident(gpu):
    layers = get_layers(2)
    res, sp = build(layers, slots=12)
    E, H, K = 32, 2048, 8
    rng = np.random.RandomState(3)
    for step in range(16):
        l = step % 2
        T = 1 if step < 12 else 2  # T * K = 16 > 12 slots: two runs of one token
        x = torch.from_numpy(rng.randn(T, H).astype(np.float16)).cuda()
        logits = torch.from_numpy(rng.randn(T, E).astype(np.float32)).cuda()
        resid = torch.from_numpy(rng.randn(T, H).astype(np.float16)).cuda()
        a = res.moe(l, x, logits=logits, top_k=K, per_k=True, combine=True, residual=resid,
                    out_dtype=torch.float16, path="decode")
        b = sp.moe(l, x, logits=logits, top_k=K, per_k=True, combine=True, residual=resid,
                   out_dtype=torch.float16, path="decode")
        assert torch.equal(a["idx"], b["idx"])
        assert torch.equal(a["per_k"], b["per_k"]), step
        assert torch.equal(a["out"], b["out"]), step
    # and against the oracle for the last step
    idx = b["idx"].cpu().numpy()
    y = layers[l].moe(x.float().cpu().numpy(), idx)
    want = O.combine(y, b["weights"].cpu().numpy(), resid.float().cpu().numpy())
    assert rel_l2(b["out"].float().cpu().numpy(), want) < RTOL_L2
    st = sp.stats()
    assert st["status"] == 0 and st["misses"] > 0 and st["hits"] > 0
    assert sp.status() == 0 and res.status() == 0


def test_spill_prefill_runs_match_resident(gpu):
    """T * K distinct experts far above the slots: the tokens run in pieces
    that fit; per-token results equal the resident table's."""
    layers = get_layers(1, bits=4)
    res, sp = build(layers, slots=20)
    E, H, K, T = 32, 2048, 8, 96
    rng = np.random.RandomState(9)
    x = torch.from_numpy(rng.randn(T, H).astype(np.float16)).cuda()
    logits = torch.from_numpy(rng.randn(T, E).astype(np.float32)).cuda()
    a = res.moe(0, x, logits=logits, top_k=K, per_k=True, combine=True, out_dtype=torch.float32, path="prefill")
    b = sp.moe(0, x, logits=logits, top_k=K, per_k=True, combine=True, out_dtype=torch.float32, path="prefill")
    assert torch.equal(a["idx"], b["idx"])
    from kandiga_b200.spill import token_runs
    assert len(token_runs(b["idx"].cpu().numpy(), E, 20)) > 1
    assert rel_l2(b["per_k"].cpu().numpy(), a["per_k"].cpu().numpy()) < 1e-6
    assert rel_l2(b["out"].cpu().numpy(), a["out"].cpu().numpy()) < 1e-6
    assert sp.stats()["status"] == 0 and sp.status() == 0


def test_spill_prefetch_makes_next_layer_resident(gpu):
    layers = get_layers(2)
    res, sp = build(layers, slots=16)
    E, H, K = 32, 2048, 8
    rng = np.random.RandomState(21)
    router = torch.from_numpy(rng.randn(E, H).astype(np.float32) * 0.05).cuda()
    x = torch.from_numpy(rng.randn(1, H).astype(np.float16)).cuda()
    sp.moe(0, x, logits=torch.randn(1, E, device="cuda"), top_k=K, combine=True, weights=None,
           out_dtype=torch.float32)
    pred = sp.predict_and_prefetch(0, x, router, top_k=K)
    sp.stats(reset=True)
    logits1 = (x.float() @ router.t()).contiguous()  # the next layer routes as predicted
    b = sp.moe(1, x, logits=logits1, top_k=K, combine=True, out_dtype=torch.float32)
    st = sp.stats()
    assert torch.equal(torch.sort(b["idx"], dim=1).values, torch.sort(pred, dim=1).values)
    assert st["misses"] == 0 and st["hits"] == K, st
    a = res.moe(1, x, logits=logits1, top_k=K, combine=True, out_dtype=torch.float32)
    assert torch.equal(a["out"], b["out"])


def test_spill_decode_in_cuda_graph(gpu):
    """router top-K -> fetch (assign + copy) -> decode kernels, captured once,
    replayed with new logits: the residency follows every replay."""
    layers = get_layers(1)
    res, sp = build(layers, slots=10)
    E, H, K = 32, 2048, 8
    x = torch.randn(1, H, device="cuda", dtype=torch.float16)
    logits = torch.randn(1, E, device="cuda")
    sp.moe(0, x, logits=logits, top_k=K, combine=True, out_dtype=torch.float32)  # workspaces before capture
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            r = sp.moe(0, x, logits=logits, top_k=K, combine=True, out_dtype=torch.float32)
    rng = np.random.RandomState(4)
    for _ in range(8):
        logits.copy_(torch.from_numpy(rng.randn(1, E).astype(np.float32)))
        x.copy_(torch.from_numpy(rng.randn(1, H).astype(np.float16)))
        g.replay()
        torch.cuda.synchronize()
        want = res.moe(0, x, logits=logits, top_k=K, combine=True, out_dtype=torch.float32)
        assert torch.equal(r["out"], want["out"])
    assert sp.stats()["status"] == 0


def test_spill_capacity_and_bad_ids(gpu):
    from kandiga_b200 import _native as N
    from kandiga_b200.spill import SpillTable
    sp = SpillTable(1, 16, 512, 512, 4, 3)
    ids = torch.tensor([9, 1, 3, 5, 7, 1, 11], dtype=torch.int32, device="cuda")
    slot = sp.fetch(0, ids).cpu().numpy()
    # six distinct experts, four slots: the four lowest ids (1, 3, 5, 7) are served
    assert list(slot[[1, 2, 3, 4, 5]] >= 0) == [True] * 5
    assert slot[0] == -1 and slot[6] == -1
    assert sp.stats(reset=True)["status"] == N.DEV_CAPACITY
    slot = sp.fetch(0, torch.tensor([-1, 2, 16], dtype=torch.int32, device="cuda")).cpu().numpy()
    assert slot[0] == -1 and slot[2] == -1 and slot[1] >= 0
    assert sp.stats()["status"] == N.DEV_BAD_EXPERT


def test_spill_store_layer_empties_residency(gpu):
    layers = get_layers(1)
    res, sp = build(layers, slots=10)
    sp.fetch(0, torch.arange(8, dtype=torch.int32, device="cuda"))
    slot_of, owner = sp.residency(0)
    assert (owner >= 0).sum() == 8
    sp.store_layer(0, res, 0)
    slot_of, owner = sp.residency(0)
    assert (slot_of == -1).all() and (owner == -1).all()
    assert sp.host_bytes == 32 * sp.expert_bytes
