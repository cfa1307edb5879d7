"""Expert parallelism over peer memory (kq_ep_*) on one GPU.

n ranks are emulated by n exchange contexts in this process joined by plain
pointers (kq_ep_connect_local); each rank's table holds only its own experts.
Every rank's dispatch is issued before any receive and every return before any
combine, on one stream, so no wait is ever pending (the kernels never wait on
one another).  Results are compared with the C oracle of the reference's
per-token expert path (kandiga/metal/kandiga_cpu_expert.m:471-552, blend
kandiga/metal/moe_block.metal:556-584): 2e-3 relative L2 on the routed part of
every output row."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.test_decode_gpu import get_layer, make_table, rel_l2

pytestmark = pytest.mark.gpu
RTOL_L2 = 2e-3


def rank_tables(layer, pl):
    tabs = []
    for r in range(pl.world):
        ids = pl.experts_of(r)
        sub = O.ExpertLayer(layer.bits, layer.hidden, layer.inter, [m[ids] for m in layer.w],
                            [m[ids] for m in layer.s], [m[ids] for m in layer.b], layer.sb_dtype, layer.act)
        tabs.append(make_table(sub))
    return tabs


def setup(layer, world, K, max_tokens, dtype=torch.float16, placement="balanced", wait_ns=None):
    from kandiga_b200.ep import ExpertPlacement, PeerExchange, PeerExpertParallelMoE, zipf_bias
    E = layer.num_experts
    pl = (ExpertPlacement.balanced(np.exp(zipf_bias(E, 1.1, 4)), world) if placement == "balanced"
          else ExpertPlacement.contiguous(E, world))
    tabs = rank_tables(layer, pl)
    exs = [PeerExchange(r, world, max_tokens, layer.hidden, K, dtype, wait_ns=wait_ns) for r in range(world)]
    PeerExchange.connect_local(exs)
    moes = [PeerExpertParallelMoE(pl, r, K, tabs[r], exs[r]) for r in range(world)]
    return pl, tabs, exs, moes


def routed_oracle(layer, x, idx, w):
    y = layer.moe(x.float().cpu().numpy(), idx.cpu().numpy())
    return O.combine(y, w.cpu().numpy(), None)


def inputs(T, H, E, K, seed, dtype=torch.float16):
    rng = np.random.RandomState(seed)
    x = torch.from_numpy(rng.randn(T, H).astype(np.float32)).to(dtype).cuda()
    logits = (rng.randn(T, E) + np.linspace(0, -2, E)).astype(np.float32)
    idx, w = O.router_topk(logits, K)
    return x, torch.from_numpy(idx).cuda(), torch.from_numpy(w).cuda()


@pytest.mark.parametrize("world,Ts", [(1, [40]), (1, [5]), (2, [20, 13]), (2, [3, 2]), (3, [7, 0, 12]),
                                      (4, [16, 16, 1, 9])])
def test_emulated_ranks_match_oracle(gpu, world, Ts):
    """rows = world * max_tokens >= 16 takes the grouped path, fewer the decode path;
    a rank with no tokens still dispatches, returns and combines."""
    from kandiga_b200.ep import emulate_ranks
    E, H, I, K = 16, 1024, 512, 4
    layer = get_layer(3, H, I, E, "f16", seed=80)
    pl, tabs, exs, moes = setup(layer, world, K, max(Ts))
    data = [inputs(T, H, E, K, 90 + r) for r, T in enumerate(Ts)]
    xs = [d[0] for d in data]
    res = [torch.randn(T, H, device="cuda") for T in Ts]
    outs = emulate_ranks(moes, 0, xs, [(d[1], d[2]) for d in data], residuals=res, out_dtype=torch.float32)
    torch.cuda.synchronize()
    for r in range(world):
        st, site = exs[r].status()
        assert st == 0, (r, st, site)
        assert tabs[r].status() == 0
        if Ts[r] == 0:
            assert outs[r].shape[0] == 0
            continue
        want = routed_oracle(layer, xs[r], data[r][1], data[r][2])
        got = (outs[r] - res[r]).cpu().numpy()
        assert rel_l2(got, want) < RTOL_L2, (r, rel_l2(got, want))
    assert all(e.calls() == 1 for e in exs)


def test_bf16_rows_shared_expert_and_gate(gpu):
    """bf16 exchange; the owner adds gate[t] * shared[t] and a bf16 residual."""
    from kandiga_b200.ep import emulate_ranks
    E, H, I, K, T = 12, 1024, 512, 3, 24
    layer = get_layer(4, H, I, E, "bf16", seed=81)
    pl, tabs, exs, moes = setup(layer, 2, K, T, dtype=torch.bfloat16, placement="contiguous")
    data = [inputs(T, H, E, K, 95 + r, torch.bfloat16) for r in range(2)]
    xs = [d[0] for d in data]
    shared = [torch.randn(T, H, device="cuda").to(torch.bfloat16) for _ in range(2)]
    gate = [torch.rand(T, device="cuda") for _ in range(2)]
    res = [torch.randn(T, H, device="cuda").to(torch.bfloat16) for _ in range(2)]
    outs = emulate_ranks(moes, 0, xs, [(d[1], d[2]) for d in data], residuals=res, shareds=shared, gates=gate,
                         out_dtype=torch.float32)
    for r in range(2):
        assert exs[r].status()[0] == 0
        want = routed_oracle(layer, xs[r], data[r][1], data[r][2])
        got = (outs[r] - res[r].float() - gate[r][:, None] * shared[r].float()).cpu().numpy()
        assert rel_l2(got, want) < RTOL_L2


def test_empty_slots_and_bad_ids(gpu):
    """-1 is an empty slot (no status); an id outside [0, E) latches
    KQ_DEV_BAD_EXPERT and is dropped; the other slots are still computed."""
    from kandiga_b200 import _native as N
    from kandiga_b200.ep import emulate_ranks
    E, H, I, K, T = 8, 1024, 512, 4, 6
    layer = get_layer(3, H, I, E, "f16", seed=82)
    pl, tabs, exs, moes = setup(layer, 2, K, T)
    x, idx, w = inputs(T, H, E, K, 7)
    idx2 = idx.clone()
    idx2[1, 2] = -1
    x1, i1, w1 = inputs(T, H, E, K, 8)
    outs = emulate_ranks(moes, 0, [x, x1], [(idx2, w), (i1, w1)], out_dtype=torch.float32)
    assert exs[0].status()[0] == 0
    keep = idx2.cpu().numpy()
    wk = w.cpu().numpy().copy()
    wk[keep < 0] = 0
    want = O.combine(layer.moe(x.float().cpu().numpy(), np.maximum(keep, 0)), wk, None)
    assert rel_l2(outs[0].cpu().numpy(), want) < RTOL_L2
    idx3 = idx.clone()
    idx3[4, 0] = 999
    emulate_ranks(moes, 0, [x, x1], [(idx3, w), (i1, w1)], out_dtype=torch.float32)
    assert exs[0].status()[0] & N.DEV_BAD_EXPERT


def test_layers_in_one_graph_replayed(gpu):
    """Three layers of two emulated ranks captured in one CUDA graph: the flags
    only grow, so replays need no reset and give identical results."""
    from kandiga_b200.ep import emulate_ranks
    E, H, I, K, T, L = 16, 1024, 512, 4, 20, 3
    layer = get_layer(3, H, I, E, "f16", seed=83)
    pl, tabs, exs, moes = setup(layer, 2, K, T)
    data = [inputs(T, H, E, K, 60 + r) for r in range(2)]
    routes = [(d[1], d[2]) for d in data]
    xs0 = [d[0] for d in data]
    outs = {}

    def step():
        xs = xs0
        for _ in range(L):
            xs = emulate_ranks(moes, 0, xs, routes, residuals=xs, out_dtype=torch.float16)
        outs["y"] = xs

    step()
    torch.cuda.synchronize()
    first = [y.clone() for y in outs["y"]]
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            step()
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    for r in range(2):
        assert torch.equal(outs["y"][r], first[r])
        assert exs[r].status()[0] == 0
        assert exs[r].calls() == L * 4
    del g


def test_wait_that_nobody_satisfies_times_out(gpu):
    """Rank 1 never dispatches: rank 0's receive gives up after the 50 ms bound,
    latches KQ_DEV_WAIT_TIMEOUT with the site (receive, source 1, flag 0), treats
    rank 1's rows as empty, and the combine that follows gives up at once."""
    import time
    from kandiga_b200 import _native as N
    E, H, I, K, T = 8, 1024, 512, 2, 4
    layer = get_layer(3, H, I, E, "f16", seed=84)
    pl, tabs, exs, moes = setup(layer, 2, K, T, wait_ns=50_000_000)
    x, idx, w = inputs(T, H, E, K, 3)
    t0 = time.time()
    moes[0].dispatch(0, x, idx, w)
    moes[0].receive()
    moes[0].compute(0)
    moes[0].send_back()
    out = moes[0].combine(T, out_dtype=torch.float32)
    st, site = exs[0].status()
    dt = time.time() - t0
    assert st & N.DEV_WAIT_TIMEOUT
    assert site[:3] == (1, 1, 0)
    assert torch.isfinite(out).all()
    assert dt < 5.0
    exs[0].clear_status()
    assert exs[0].status()[0] == 0


@pytest.mark.parametrize("world,Ts", [(2, [24, 9]), (3, [5, 16, 0])])
def test_shared_expert_as_own_rank_slot(gpu, world, Ts):
    """A shared expert held by every rank (the last expert of each rank's table)
    runs as slot K of the token's row on its own rank, weighted by its gate:
    out = res + sum_k w_k y_k + gate * y_shared, against the oracle with the
    shared expert as assignment K + 1."""
    from kandiga_b200.ep import (ExpertPlacement, PeerExchange, PeerExpertParallelMoE, emulate_ranks,
                                 zipf_bias)
    E, H, I, K = 12, 1024, 512, 3
    full = get_layer(3, H, I, E + 1, "f16", seed=85)  # expert E is the shared one
    pl = ExpertPlacement.balanced(np.exp(zipf_bias(E, 1.1, 5)), world)
    tabs, moes, exs = [], [], []
    for r in range(world):
        ids = np.concatenate([pl.experts_of(r), [E]])
        sub = O.ExpertLayer(full.bits, H, I, [m[ids] for m in full.w], [m[ids] for m in full.s],
                            [m[ids] for m in full.b], full.sb_dtype, full.act)
        tabs.append(make_table(sub))
        exs.append(PeerExchange(r, world, max(Ts), H, K + 1))
    PeerExchange.connect_local(exs)
    for r in range(world):
        moes.append(PeerExpertParallelMoE(pl, r, K, tabs[r], exs[r], shared_id=len(pl.experts_of(r))))
    data = [inputs(T, H, E, K, 40 + r) for r, T in enumerate(Ts)]
    gates = [torch.rand(T, device="cuda") for T in Ts]
    res = [torch.randn(T, H, device="cuda") for T in Ts]
    outs = emulate_ranks(moes, 0, [d[0] for d in data], [(d[1], d[2]) for d in data], residuals=res,
                         out_dtype=torch.float32, shared_gates=gates)
    for r in range(world):
        assert exs[r].status()[0] == 0 and tabs[r].status() == 0
        if Ts[r] == 0:
            continue
        idx = np.concatenate([data[r][1].cpu().numpy(), np.full((Ts[r], 1), E, np.int32)], 1)
        w = np.concatenate([data[r][2].cpu().numpy(), gates[r].cpu().numpy()[:, None]], 1)
        want = O.combine(full.moe(data[r][0].float().cpu().numpy(), idx), w, None)
        assert rel_l2((outs[r] - res[r]).cpu().numpy(), want) < RTOL_L2
