"""GPU parity of the streaming batch decode (kq_moe_decode_batch): n independent
single-token items, each the reference's per-token expert path
(kandiga/metal/kandiga_cpu_expert.m:471-552, routing
kandiga/metal/moe_block.metal:419-505, blend :556-584), against the C oracle.
Tolerance: 2e-3 relative L2 per (item, k) expert output and per combined row;
router indices bit-exact; two runs bit-identical."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.test_decode_gpu import get_layer, make_table, rel_l2, to_dev

pytestmark = pytest.mark.gpu
RTOL_L2 = 2e-3


def multi_layer_table(layers):
    from kandiga_b200.experts import ExpertTable
    l0 = layers[0]
    t = ExpertTable(len(layers), l0.num_experts, l0.hidden, l0.inter, l0.bits, l0.sb_dtype, l0.act)
    for i, lay in enumerate(layers):
        t.load_mlx(i, *to_dev(lay))
    torch.cuda.synchronize()
    return t


def check_items(layers_np, layer_of, x, idx, w, r, res=None, norm=None, eps=1e-6):
    xf = x.float().cpu().numpy()
    if norm is not None:
        nw = norm.float().cpu().numpy()
        xf = xf / np.sqrt(np.mean(xf * xf, axis=1, keepdims=True) + eps) * nw
    n, K = idx.shape
    for j in range(n):
        y = layers_np[layer_of[j]].moe(xf[j:j + 1], idx[j:j + 1])
        if r["per_k"] is not None:
            pk = r["per_k"][j].float().cpu().numpy()
            worst = max(rel_l2(pk[k], y[0, k]) for k in range(K))
            assert worst < RTOL_L2, (j, worst)
        if r["out"] is not None:
            want = O.combine(y, w[j:j + 1], None if res is None else res[j:j + 1].float().cpu().numpy())
            got = r["out"][j:j + 1].float().cpu().numpy()
            assert rel_l2(got, want) < RTOL_L2, (j, rel_l2(got, want))


@pytest.mark.parametrize("bits,sb", [(3, "f16"), (4, "bf16")])
def test_batch_one_layer_matches_oracle(gpu, bits, sb):
    E, H, I, K, n = 32, 2048, 512, 8, 24
    layer = get_layer(bits, H, I, E, sb, seed=50 + bits)
    t = make_table(layer)
    rng = np.random.RandomState(bits)
    x = torch.from_numpy(rng.randn(n, H).astype(np.float16)).cuda()
    logits = torch.from_numpy(rng.randn(n, E).astype(np.float32)).cuda()
    r = t.decode_batch(x, logits=logits, top_k=K, per_k=True, combine=True, out_dtype=torch.float32)
    idx_ref, _ = O.router_topk(logits.cpu().numpy(), K)
    assert np.array_equal(r["idx"].cpu().numpy(), idx_ref)
    check_items([layer], [0] * n, x, idx_ref, r["weights"].cpu().numpy(), r)
    assert t.batch_status() == 0
    r2 = t.decode_batch(x, logits=logits, top_k=K, per_k=True, combine=True, out_dtype=torch.float32)
    assert torch.equal(r["out"], r2["out"]) and torch.equal(r["per_k"], r2["per_k"])
    # agrees with the per-call decode path
    d = t.moe(0, x, logits=logits, top_k=K, per_k=True, combine=True, out_dtype=torch.float32, path="decode")
    assert rel_l2(r["out"].cpu().numpy(), d["out"].cpu().numpy()) < RTOL_L2


def test_batch_items_across_layers_long_stream(gpu):
    """300 items over 3 layers with different weights: the rings of items,
    activations and partial sums wrap around many times."""
    E, H, I, K, n = 16, 1024, 512, 8, 300
    lays = [get_layer(3, H, I, E, "f16", seed=60 + i) for i in range(3)]
    t = multi_layer_table(lays)
    rng = np.random.RandomState(7)
    layer_of = rng.randint(0, 3, n).astype(np.int32)
    x = torch.from_numpy(rng.randn(n, H).astype(np.float16)).cuda()
    logits = torch.from_numpy(rng.randn(n, E).astype(np.float32)).cuda()
    lt = torch.from_numpy(layer_of).cuda()
    r = t.decode_batch(x, layers=lt, logits=logits, top_k=K, per_k=True, combine=True, out_dtype=torch.float32)
    idx = r["idx"].cpu().numpy()
    rows = list(range(0, n, 23)) + [n - 1]
    check_items(lays, layer_of[rows], x[rows], idx[rows], r["weights"].cpu().numpy()[rows],
                dict(out=r["out"][rows], per_k=r["per_k"][rows]))
    assert t.batch_status() == 0


@pytest.mark.parametrize("K", [9, 3, 1])
def test_batch_expert_groups_residual_norm(gpu, K):
    """K = 9: three expert groups per down row tile (the last to arrive adds
    all three); bf16 input with an RMSNorm prologue; fp32 residual."""
    E, H, I, n = 24, 2048, 1024, 10
    layer = get_layer(3, H, I, E, "bf16", seed=70)
    t = make_table(layer)
    rng = np.random.RandomState(K)
    x = torch.from_numpy(rng.randn(n, H).astype(np.float32) * 3).to(torch.bfloat16).cuda()
    norm = torch.from_numpy((1 + 0.1 * rng.randn(H)).astype(np.float32)).to(torch.bfloat16).cuda()
    logits = torch.from_numpy(rng.randn(n, E).astype(np.float32)).cuda()
    res = torch.from_numpy(rng.randn(n, H).astype(np.float32)).cuda()
    r = t.decode_batch(x, logits=logits, top_k=K, per_k=True, combine=True, residual=res, norm_w=norm,
                       out_dtype=torch.float32)
    check_items([layer], [0] * n, x, r["idx"].cpu().numpy(), r["weights"].cpu().numpy(), r, res=res, norm=norm)
    assert t.batch_status() == 0


def test_batch_given_routing_and_bad_expert(gpu):
    from kandiga_b200 import _native as N
    E, H, I, K, n = 8, 1024, 512, 4, 6
    layer = get_layer(4, H, I, E, "f16", seed=71)
    t = make_table(layer)
    rng = np.random.RandomState(3)
    x = torch.from_numpy(rng.randn(n, H).astype(np.float16)).cuda()
    idx = torch.from_numpy(rng.randint(0, E, (n, K)).astype(np.int32)).cuda()
    w = torch.from_numpy(rng.rand(n, K).astype(np.float32)).cuda()
    r = t.decode_batch(x, idx=idx, weights=w, per_k=True, combine=True, out_dtype=torch.float32)
    check_items([layer], [0] * n, x, idx.cpu().numpy(), w.cpu().numpy(), r)
    assert t.batch_status() == 0
    idx[2, 1] = 99
    r = t.decode_batch(x, idx=idx, weights=w, per_k=True, combine=False, out_dtype=torch.float32)
    assert t.batch_status() & N.DEV_BAD_EXPERT
    assert torch.count_nonzero(r["per_k"][2, 1]) == 0


def test_batch_small_shape_more_ctas_than_units(gpu):
    """H 512, I 128, K 2: 64 units per item, fewer than the SMs, so most CTAs
    have nothing to do for a given item and pass its ring slot on."""
    E, H, I, K, n = 8, 512, 128, 2, 10
    layer = get_layer(4, H, I, E, "f16", seed=72)
    t = make_table(layer)
    rng = np.random.RandomState(9)
    x = torch.from_numpy(rng.randn(n, H).astype(np.float16)).cuda()
    logits = torch.from_numpy(rng.randn(n, E).astype(np.float32)).cuda()
    r = t.decode_batch(x, logits=logits, top_k=K, per_k=True, combine=True, out_dtype=torch.float32)
    idx_ref, _ = O.router_topk(logits.cpu().numpy(), K)
    assert np.array_equal(r["idx"].cpu().numpy(), idx_ref)
    check_items([layer], [0] * n, x, idx_ref, r["weights"].cpu().numpy(), r)
    assert t.batch_status() == 0
