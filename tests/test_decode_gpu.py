"""GPU parity of the routed-expert decode path (libkq.so through its C ABI)
against the C oracle of the reference's scalar path.

Tolerance: expert-MLP outputs within 2e-3 relative L2 of the fp32 oracle
(per (token, k) vector); codes/scales/biases and router indices bit-exact."""
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


def make_table(layer: O.ExpertLayer, num_layers=1):
    from kandiga_b200.experts import ExpertTable
    t = ExpertTable(num_layers, layer.num_experts, layer.hidden, layer.inter, layer.bits, layer.sb_dtype,
                    layer.act)
    g, u, d = to_dev(layer)
    for l in range(num_layers):
        t.load_mlx(l, g, u, d)
    torch.cuda.synchronize()
    return t


LAYERS = {}


def get_layer(bits, hidden, inter, E, sb="f16", act="silu", seed=0):
    key = (bits, hidden, inter, E, sb, act, seed)
    if key not in LAYERS:
        LAYERS[key] = O.ExpertLayer.random(bits, hidden, inter, E, seed=seed, sb_dtype=sb, act=act)
    return LAYERS[key]


@pytest.mark.parametrize("bits,sb", [(3, "f16"), (4, "f16"), (3, "bf16"), (4, "bf16")])
def test_table_roundtrip_bit_exact(gpu, bits, sb):
    layer = get_layer(bits, 1024, 512, 3, sb, seed=bits)
    t = make_table(layer)
    for e in range(3):
        for m in range(3):
            w, s, b = t.unpack_mlx(0, e, m)
            assert np.array_equal(w.cpu().numpy().reshape(-1), layer.w[m][e].view(np.uint8).reshape(-1))
            assert np.array_equal(s.cpu().numpy().view(np.uint16), layer.s[m][e])
            assert np.array_equal(b.cpu().numpy().view(np.uint16), layer.b[m][e])


def test_table_roundtrip_edge_codes(gpu):
    """all-zero / all-max codes and byte-straddling patterns survive the repack."""
    layer = get_layer(3, 512, 512, 2, seed=5)
    for m in range(3):
        q = O.unpack_codes(layer.w[m][0], 3, layer.w[m][0].shape[1] * 8 // 3)
        q[:] = 7
        q[1::2, ::3] = 0
        q[2] = np.arange(q.shape[1]) % 8
        layer.w[m][0] = O.pack_codes(q, 3)
    t = make_table(layer)
    for m in range(3):
        w, s, b = t.unpack_mlx(0, 0, m)
        assert np.array_equal(w.cpu().numpy().reshape(-1), layer.w[m][0].reshape(-1))


@pytest.mark.parametrize("bits,sb,hidden,inter", [(3, "f16", 2048, 512), (4, "f16", 2048, 512),
                                                   (3, "bf16", 2048, 512), (4, "bf16", 1024, 1024),
                                                   (3, "f16", 3072, 1024)])
def test_decode_per_expert_matches_oracle(gpu, bits, sb, hidden, inter):
    E = 16
    layer = get_layer(bits, hidden, inter, E, sb, seed=1)
    t = make_table(layer)
    rng = np.random.RandomState(7)
    for T, K in ((1, 8), (3, 4), (2, 1)):
        x = rng.randn(T, hidden).astype(np.float16)
        idx = np.stack([rng.choice(E, K, replace=False) for _ in range(T)]).astype(np.int32)
        ref = layer.moe(x.astype(np.float32), idx)
        r = t.moe(0, torch.from_numpy(x).cuda(), idx=torch.from_numpy(idx).cuda(), per_k=True, combine=False,
                  out_dtype=torch.float32)
        got = r["per_k"].cpu().numpy()
        for ti in range(T):
            for k in range(K):
                assert rel_l2(got[ti, k], ref[ti, k]) < RTOL_L2, (T, K, ti, k, rel_l2(got[ti, k], ref[ti, k]))
        assert t.status() == 0


def test_decode_fused_router_and_combine(gpu):
    E, H, I, K = 32, 2048, 512, 8
    layer = get_layer(3, H, I, E, "f16", seed=2)
    t = make_table(layer)
    rng = np.random.RandomState(11)
    T = 4
    x = rng.randn(T, H).astype(np.float16)
    logits = rng.randn(T, E).astype(np.float32)
    logits[1, [5, 9]] = 4.0  # a tie at the top: lowest index first
    res = rng.randn(T, H).astype(np.float16)
    idx_ref, w_ref = O.router_topk(logits, K)
    r = t.moe(0, torch.from_numpy(x).cuda(), logits=torch.from_numpy(logits).cuda(), top_k=K, per_k=True,
              combine=True, residual=torch.from_numpy(res).cuda(), out_dtype=torch.float16)
    assert np.array_equal(r["idx"].cpu().numpy(), idx_ref)
    np.testing.assert_allclose(r["weights"].cpu().numpy(), w_ref, rtol=1e-5, atol=1e-7)
    y = layer.moe(x.astype(np.float32), idx_ref)
    out_ref = O.combine(y, w_ref, res.astype(np.float32))
    got = r["out"].float().cpu().numpy()
    for ti in range(T):
        assert rel_l2(got[ti], out_ref[ti]) < RTOL_L2
    # fp16 per-k outputs too
    pk = r["per_k"].float().cpu().numpy()
    for ti in range(T):
        for k in range(K):
            assert rel_l2(pk[ti, k], y[ti, k]) < RTOL_L2
    assert t.status() == 0


@pytest.mark.parametrize("xdt", [torch.bfloat16, torch.float32])
def test_decode_input_dtypes(gpu, xdt):
    E, H, I = 8, 2048, 512
    layer = get_layer(3, H, I, E, "bf16", seed=3)
    t = make_table(layer)
    rng = np.random.RandomState(3)
    x = torch.from_numpy(rng.randn(2, H).astype(np.float32) * 40.0).to(xdt).cuda()  # large magnitude
    idx = torch.tensor([[1, 4, 7], [0, 2, 5]], dtype=torch.int32, device="cuda")
    w = torch.rand(2, 3, device="cuda")
    r = t.moe(0, x, idx=idx, weights=w, per_k=True, combine=True, out_dtype=torch.float32)
    ref = layer.moe(x.float().cpu().numpy(), idx.cpu().numpy())
    got = r["per_k"].cpu().numpy()
    for ti in range(2):
        for k in range(3):
            assert rel_l2(got[ti, k], ref[ti, k]) < RTOL_L2
    out_ref = O.combine(ref, w.cpu().numpy())
    assert rel_l2(r["out"].cpu().numpy(), out_ref) < RTOL_L2


def test_decode_gelu_padded_inter(gpu):
    """expert_dim 704 (GELU-tanh, the large library's Gemma path): I is padded to 1024 in the tiles."""
    layer = get_layer(3, 1024, 704, 4, "bf16", act="gelu", seed=4)
    t = make_table(layer)
    x = np.random.RandomState(8).randn(1, 1024).astype(np.float16)
    idx = np.array([[3, 0]], np.int32)
    ref = layer.moe(x.astype(np.float32), idx)
    r = t.moe(0, torch.from_numpy(x).cuda(), idx=torch.from_numpy(idx).cuda(), per_k=True, combine=False,
              out_dtype=torch.float32)
    for k in range(2):
        assert rel_l2(r["per_k"][0, k].cpu().numpy(), ref[0, k]) < RTOL_L2


def test_decode_multi_layer_and_repeat(gpu):
    """two layers, repeated calls: the arrival counters reset themselves."""
    layer = get_layer(3, 2048, 512, 8, "f16", seed=6)
    t = make_table(layer, num_layers=2)
    rng = np.random.RandomState(1)
    x = torch.from_numpy(rng.randn(1, 2048).astype(np.float16)).cuda()
    idx = torch.tensor([[0, 3, 5, 7]], dtype=torch.int32, device="cuda")
    w = torch.tensor([[0.4, 0.3, 0.2, 0.1]], device="cuda")
    outs = [t.moe(l % 2, x, idx=idx, weights=w, combine=True, out_dtype=torch.float32)["out"].clone()
            for l in range(6)]
    for o in outs[1:]:
        assert torch.equal(o, outs[0])
    ref = O.combine(layer.moe(x.float().cpu().numpy(), idx.cpu().numpy()), w.cpu().numpy())
    assert rel_l2(outs[0].cpu().numpy(), ref) < RTOL_L2


def test_decode_workspace_reused_across_shapes(gpu):
    """one workspace, calls with different T and K: each combine must start from zeroed counters."""
    layer = get_layer(3, 2048, 512, 16, "f16", seed=6)
    t = make_table(layer)
    rng = np.random.RandomState(12)
    for T, K in ((3, 8), (1, 4), (5, 2), (2, 8), (1, 1)):
        x = torch.from_numpy(rng.randn(T, 2048).astype(np.float16)).cuda()
        logits = torch.from_numpy(rng.randn(T, 16).astype(np.float32)).cuda()
        r = t.moe(0, x, logits=logits, top_k=K, combine=True, out_dtype=torch.float32)
        idx = r["idx"].cpu().numpy()
        want = O.combine(layer.moe(x.float().cpu().numpy(), idx), r["weights"].cpu().numpy())
        assert rel_l2(r["out"].cpu().numpy(), want) < RTOL_L2, (T, K)


def test_decode_bad_expert_flags_status(gpu):
    from kandiga_b200 import _native as N
    layer = get_layer(3, 2048, 512, 8, "f16", seed=6)
    t = make_table(layer)
    x = torch.randn(1, 2048, device="cuda", dtype=torch.float16)
    idx = torch.tensor([[1, 99]], dtype=torch.int32, device="cuda")
    r = t.moe(0, x, idx=idx, per_k=True, combine=False, out_dtype=torch.float32)
    assert t.status() & N.DEV_BAD_EXPERT
    assert torch.count_nonzero(r["per_k"][0, 1]) == 0
    assert torch.count_nonzero(r["per_k"][0, 0]) > 0
    assert t.status() == 0  # read clears


def test_decode_empty_batch(gpu):
    layer = get_layer(3, 2048, 512, 8, "f16", seed=6)
    t = make_table(layer)
    x = torch.empty(0, 2048, device="cuda", dtype=torch.float16)
    idx = torch.empty(0, 8, dtype=torch.int32, device="cuda")
    r = t.moe(0, x, idx=idx, per_k=True, combine=False)
    assert r["per_k"].shape == (0, 8, 2048)


def test_switchglu_dropin(gpu):
    from kandiga_b200.experts import SwitchGLU
    layer = get_layer(4, 2048, 512, 16, "f16", seed=1)
    t = make_table(layer)
    sw = SwitchGLU(t, 0, hidden_size=2048)
    x = torch.randn(1, 3, 2048, device="cuda", dtype=torch.float16)
    inds = torch.randint(0, 16, (1, 3, 8), device="cuda")
    y = sw(x, inds)
    assert y.shape == (1, 3, 8, 2048) and y.dtype == torch.float16
    ref = layer.moe(x.float().reshape(3, 2048).cpu().numpy(), inds.reshape(3, 8).int().cpu().numpy())
    assert rel_l2(y.float().reshape(3, 8, 2048).cpu().numpy(), ref) < RTOL_L2


def test_router_kernel_bit_exact_indices(gpu):
    from kandiga_b200.experts import router_topk
    rng = np.random.RandomState(5)
    for E, K in ((256, 8), (64, 4), (1024, 16), (8, 8)):
        logits = rng.randn(33, E).astype(np.float32)
        logits[0, :] = 0.0  # all equal
        idx, w = router_topk(torch.from_numpy(logits).cuda(), K)
        ir, wr = O.router_topk(logits, K)
        assert np.array_equal(idx.cpu().numpy(), ir)
        np.testing.assert_allclose(w.cpu().numpy(), wr, rtol=2e-6, atol=1e-7)
