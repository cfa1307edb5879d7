"""GPU parity of the grouped tensor-core prefill path (kq_moe_prefill) against
the C oracle of the reference's expert MLP.  Tolerance: 2e-3 relative L2 per
(token, k) expert output and per combined token row."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.test_decode_gpu import get_layer, make_table, rel_l2

pytestmark = pytest.mark.gpu
RTOL_L2 = 2e-3


def check(layer, t, x, idx, w, r, res=None):
    y = layer.moe(x.float().cpu().numpy(), idx)
    if r["per_k"] is not None:
        pk = r["per_k"].float().cpu().numpy()
        worst = max(rel_l2(pk[i, k], y[i, k]) for i in range(idx.shape[0]) for k in range(idx.shape[1]))
        assert worst < RTOL_L2, worst
    if r["out"] is not None:
        want = O.combine(y, w, None if res is None else res.float().cpu().numpy())
        got = r["out"].float().cpu().numpy()
        worst = max(rel_l2(got[i], want[i]) for i in range(idx.shape[0]))
        assert worst < RTOL_L2, worst


@pytest.mark.parametrize("bits,sb", [(4, "f16"), (3, "f16"), (4, "bf16"), (3, "bf16")])
def test_prefill_matches_oracle(gpu, bits, sb):
    E, H, I, K, T = 16, 2048, 512, 8, 96
    layer = get_layer(bits, H, I, E, sb, seed=20 + bits)
    t = make_table(layer)
    rng = np.random.RandomState(bits)
    x = torch.from_numpy(rng.randn(T, H).astype(np.float16)).cuda()
    logits = torch.from_numpy(rng.randn(T, E).astype(np.float32)).cuda()
    r = t.moe(0, x, logits=logits, top_k=K, per_k=True, combine=True, out_dtype=torch.float32, path="prefill")
    idx_ref, w_ref = O.router_topk(logits.cpu().numpy(), K)
    assert np.array_equal(r["idx"].cpu().numpy(), idx_ref)
    check(layer, t, x, idx_ref, r["weights"].cpu().numpy(), r)
    assert t.status() == 0


def test_prefill_skewed_chunks_and_residual(gpu):
    """one expert receives every token (N-chunks of 128 + a ragged tail), others few."""
    E, H, I, K, T = 8, 1024, 1024, 2, 300
    layer = get_layer(4, H, I, E, "f16", seed=31)
    t = make_table(layer)
    rng = np.random.RandomState(4)
    x = torch.from_numpy(rng.randn(T, H).astype(np.float16)).cuda()
    idx = np.zeros((T, K), np.int32)
    idx[:, 0] = 3
    idx[:, 1] = rng.randint(0, E, T)
    idx[idx[:, 1] == 3, 1] = 5
    w = rng.rand(T, K).astype(np.float32)
    res = torch.from_numpy(rng.randn(T, H).astype(np.float32)).cuda()
    r = t.moe(0, x, idx=torch.from_numpy(idx).cuda(), weights=torch.from_numpy(w).cuda(), per_k=True, combine=True,
              residual=res, out_dtype=torch.float32, path="prefill")
    check(layer, t, x, idx, w, r, res)


@pytest.mark.parametrize("xdt", [torch.bfloat16, torch.float32])
def test_prefill_input_dtypes(gpu, xdt):
    E, H, I, K, T = 16, 2048, 512, 4, 40
    layer = get_layer(3, H, I, E, "f16", seed=9)
    t = make_table(layer)
    rng = np.random.RandomState(6)
    x = torch.from_numpy(rng.randn(T, H).astype(np.float32) * 30).to(xdt).cuda()
    logits = torch.from_numpy(rng.randn(T, E).astype(np.float32)).cuda()
    r = t.moe(0, x, logits=logits, top_k=K, per_k=True, combine=True, out_dtype=torch.float32, path="prefill")
    idx = r["idx"].cpu().numpy()
    check(layer, t, x, idx, r["weights"].cpu().numpy(), r)


def test_prefill_matches_decode_path(gpu):
    E, H, I, K, T = 32, 2048, 512, 8, 64
    layer = get_layer(3, H, I, E, "f16", seed=2)
    t = make_table(layer)
    rng = np.random.RandomState(10)
    x = torch.from_numpy(rng.randn(T, H).astype(np.float16)).cuda()
    logits = torch.from_numpy(rng.randn(T, E).astype(np.float32)).cuda()
    a = t.moe(0, x, logits=logits, top_k=K, combine=True, out_dtype=torch.float32, path="prefill")["out"]
    b = t.moe(0, x, logits=logits, top_k=K, combine=True, out_dtype=torch.float32, path="decode")["out"]
    assert rel_l2(a.cpu().numpy(), b.cpu().numpy()) < RTOL_L2


@pytest.mark.parametrize("H,I", [(2560, 512), (1024, 2560)])
def test_prefill_wide_k(gpu, H, I):
    """K = 2560 in gate/up (H = 2560) or in down (I = 2560): five 512-wide
    super-tiles per item, bf16 scales."""
    E, K, T = 8, 2, 40
    layer = get_layer(4, H, I, E, "bf16", seed=H + I)
    t = make_table(layer)
    rng = np.random.RandomState(H)
    x = torch.from_numpy(rng.randn(T, H).astype(np.float16)).cuda()
    logits = torch.from_numpy(rng.randn(T, E).astype(np.float32)).cuda()
    r = t.moe(0, x, logits=logits, top_k=K, per_k=True, combine=True, out_dtype=torch.float32, path="prefill")
    check(layer, t, x, r["idx"].cpu().numpy(), r["weights"].cpu().numpy(), r)
    assert t.status() == 0


def test_prefill_bad_expert(gpu):
    from kandiga_b200 import _native as N
    E, H, I, K, T = 8, 1024, 512, 2, 20
    layer = get_layer(4, H, I, E, "f16", seed=7)
    t = make_table(layer)
    x = torch.randn(T, H, device="cuda").half()
    idx = torch.randint(0, E, (T, K), device="cuda", dtype=torch.int32)
    idx[3, 1] = 77
    r = t.moe(0, x, idx=idx, per_k=True, combine=False, out_dtype=torch.float32, path="prefill")
    assert t.status() & N.DEV_BAD_EXPERT
    assert torch.count_nonzero(r["per_k"][3, 1]) == 0


def test_prefill_large_batch_bitwise_repeatable(gpu):
    """T*K = 8192 assignments (several grouping rounds, ~128 tokens per expert):
    prefill agrees with the decode path and with the oracle on sampled tokens,
    and two runs give identical bits although the order of an expert's tokens
    inside its segment may differ between runs."""
    E, H, I, K, T = 64, 1024, 512, 8, 1024
    layer = get_layer(4, H, I, E, "f16", seed=12)
    t = make_table(layer)
    rng = np.random.RandomState(12)
    x = torch.from_numpy(rng.randn(T, H).astype(np.float16)).cuda()
    logits = torch.from_numpy(rng.randn(T, E).astype(np.float32)).cuda()
    a = t.moe(0, x, logits=logits, top_k=K, per_k=True, combine=True, out_dtype=torch.float32, path="prefill")
    b = t.moe(0, x, logits=logits, top_k=K, per_k=True, combine=True, out_dtype=torch.float32, path="prefill")
    assert torch.equal(a["out"], b["out"]) and torch.equal(a["per_k"], b["per_k"])
    d = t.moe(0, x, logits=logits, top_k=K, combine=True, out_dtype=torch.float32, path="decode")["out"]
    assert rel_l2(a["out"].cpu().numpy(), d.cpu().numpy()) < RTOL_L2
    rows = [0, 1, 511, 1023]
    idx = a["idx"].cpu().numpy()[rows]
    y = layer.moe(x.float().cpu().numpy()[rows], idx)
    pk = a["per_k"].float().cpu().numpy()[rows]
    worst = max(rel_l2(pk[i, k], y[i, k]) for i in range(len(rows)) for k in range(K))
    assert worst < RTOL_L2, worst
    assert t.status() == 0


def test_prefill_bench_shape(gpu):
    """The benchmark's workload shape: E=256 top-8, T=512 tokens, H2048/I512
    4-bit (about 16 tokens per expert, many work items per CTA).  Two runs give
    identical bits, the result agrees with the decode path, and sampled tokens
    agree with the oracle (the layer is quantized on the GPU; the oracle gets
    the routed experts' MLX tensors)."""
    from kandiga_b200.experts import ExpertTable
    from kandiga_b200.quant import quantize_affine
    E, H, I, K, T = 256, 2048, 512, 8, 512
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(77)
    mats = []
    for rows, cols in ((I, H), (I, H), (H, I)):
        ws, ss, bs = [], [], []
        for _ in range(0, E, 64):
            w = torch.randn(64 * rows, cols, generator=g, device=dev) * 0.02
            p, s, b = quantize_affine(w, 4, 64, "f16")
            ws.append(p.reshape(64, rows, -1))
            ss.append(s.reshape(64, rows, -1))
            bs.append(b.reshape(64, rows, -1))
        mats.append((torch.cat(ws).contiguous(), torch.cat(ss).view(torch.int16).contiguous(),
                     torch.cat(bs).view(torch.int16).contiguous()))
    t = ExpertTable(1, E, H, I, 4, "f16")
    t.load_mlx(0, *mats)
    x = torch.randn(T, H, generator=g, device=dev).half()
    logits = torch.randn(T, E, generator=g, device=dev)
    a = t.moe(0, x, logits=logits, top_k=K, per_k=True, combine=True, out_dtype=torch.float32, path="prefill")
    b = t.moe(0, x, logits=logits, top_k=K, per_k=True, combine=True, out_dtype=torch.float32, path="prefill")
    assert t.status() == 0
    assert torch.equal(a["out"], b["out"]) and torch.equal(a["per_k"], b["per_k"])
    d = t.moe(0, x, logits=logits, top_k=K, combine=True, out_dtype=torch.float32, path="decode")["out"]
    assert rel_l2(a["out"].cpu().numpy(), d.cpu().numpy()) < RTOL_L2
    rows = [0, 257, 511]
    idx = a["idx"].cpu().numpy()[rows]
    ids = np.unique(idx)
    remap = {int(e): i for i, e in enumerate(ids)}
    sel = torch.from_numpy(ids.astype(np.int64)).to(dev)
    sub = O.ExpertLayer(4, H, I, [m[0][sel].cpu().numpy().view(np.uint32) for m in mats],
                        [m[1][sel].cpu().numpy().view(np.uint16) for m in mats],
                        [m[2][sel].cpu().numpy().view(np.uint16) for m in mats], "f16", "silu")
    y = sub.moe(x.float().cpu().numpy()[rows], np.vectorize(remap.get)(idx).astype(np.int32))
    pk = a["per_k"].float().cpu().numpy()[rows]
    worst = max(rel_l2(pk[i, k], y[i, k]) for i in range(len(rows)) for k in range(K))
    assert worst < RTOL_L2, worst


@pytest.mark.parametrize("xdt,mag", [(torch.bfloat16, 3e3), (torch.bfloat16, 1e4), (torch.float16, 2e3)])
def test_prefill_large_activations(gpu, xdt, mag):
    """Inputs of magnitude 1e3-1e4: gate/up outputs reach ~1e5 and SwiGLU
    products ~1e7-1e9, far beyond fp16.  The activations are stored with a
    power-of-two exponent per (token, expert, 16 rows) and brought to one
    exponent per (token, expert) before the down projection; results match the
    fp32 oracle to the usual 2e-3."""
    E, H, I, K, T = 16, 2048, 512, 8, 48
    layer = get_layer(4, H, I, E, "f16", seed=41)
    t = make_table(layer)
    rng = np.random.RandomState(41)
    xf = rng.randn(T, H).astype(np.float32) * np.float32(mag)
    xf[::7] *= 0.01  # some tokens stay in range: one call mixes scaled and unscaled positions
    x = torch.from_numpy(xf).to(xdt).cuda()
    logits = torch.from_numpy(rng.randn(T, E).astype(np.float32)).cuda()
    r = t.moe(0, x, logits=logits, top_k=K, per_k=True, combine=True, out_dtype=torch.float32, path="prefill")
    assert torch.isfinite(r["per_k"]).all() and torch.isfinite(r["out"]).all()
    check(layer, t, x, r["idx"].cpu().numpy(), r["weights"].cpu().numpy(), r)
    assert t.status() == 0
    # the next call on in-range inputs is not affected by the scaled one before it
    x2 = torch.from_numpy(rng.randn(T, H).astype(np.float32)).to(xdt).cuda()
    r2 = t.moe(0, x2, logits=logits, top_k=K, per_k=True, combine=True, out_dtype=torch.float32, path="prefill")
    check(layer, t, x2, r2["idx"].cpu().numpy(), r2["weights"].cpu().numpy(), r2)


def _scaled_experts(layer, experts, factor):
    """a copy of `layer` whose experts `experts` have every scale and bias
    multiplied by `factor` (a power of two: exact in fp16 and bf16)"""
    s = [a.copy() for a in layer.s]
    b = [a.copy() for a in layer.b]
    for m in range(3):
        for e in experts:
            s[m][e] = O.f32_to_sb(O.sb_to_f32(s[m][e], layer.sb_dtype) * np.float32(factor), layer.sb_dtype)
            b[m][e] = O.f32_to_sb(O.sb_to_f32(b[m][e], layer.sb_dtype) * np.float32(factor), layer.sb_dtype)
    return O.ExpertLayer(layer.bits, layer.hidden, layer.inter, layer.w, s, b, layer.sb_dtype, layer.act)


@pytest.mark.parametrize("sb,factor", [("f16", 2.0 ** 14), ("bf16", 2.0 ** 18)])
def test_prefill_large_scale_groups(gpu, sb, factor):
    """Experts whose groups all have |scale| >= 64 (~120-500 with fp16 scales,
    ~4e3 with bf16; weights up to ~4e3 / ~3e4, still fp16 numbers) beside
    experts of ordinary scale.  The dequantisation forms q exactly and then
    q*s + b in one rounding, so no intermediate overflows; the SwiGLU products
    of the large experts (~1e6 / ~1e10) leave fp16 range and are stored with
    power-of-two exponents.  Prefill and decode both match the fp32 oracle to
    2e-3."""
    E, H, I, K, T = 8, 1024, 512, 4, 64
    layer = _scaled_experts(get_layer(3, H, I, E, sb, seed=43), [1, 4, 6], factor)
    assert np.abs(O.sb_to_f32(layer.s[0][1], sb)).min() >= 64
    t = make_table(layer)
    rng = np.random.RandomState(43)
    x = torch.from_numpy(rng.randn(T, H).astype(np.float16)).cuda()
    logits = torch.from_numpy(rng.randn(T, E).astype(np.float32)).cuda()
    for path in ("prefill", "decode"):
        r = t.moe(0, x, logits=logits, top_k=K, per_k=True, combine=True, out_dtype=torch.float32, path=path)
        assert torch.isfinite(r["per_k"]).all()
        check(layer, t, x, r["idx"].cpu().numpy(), r["weights"].cpu().numpy(), r)
        assert t.status() == 0


def test_prefill_weight_out_of_fp16_range_is_reported(gpu):
    """A bf16 group whose weights exceed the fp16 range (|q s + b| > 65504)
    cannot be dequantised to fp16: the call latches KQ_DEV_RANGE."""
    from kandiga_b200 import _native as N
    E, H, I, K, T = 4, 1024, 512, 2, 16
    layer = get_layer(3, H, I, E, "bf16", seed=44)
    s = [a.copy() for a in layer.s]
    b = [a.copy() for a in layer.b]
    s[0][1, 3, 2] = O.f32_to_sb(np.array([3.0e4], np.float32), "bf16")[0]
    b[0][1, 3, 2] = O.f32_to_sb(np.array([-1.0e5], np.float32), "bf16")[0]
    layer = O.ExpertLayer(layer.bits, layer.hidden, layer.inter, layer.w, s, b, "bf16", layer.act)
    t = make_table(layer)
    x = torch.randn(T, H, device="cuda").half()
    idx = torch.ones(T, K, device="cuda", dtype=torch.int32)
    idx[:, 1] = 2
    t.moe(0, x, idx=idx, per_k=True, combine=False, out_dtype=torch.float32, path="prefill")
    assert t.status() & N.DEV_RANGE
    assert t.status() == 0  # reading clears the word
