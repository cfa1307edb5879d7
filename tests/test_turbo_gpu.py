"""GPU parity of the TurboQuant cache (kq_tq_*) against the numpy restatement of
kandiga/kv_compress.py (oracle.TurboQuantRef), plus the reference's own test
tolerances (kandiga tests/test_kv_compress.py).

The rotation x R and the QJL product are fp32 FMA chains on the GPU and BLAS
sgemm on the CPU, so a code or a sign can differ where a value sits on a
rounding boundary: the codes must agree on >= 99.5% of elements (and differ
by at most one level), the signs on >= 99%, and scales/zeros to 1e-5
relative.  Reconstruction is compared on the GPU's own codes (fp16 output,
rel L2 < 1e-3); attention scores and outputs against the oracle's softmax
attention over the reference reconstruction of those codes (2e-3)."""
import ctypes

import numpy as np
import pytest
import torch

from kandiga_b200 import _native as N
from kandiga_b200.kv_compress import TurboQuantCache
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def kv_with_outliers(rng, b, h, s, d, frac=0.01):
    k = rng.randn(b, h, s, d).astype(np.float32)
    v = rng.randn(b, h, s, d).astype(np.float32)
    n = max(1, int(round(frac * h * d)))
    pairs = rng.choice(h * d, n, replace=False)
    for p in pairs:
        k[:, p // d, :, p % d] *= 8
        v[:, p // d, :, p % d] *= 8
    return k, v


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


@pytest.mark.parametrize("d,dtype", [(128, torch.float16), (64, torch.float32), (128, torch.bfloat16)])
def test_append_matches_oracle(gpu, d, dtype):
    rng = np.random.RandomState(d)
    b, h, s = 2, 4, 300
    k, v = kv_with_outliers(rng, b, h, s, d)
    kt = torch.from_numpy(k).to(dtype)
    vt = torch.from_numpy(v).to(dtype)
    cache = TurboQuantCache(d, h, seed=42, capacity=64)
    cache.update(kt[:, :, :100].cuda(), vt[:, :, :100].cuda())  # two appends, capacity growth
    cache.update(kt[:, :, 100:].cuda(), vt[:, :, 100:].cuda())
    assert cache.seq_len == s
    ref = O.TurboQuantRef(d, h, 42)
    for which, x in ((0, kt), (1, vt)):
        q_ref, s_ref, z_ref, g_ref = ref.quantize(x.float().numpy())
        codes, scales, zeros, signs = [t.cpu().numpy() for t in cache.export(which)]
        np.testing.assert_allclose(scales, s_ref, rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(zeros, z_ref, rtol=1e-5, atol=1e-5)
        agree = np.mean(codes == q_ref)
        assert agree >= 0.995, agree
        assert np.max(np.abs(codes.astype(np.int32) - q_ref)) <= 1
        assert np.mean(signs == g_ref) >= 0.99
        assert codes.min() >= 0 and codes.max() <= 7 and set(np.unique(signs)) <= {0, 1}


def test_reconstruction_on_own_codes(gpu):
    rng = np.random.RandomState(5)
    b, h, s, d = 1, 8, 257, 128
    k, v = kv_with_outliers(rng, b, h, s, d)
    cache = TurboQuantCache(d, h, seed=42)
    cache.update(torch.from_numpy(k).half().cuda(), torch.from_numpy(v).half().cuda())
    ref = O.TurboQuantRef(d, h, 42)
    for which, acc in ((0, cache.keys), (1, cache.values)):
        codes, scales, zeros, signs = [t.cpu().numpy() for t in cache.export(which)]
        want = ref.dequantize(codes, scales, zeros, signs).astype(np.float32)
        got = acc.float().cpu().numpy()
        assert got.dtype == np.float32 and acc.dtype == torch.float16
        assert rel_l2(got, want) < 1e-3


def test_reference_tolerances(gpu):
    """kandiga tests/test_kv_compress.py: roundtrip mean-abs error < 0.5,
    sequential updates, memory savings, cosine similarity > 0.85."""
    np.random.seed(42)
    cache = TurboQuantCache(head_dim=64, num_heads=4, seed=123)
    keys = np.random.randn(1, 4, 16, 64).astype(np.float32)
    values = np.random.randn(1, 4, 16, 64).astype(np.float32)
    cache.update(torch.from_numpy(keys).cuda(), torch.from_numpy(values).cuda())
    assert tuple(cache.keys.shape) == keys.shape and tuple(cache.values.shape) == values.shape
    assert np.mean(np.abs(cache.keys.float().cpu().numpy() - keys)) < 0.5
    assert np.mean(np.abs(cache.values.float().cpu().numpy() - values)) < 0.5

    cache = TurboQuantCache(head_dim=64, num_heads=2, seed=0, capacity=2)
    for _ in range(5):
        cache.update(torch.randn(1, 2, 1, 64, device="cuda"), torch.randn(1, 2, 1, 64, device="cuda"))
    assert cache.seq_len == 5
    assert tuple(cache.keys.shape) == (1, 2, 5, 64) and tuple(cache.values.shape) == (1, 2, 5, 64)

    cache = TurboQuantCache(head_dim=128, num_heads=8)
    cache.update(torch.randn(1, 8, 100, 128, device="cuda"), torch.randn(1, 8, 100, 128, device="cuda"))
    assert cache.memory_bytes < 1 * 8 * 100 * 128 * 2 * 2
    assert cache.memory_uncompressed == 1 * 8 * 100 * 128 * 2 * 2

    cache = TurboQuantCache(head_dim=128, num_heads=1, seed=77)
    np.random.seed(99)
    k = np.random.randn(1, 1, 32, 128).astype(np.float32)
    kt = torch.from_numpy(k).cuda()
    cache.update(kt, kt)
    ko = k.reshape(32, 128)
    kr = cache.keys.float().cpu().numpy().reshape(32, 128)
    for i in range(32):
        cos = np.dot(ko[i], kr[i]) / (np.linalg.norm(ko[i]) * np.linalg.norm(kr[i]) + 1e-8)
        assert cos > 0.85, (i, cos)


@pytest.mark.parametrize("h,hq,s", [(8, 8, 1000), (4, 16, 1537), (2, 2, 1)])
def test_attend_matches_oracle(gpu, h, hq, s):
    rng = np.random.RandomState(h * 100 + s)
    b, d = 1, 128
    k, v = kv_with_outliers(rng, b, h, s, d)
    q = rng.randn(b, hq, d).astype(np.float32)
    cache = TurboQuantCache(d, h, seed=42)
    cache.update(torch.from_numpy(k).half().cuda(), torch.from_numpy(v).half().cuda())
    out, scores = cache.attend(torch.from_numpy(q).half().cuda(), return_scores=True)
    ref = O.TurboQuantRef(d, h, 42)
    kc = [t.cpu().numpy()[0] for t in cache.export(0)]
    vc = [t.cpu().numpy()[0] for t in cache.export(1)]
    v_hat = ref.dequantize(*vc)  # the reference's fp16 value reconstruction
    g = hq // h
    qh = q[0].astype(np.float16).astype(np.float32)
    for kv in range(h):
        sub = O.TurboQuantRef(d, 1, 42)
        o_ref, s_ref = sub.attend(qh[kv * g:(kv + 1) * g], *(np.repeat(c[kv:kv + 1], g, axis=0) for c in kc),
                                  np.repeat(v_hat[kv:kv + 1], g, axis=0))
        got_s = scores[0, kv * g:(kv + 1) * g].cpu().numpy()
        assert np.max(np.abs(got_s - s_ref)) <= 2e-3 * max(1.0, np.max(np.abs(s_ref)))
        assert rel_l2(out[0, kv * g:(kv + 1) * g].cpu().numpy(), o_ref) < 2e-3


def test_capacity_and_errors(gpu):
    lib = N.load()
    r, p = O.TurboQuantRef(64, 2, 1).rotation, O.TurboQuantRef(64, 2, 1).qjl_proj
    h = ctypes.c_void_p()
    assert lib.kq_tq_create(64, 2, 1, 4, r.ctypes.data_as(ctypes.c_void_p), p.ctypes.data_as(ctypes.c_void_p),
                            ctypes.byref(h)) == N.KQ_OK
    try:
        x = torch.randn(1, 2, 5, 64, device="cuda")
        s = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        assert lib.kq_tq_append(h, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(x.data_ptr()), N.DT_F32, 5,
                                s) == N.KQ_ERR_CAPACITY
        assert lib.kq_tq_seq_len(h) == 0
        assert lib.kq_tq_append(h, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(x.data_ptr()), N.DT_F32, 3,
                                s) == N.KQ_OK
        assert lib.kq_tq_reserve(h, 16, s) == N.KQ_OK and lib.kq_tq_capacity(h) == 16
        assert lib.kq_tq_append(h, ctypes.c_void_p(x.data_ptr()), ctypes.c_void_p(x.data_ptr()), N.DT_F32, 5,
                                s) == N.KQ_OK
        assert lib.kq_tq_seq_len(h) == 8
        q = torch.randn(1, 3, 64, device="cuda")
        out = torch.empty(1, 3, 64, device="cuda")
        assert lib.kq_tq_attend(h, ctypes.c_void_p(q.data_ptr()), N.DT_F32, 3, ctypes.c_void_p(out.data_ptr()),
                                None, None, 0, s) == N.ERRORS_INV["KQ_ERR_ARG"]
        assert lib.kq_tq_attend(h, ctypes.c_void_p(q.data_ptr()), N.DT_F32, 2, ctypes.c_void_p(out.data_ptr()),
                                None, None, 0, s) == N.ERRORS_INV["KQ_ERR_WORKSPACE"]
    finally:
        lib.kq_tq_destroy(h)
    torch.cuda.synchronize()


def test_growth_preserves_contents(gpu):
    rng = np.random.RandomState(3)
    k, v = kv_with_outliers(rng, 1, 2, 40, 64)
    cache = TurboQuantCache(64, 2, seed=9, capacity=8)
    cache.update(torch.from_numpy(k[:, :, :7]).cuda(), torch.from_numpy(v[:, :, :7]).cuda())
    before = [t.clone() for t in cache.export(0)]
    cache.update(torch.from_numpy(k[:, :, 7:]).cuda(), torch.from_numpy(v[:, :, 7:]).cuda())
    assert cache.capacity() >= 40
    after = cache.export(0)
    for a, b_ in zip(before, after):
        assert torch.equal(a, b_[:, :, :7])


def test_session_round_trip_of_compressed_cache(gpu, tmp_path):
    """TurboQuantCache layers saved through save_session keep their packed codes:
    after load_session the reconstructions and attention are bit-identical, and
    appending more tokens gives what an unsaved cache gives."""
    from kandiga_b200.kv_compress import TurboQuantCache, load_session, save_session
    g = torch.Generator(device="cuda").manual_seed(3)
    caches, ref = [], []
    for seed, D, Hh, T in ((42, 128, 4, 300), (7, 64, 2, 17)):
        k = torch.randn(1, Hh, T, D, generator=g, device="cuda").half()
        v = torch.randn(1, Hh, T, D, generator=g, device="cuda").half()
        c = TurboQuantCache(D, Hh, seed=seed, capacity=64)
        c.update(k, v)
        r = TurboQuantCache(D, Hh, seed=seed, capacity=64)
        r.update(k, v)
        caches.append(c)
        ref.append(r)
    path = str(tmp_path / "sess.npz")
    save_session(path, caches, history=["x"], tokens_fed=317, model="tiny")
    got, meta = load_session(path, model="tiny")
    assert meta["layer_info"]["0"]["type"] == "TurboQuantCache" and meta["layer_info"]["0"]["offset"] == 300
    for c, d, r in zip(caches, got, ref):
        assert d.seq_len == c.seq_len and d.head_dim == c.head_dim and d.num_heads == c.num_heads
        assert torch.equal(d.keys, c.keys) and torch.equal(d.values, c.values)
        for a, b in zip(d.state(), c.state()):
            assert torch.equal(a, b)
        q = torch.randn(1, c.num_heads, c.head_dim, generator=g, device="cuda").half()
        assert torch.equal(d.attend(q), c.attend(q))
        k2 = torch.randn(1, c.num_heads, 40, c.head_dim, generator=g, device="cuda").half()
        v2 = torch.randn(1, c.num_heads, 40, c.head_dim, generator=g, device="cuda").half()
        d.update(k2, v2)
        r.update(k2, v2)
        assert torch.equal(d.keys, r.keys) and torch.equal(d.values, r.values)


def test_configs3_shape_append_and_attend(gpu):
    """The benched TurboQuant shape itself: 8 KV heads x 32768 tokens x D128,
    K and V fp16 N(0,1) with 1% of the (head, channel) pairs scaled x8, one
    bulk append, then single-query attention (8 query heads).  32768 tokens
    are 128 chunks per head, so the chunk-partial merge runs more than one
    batch of chunks per warp.  Codes are compared with the numpy restatement of
    kandiga/kv_compress.py:59-92 and the attention with softmax attention over
    the reference reconstruction (kandiga/kv_compress.py:94-118) of the GPU's
    own codes, with the bars of the smaller cases."""
    rng = np.random.RandomState(3)
    b, h, s, d = 1, 8, 32768, 128
    k, v = kv_with_outliers(rng, b, h, s, d)
    kt = torch.from_numpy(k).half()
    vt = torch.from_numpy(v).half()
    cache = TurboQuantCache(d, h, seed=42)
    cache.update(kt.cuda(), vt.cuda())
    assert cache.seq_len == s
    ref = O.TurboQuantRef(d, h, 42)
    for which, x in ((0, kt), (1, vt)):
        q_ref, s_ref, z_ref, g_ref = ref.quantize(x.float().numpy())
        codes, scales, zeros, signs = [t.cpu().numpy() for t in cache.export(which)]
        np.testing.assert_allclose(scales, s_ref, rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(zeros, z_ref, rtol=1e-5, atol=1e-5)
        assert np.mean(codes == q_ref) >= 0.995
        assert np.max(np.abs(codes.astype(np.int32) - q_ref)) <= 1
        assert np.mean(signs == g_ref) >= 0.99
    q = rng.randn(b, h, d).astype(np.float32)
    out, scores = cache.attend(torch.from_numpy(q).half().cuda(), return_scores=True)
    kc = [t.cpu().numpy()[0] for t in cache.export(0)]
    v_hat = ref.dequantize(*[t.cpu().numpy()[0] for t in cache.export(1)])
    qh = q[0].astype(np.float16).astype(np.float32)
    o_ref, s_ref = ref.attend(qh, *kc, v_hat)
    got_s = scores[0].cpu().numpy()
    assert np.max(np.abs(got_s - s_ref)) <= 2e-3 * max(1.0, np.max(np.abs(s_ref)))
    assert rel_l2(out[0].cpu().numpy(), o_ref) < 2e-3
    # the same query again gives bit-identical results (fixed merge order)
    out2 = cache.attend(torch.from_numpy(q).half().cuda())
    assert torch.equal(out, out2)


@pytest.mark.parametrize("d,h,hq,s", [(96, 2, 4, 300), (80, 4, 4, 513), (40, 2, 2, 77)])
def test_any_head_dim(gpu, d, h, hq, s):
    """head_dim other than 64 / 128 (the reference takes any, kandiga/kv_compress.py:30-57):
    the same oracle comparisons for append, reconstruction and attention, and a
    save / restore round trip of the packed storage."""
    rng = np.random.RandomState(d + s)
    b = 1
    k, v = kv_with_outliers(rng, b, h, s, d)
    cache = TurboQuantCache(d, h, seed=42, capacity=32)
    cache.update(torch.from_numpy(k[:, :, :s // 2]).half().cuda(), torch.from_numpy(v[:, :, :s // 2]).half().cuda())
    cache.update(torch.from_numpy(k[:, :, s // 2:]).half().cuda(), torch.from_numpy(v[:, :, s // 2:]).half().cuda())
    ref = O.TurboQuantRef(d, h, 42)
    for which, x, acc in ((0, k, cache.keys), (1, v, cache.values)):
        xh = x.astype(np.float16).astype(np.float32)
        q_ref, s_ref, z_ref, g_ref = ref.quantize(xh)
        codes, scales, zeros, signs = [t.cpu().numpy() for t in cache.export(which)]
        assert codes.shape == (b, h, s, d)
        np.testing.assert_allclose(scales, s_ref, rtol=1e-5, atol=1e-6)
        np.testing.assert_allclose(zeros, z_ref, rtol=1e-5, atol=1e-5)
        assert np.mean(codes == q_ref) >= 0.995
        assert np.max(np.abs(codes.astype(np.int32) - q_ref)) <= 1
        assert np.mean(signs == g_ref) >= 0.99
        want = ref.dequantize(codes, scales, zeros, signs).astype(np.float32)
        got = acc.float().cpu().numpy()
        assert got.shape == (b, h, s, d) and rel_l2(got, want) < 1e-3
    q = rng.randn(b, hq, d).astype(np.float32)
    out, scores = cache.attend(torch.from_numpy(q).half().cuda(), return_scores=True)
    assert tuple(out.shape) == (b, hq, d)
    kc = [t.cpu().numpy()[0] for t in cache.export(0)]
    v_hat = ref.dequantize(*[t.cpu().numpy()[0] for t in cache.export(1)])
    g = hq // h
    qh = q[0].astype(np.float16).astype(np.float32)
    for kv in range(h):
        sub = O.TurboQuantRef(d, 1, 42)
        o_ref, s_ref = sub.attend(qh[kv * g:(kv + 1) * g], *(np.repeat(c[kv:kv + 1], g, axis=0) for c in kc),
                                  np.repeat(v_hat[kv:kv + 1], g, axis=0))
        got_s = scores[0, kv * g:(kv + 1) * g].cpu().numpy()
        assert np.max(np.abs(got_s - s_ref)) <= 2e-3 * max(1.0, np.max(np.abs(s_ref)))
        assert rel_l2(out[0, kv * g:(kv + 1) * g].cpu().numpy(), o_ref) < 2e-3
    st = cache.state()
    other = TurboQuantCache(d, h, seed=42)
    other.load_state(st)
    assert torch.equal(other.keys, cache.keys) and torch.equal(other.values, cache.values)
