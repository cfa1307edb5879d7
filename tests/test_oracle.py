"""CPU tests: the oracle against the reference's own outputs (golden fixtures made
from the reference by tests/golden/make_golden.py) and, where the reference's
scalar C has been compiled into oracle/_ref, against it live."""
import os

import numpy as np
import pytest

from oracle import oracle as O

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _ref_small():
    ref = O.ref_lib("small")
    from oracle import build_ref
    if ref is None and build_ref.reference_root() is not None:
        build_ref.build()
        O._REF.clear()
        ref = O.ref_lib("small")
    return ref


# ---- 3/4-bit unpack (kandiga/metal/kandiga_cpu_expert.m:194-201,285-291) ----------

def test_unpack3_known_answers():
    # byte-straddling fields: code 2 spans byte0 bit6..byte1 bit0, code 5 spans byte1 bit7..byte2 bit1
    codes = np.array([1, 2, 5, 3, 4, 7, 6, 0], np.uint8)
    row = np.zeros(3, np.uint8)
    O.lib().kqo_pack3(codes.ctypes.data_as(O._u8p), 8, row.ctypes.data_as(O._u8p))
    word = int(row[0]) | int(row[1]) << 8 | int(row[2]) << 16
    assert word == sum(int(c) << (3 * i) for i, c in enumerate(codes))
    out = np.zeros(8, np.uint8)
    O.lib().kqo_unpack3(row.ctypes.data_as(O._u8p), 8, out.ctypes.data_as(O._u8p))
    assert np.array_equal(out, codes)
    for fill in (0, 7):
        c = np.full(64, fill, np.uint8)
        r = np.zeros(24, np.uint8)
        O.lib().kqo_pack3(c.ctypes.data_as(O._u8p), 64, r.ctypes.data_as(O._u8p))
        assert (r == (0 if fill == 0 else 0xFF)).all()


def test_pack_unpack_roundtrip_vectorised_matches_c():
    rng = np.random.RandomState(3)
    for bits in (3, 4):
        q = rng.randint(0, 1 << bits, size=(5, 256)).astype(np.uint8)
        packed = O.pack_codes(q, bits)
        assert np.array_equal(O.unpack_codes(packed, bits, 256), q)
        for r in range(5):
            out = np.zeros(256, np.uint8)
            if bits == 3:
                O.lib().kqo_unpack3(np.ascontiguousarray(packed[r]).ctypes.data_as(O._u8p), 256,
                                    out.ctypes.data_as(O._u8p))
            else:
                O.lib().kqo_unpack4(np.ascontiguousarray(packed[r]).ctypes.data, 256, out.ctypes.data_as(O._u8p))
            assert np.array_equal(out, q[r])


def test_quantizer_properties():
    rng = np.random.RandomState(0)
    w = (rng.randn(32, 512) * 0.02).astype(np.float32)
    w[0, :64] = 0.5  # constant group
    w[1, :64] = 0.0  # all-zero group
    for bits in (3, 4):
        p, s, b = O.quantize_affine(w, bits, 64, "f16", mode="minmax")
        q = O.unpack_codes(p, bits, 512)
        assert q.max() <= (1 << bits) - 1
        deq = O.dequantize_affine(p, s, b, bits, 512)
        err = np.abs(deq - w).reshape(32, 8, 64).max(-1)
        step = O.sb_to_f32(s, "f16")
        assert (err <= step * 0.5 + 1e-3).all()
        # MLX's edge selection: the end of larger magnitude, and zero, exact
        p, s, b = O.quantize_affine(w, bits, 64, "f16")
        q = O.unpack_codes(p, bits, 512).reshape(32, 8, 64)
        assert q.max() <= (1 << bits) - 1
        deq = O.dequantize_affine(p, s, b, bits, 512).reshape(32, 8, 64)
        step = np.abs(O.sb_to_f32(s, "f16"))
        err = np.abs(deq - w.reshape(32, 8, 64)).max(-1)
        assert (err <= step * 1.5 + 1e-3).all()  # the far end may clip by up to half a step more
        assert np.all(deq[1, 0] == 0) and np.allclose(deq[0, 0], 0.5, rtol=1e-3)


def test_quantizer_known_answers():
    """Groups worked by hand through MLX's affine quantizer (3-bit, fp32 then fp16 storage)."""
    g = np.zeros((1, 64), np.float32)
    g[0, 0], g[0, 1], g[0, 2] = -1.0, 0.5, 0.1   # |min| > |max|: edge = min
    # scale0 = 1.5 / 7; q0 = round(-1 / scale0) = round(-4.67) = -5; scale = -1 / -5 = 0.2; bias = -1
    p, s, b = O.quantize_affine(g, 3, 64, "f16")
    assert O.sb_to_f32(s, "f16")[0, 0] == np.float32(np.float16(0.2))
    assert O.sb_to_f32(b, "f16")[0, 0] == -1.0
    q = O.unpack_codes(p, 3, 64)[0]
    # w = -1 -> 0; w = 0.5 -> round(7.5) = 8 -> clipped to 7; w = 0.1 -> round(5.5) = 6;
    # w = 0 -> 5 (zero exact: 5 * 0.2 - 1 = 0)
    assert (q[0], q[1], q[2], q[3]) == (0, 7, 6, 5)
    g2 = -g                                       # |max| > |min|: edge = max, negative scale
    p, s, b = O.quantize_affine(g2, 3, 64, "f16")
    assert O.sb_to_f32(s, "f16")[0, 0] == np.float32(np.float16(-0.2))
    assert O.sb_to_f32(b, "f16")[0, 0] == 1.0
    q = O.unpack_codes(p, 3, 64)[0]
    assert (q[0], q[1], q[2], q[3]) == (0, 7, 6, 5)
    z = np.zeros((1, 64), np.float32)             # all zero: q0 = 0, bias 0, scale -1e-7
    p, s, b = O.quantize_affine(z, 4, 64, "f16")
    assert O.sb_to_f32(b, "f16")[0, 0] == 0.0 and np.all(O.unpack_codes(p, 4, 64) == 0)


# ---- expert MLP: C oracle vs the reference's scalar C ---------------------------------

def test_expert_golden_bit_exact():
    g = np.load(os.path.join(GOLD, "expert_golden.npz"))
    for bits in (3, 4):
        layer = O.ExpertLayer.random(bits, 2048, 512, 3, seed=100 + bits, sb_dtype="bf16")
        import hashlib
        assert hashlib.sha256(layer.layer_blob()).hexdigest().encode() == g[f"b{bits}_sha"].tobytes()
        y = layer.moe(g[f"b{bits}_x"][None], np.arange(3, dtype=np.int32)[None])
        assert np.array_equal(y[0], g[f"b{bits}_y"])


def test_oracle_matches_reference_c_live():
    ref = _ref_small()
    if ref is None:
        pytest.skip("reference scalar C not built (no reference tree and no oracle/_ref)")
    rng = np.random.RandomState(11)
    for bits in (3, 4):
        layer = O.ExpertLayer.random(bits, 2048, 512, 4, seed=bits, sb_dtype="bf16")
        blob = np.frombuffer(layer.layer_blob(), np.uint8).copy()
        x = rng.randn(3, 2048).astype(np.float32)
        idx = rng.randint(0, 4, size=(3, 2)).astype(np.int32)
        out = np.zeros((3, 2, 2048), np.float32)
        rc = ref.ref_moe_layer(bits, blob.ctypes.data, x.ctypes.data_as(O._f32p), idx.ctypes.data_as(O._i32p),
                               3, 2, out.ctypes.data_as(O._f32p), 2)
        assert rc == 0
        assert np.array_equal(out, layer.moe(x, idx))
        # single matvec entry point
        y_ref = np.zeros(512, np.float32)
        fn = ref.ref_matvec3 if bits == 3 else ref.ref_matvec4
        fn(layer.w[0][1].ctypes.data, layer.s[0][1].ctypes.data_as(O._u16p), layer.b[0][1].ctypes.data_as(O._u16p),
           x[0].ctypes.data_as(O._f32p), y_ref.ctypes.data_as(O._f32p), 512, 2048)
        assert np.array_equal(y_ref, O.matvec(bits, layer.w[0][1], layer.s[0][1], layer.b[0][1], x[0], "bf16"))


def test_oracle_matches_reference_lg_gelu_live():
    ref = O.ref_lib("lg")
    if ref is None:
        _ref_small()
        O._REF.pop("lg", None)
        ref = O.ref_lib("lg")
    if ref is None:
        pytest.skip("reference scalar C not built")
    import ctypes
    for bits, inter, act in ((3, 704, "gelu"), (4, 512, "silu")):
        layer = O.ExpertLayer.random(bits, 1024, inter, 2, seed=21, sb_dtype="bf16", act=act, variant="lg")
        offs = (ctypes.c_size_t * 9)(*layer.tensor_offsets())
        x = np.random.RandomState(5).randn(1024).astype(np.float32)
        for e in range(2):
            blob = np.frombuffer(layer.expert_blob(e), np.uint8).copy()
            y = np.zeros(1024, np.float32)
            assert ref.ref_lg_expert(bits, 1 if act == "gelu" else 0, 1024, inter, offs, blob.ctypes.data,
                                     x.ctypes.data_as(O._f32p), y.ctypes.data_as(O._f32p)) == 0
            mine = layer.moe(x[None], np.array([[e]], np.int32))[0, 0]
            assert np.array_equal(y, mine), (bits, act)


def test_fp32_dequant_reference_agrees():
    layer = O.ExpertLayer.random(3, 1024, 512, 2, seed=9)
    x = np.random.RandomState(1).randn(2, 1024).astype(np.float32)
    idx = np.array([[0, 1], [1, 0]], np.int32)
    a = layer.moe(x, idx)
    b = layer.dequant_fp32_moe(x, idx)
    assert np.linalg.norm(a - b) / np.linalg.norm(b) < 1e-5


# ---- router / combine / grouping ----------------------------------------------------------

def test_router_ties_lowest_index_and_renorm():
    logits = np.zeros((2, 16), np.float32)
    logits[0, [3, 7, 9]] = 1.0   # three-way tie at the top
    logits[1] = np.arange(16)[::-1]
    idx, w = O.router_topk(logits, 4)
    assert idx[0].tolist() == [3, 7, 9, 0]
    assert idx[1].tolist() == [0, 1, 2, 3]
    np.testing.assert_allclose(w.sum(1), 1.0, rtol=1e-6)
    e = np.exp(np.array([1, 1, 1, 0], np.float32) - 1)
    np.testing.assert_allclose(w[0], e / e.sum(), rtol=1e-6)


def test_router_matches_softmax_definition():
    rng = np.random.RandomState(4)
    logits = rng.randn(5, 256).astype(np.float32)
    idx, w = O.router_topk(logits, 8)
    p = np.exp(logits - logits.max(1, keepdims=True))
    p /= p.sum(1, keepdims=True)
    order = np.argsort(-p, axis=1, kind="stable")[:, :8]
    assert np.array_equal(idx, order)
    sel = np.take_along_axis(p, order, 1)
    np.testing.assert_allclose(w, sel / sel.sum(1, keepdims=True), rtol=1e-5)


def test_combine_order():
    rng = np.random.RandomState(2)
    y = rng.randn(2, 3, 8).astype(np.float32)
    w = rng.rand(2, 3).astype(np.float32)
    res = rng.randn(2, 8).astype(np.float32)
    out = O.combine(y, w, res)
    np.testing.assert_allclose(out, res + (y * w[..., None]).sum(1), rtol=1e-6, atol=1e-6)


def test_group_by_expert_is_stable_csr():
    idx = np.array([[3, 1], [1, 3], [2, 1]], np.int32)
    s_tok, s_exp, s_k, starts, uniq = O.group_by_expert(idx)
    assert uniq.tolist() == [1, 2, 3]
    assert starts.tolist() == [0, 3, 4, 6]
    assert s_tok.tolist() == [0, 1, 2, 2, 0, 1]
    assert s_k.tolist() == [1, 0, 1, 0, 0, 1]


# ---- BKEX (kandiga/_pack_experts.py:95-132) ------------------------------------------------

def test_bkex_header_golden():
    hdr = open(os.path.join(GOLD, "bkex_header.bin"), "rb").read()
    layer = O.ExpertLayer.random(3, 2048, 512, 1, seed=0, sb_dtype="bf16")
    assert O.bkex_header(256, O.bkex_tensors_for(layer)) == hdr
    info = O.bkex_parse(hdr)
    # known answers of tests/test_pack.py:8-30 (3-bit variant) and the C constants
    assert info["version"] == 1 and info["num_experts"] == 256 and len(info["tensors"]) == 9
    assert info["expert_size"] == 1376256
    assert [t["offset"] for t in info["tensors"]] == [0, 393216, 425984, 458752, 851968, 884736,
                                                      917504, 1310720, 1343488]


# ---- TQ3 (kandiga/tq3/quantize.py) ----------------------------------------------------------

def test_tq3_golden_bit_exact():
    g = np.load(os.path.join(GOLD, "tq3_golden.npz"))
    data, shape, nb = O.tq3_quantize(g["w"])
    assert nb == int(g["num_blocks"])
    assert np.array_equal(np.frombuffer(data, np.uint8), g["blocks"])
    deq = O.tq3_dequantize(g["blocks"].tobytes(), g["w"].shape, nb)
    assert np.array_equal(deq, g["deq"])
    assert np.array_equal(O.tq3_dequantize(g["legacy_blocks"].tobytes(), (192,), 6), g["legacy_deq"])
    assert np.array_equal(O.tq3_wht_forward(g["wht_in"][None])[0].astype(np.float32),
                          g["wht_fwd"].astype(np.float32))
    assert np.array_equal(O.tq3_wht_inverse(g["wht_in"][None])[0], g["wht_inv"])


def test_tq3_cosine_published():
    # README.md:172 reports per-layer cosine 0.990
    w = (np.random.RandomState(0).randn(64, 256) * 0.02).astype(np.float32)
    data, shape, nb = O.tq3_quantize(w)
    d = O.tq3_dequantize(data, shape, nb)
    cos = (d * w).sum() / np.linalg.norm(d) / np.linalg.norm(w)
    assert cos > 0.985


# ---- TurboQuant (kandiga/kv_compress.py) --------------------------------------------------

def test_turboquant_golden_bit_exact():
    g = np.load(os.path.join(GOLD, "turboquant_golden.npz"))
    for tag in "ab":
        D, H, S, seed, seq_len, mem = [int(v) for v in g[tag + "_meta"]]
        r = O.TurboQuantRef(D, H, seed)
        assert np.array_equal(r.rotation, g[tag + "_rotation"])
        assert np.array_equal(r.qjl_proj, g[tag + "_qjl"])
        for kv in "kv":
            x = g[f"{tag}_{kv}"]
            a = r.quantize(x[:, :, :S - 1])
            b = r.quantize(x[:, :, S - 1:])
            got = [np.concatenate([a[i], b[i]], 2) for i in range(4)]
            for gi, name in zip(got, "qszs"):
                pass
            assert np.array_equal(got[0], g[f"{tag}_{kv}q"])
            assert np.array_equal(got[1], g[f"{tag}_{kv}s"])
            assert np.array_equal(got[2], g[f"{tag}_{kv}z"])
            assert np.array_equal(got[3], g[f"{tag}_{kv}sign"])
            rec = r.dequantize(*got)
            assert np.array_equal(rec, g[tag + ("_keys" if kv == "k" else "_values")])


def test_turboquant_reference_tolerances():
    """tests/test_kv_compress.py:11-116 of the reference, restated on the oracle."""
    r = O.TurboQuantRef(128, 8)
    np.testing.assert_allclose(r.rotation @ r.rotation.T, np.eye(128), atol=1e-5)
    r = O.TurboQuantRef(64, 4, seed=123)
    np.random.seed(42)
    k = np.random.randn(1, 4, 16, 64).astype(np.float32)
    rec = r.dequantize(*r.quantize(k)).astype(np.float32)
    assert np.mean(np.abs(rec - k)) < 0.5
    r = O.TurboQuantRef(128, 1, seed=77)
    np.random.seed(99)
    k = np.random.randn(1, 1, 32, 128).astype(np.float32)
    rec = r.dequantize(*r.quantize(k)).astype(np.float32).reshape(32, 128)
    k = k.reshape(32, 128)
    cos = (rec * k).sum(1) / (np.linalg.norm(rec, axis=1) * np.linalg.norm(k, axis=1) + 1e-8)
    assert (cos > 0.85).all()
