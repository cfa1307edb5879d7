"""GPU tests of the reference-compatible host ABI (bakan_cpu_expert_*) on BKEX
layer files, called the way the reference's _CPUExpertLib calls it
(kandiga/engine.py:79-214)."""
import ctypes
import os

import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


def write_bkex(dirname, layers):
    for l, layer in enumerate(layers):
        hdr = O.bkex_header(layer.num_experts, O.bkex_tensors_for(layer))
        with open(os.path.join(dirname, f"layer_{l:02d}.bin"), "wb") as f:
            f.write(hdr)
            f.write(layer.layer_blob())


@pytest.fixture(scope="module")
def packed(tmp_path_factory, gpu):
    d = tmp_path_factory.mktemp("packed")
    layers = [O.ExpertLayer.random(3, 2048, 512, 6, seed=40 + l, sb_dtype="bf16") for l in range(2)]
    write_bkex(str(d), layers)
    return str(d), layers


def test_expert_lib_f16_matches_reference(packed):
    from kandiga_b200.experts import ExpertLib
    d, layers = packed
    lib = ExpertLib()
    eng = lib.init(d, 2)
    try:
        assert lib.num_layers(eng) == 2
        rng = np.random.RandomState(0)
        for l in range(2):
            x = rng.randn(2048).astype(np.float16)
            idx = np.array([5, 0, 3, 2], np.int32)
            out = lib.expert_mlp_f16(eng, l, x, idx, 4)
            ref = layers[l].moe(x.astype(np.float32)[None], idx[None])[0]
            rref = O.ref_lib("small")
            if rref is not None:  # the reference's own scalar C on the same bytes
                blob = np.frombuffer(layers[l].layer_blob(), np.uint8).copy()
                r2 = np.zeros((1, 4, 2048), np.float32)
                xf = x.astype(np.float32)[None].copy()
                rref.ref_moe_layer(3, blob.ctypes.data, xf.ctypes.data_as(O._f32p), idx[None].copy().ctypes.data_as(O._i32p),
                                   1, 4, r2.ctypes.data_as(O._f32p), 1)
                assert np.array_equal(r2[0], ref)
            for k in range(4):
                assert rel_l2(out[k].astype(np.float32), ref[k]) < 2e-3
        # bf16 input path (MLX hands bf16 over as uint16 bit patterns)
        xb = rng.randn(2048).astype(np.float32)
        xbits = O.f32_to_bf16_bits(xb)
        out = lib.expert_mlp_bf16(eng, 1, xbits, np.array([1, 4], np.int32), 2)
        ref = layers[1].moe(O.bf16_bits_to_f32(xbits)[None], np.array([[1, 4]], np.int32))[0]
        for k in range(2):
            assert rel_l2(out[k].astype(np.float32), ref[k]) < 2e-3
    finally:
        lib.destroy(eng)


def test_fp32_api_batch_prefill_and_pread(packed):
    from kandiga_b200 import _native as N
    d, layers = packed
    L = N.load()
    eng = L.bakan_cpu_expert_init(d.encode(), 2)
    assert eng
    try:
        rng = np.random.RandomState(1)
        x = rng.randn(2048).astype(np.float32)
        idx = np.array([2, 4], np.int32)
        out = np.zeros((2, 2048), np.float32)
        assert L.bakan_cpu_expert_mlp(eng, 0, x.ctypes.data_as(ctypes.c_void_p), idx.ctypes.data_as(N.c_i32p), 2,
                                      out.ctypes.data_as(ctypes.c_void_p)) == 0
        ref = layers[0].moe(x[None], idx[None])[0]
        assert rel_l2(out, ref) < 2e-3
        # batch: T tokens x K
        T, K = 3, 2
        xb = rng.randn(T, 2048).astype(np.float16)
        ib = rng.randint(0, 6, size=(T, K)).astype(np.int32)
        ob = np.zeros((T, K, 2048), np.float16)
        assert L.bakan_cpu_expert_mlp_batch_f16(eng, 1, xb.ctypes.data_as(ctypes.c_void_p),
                                                ib.ctypes.data_as(N.c_i32p), T, K,
                                                ob.ctypes.data_as(ctypes.c_void_p)) == 0
        rb = layers[1].moe(xb.astype(np.float32), ib)
        assert rel_l2(ob.astype(np.float32), rb) < 2e-3
        # CSR prefill (kandiga/engine.py:518-575 builds these arrays)
        s_tok, s_exp, s_k, starts, uniq = O.group_by_expert(ib)
        op = np.full((T, K, 2048), 7, np.float16)
        arrs = [np.ascontiguousarray(a, np.int32) for a in (s_tok, s_exp, s_k, starts, uniq)]
        assert L.bakan_cpu_expert_mlp_prefill_f16(eng, 1, xb.ctypes.data_as(ctypes.c_void_p), T, K, 2048,
                                                  *[a.ctypes.data_as(N.c_i32p) for a in arrs], len(uniq),
                                                  op.ctypes.data_as(ctypes.c_void_p)) == 0
        assert np.array_equal(op, ob)
        # CSR prefill on the tensor-core path (T >= 16) with the last group left
        # out: its (token, k) rows keep their previous contents
        T2 = 40
        x2 = rng.randn(T2, 2048).astype(np.float16)
        i2 = np.stack([rng.choice(6, K, replace=False) for _ in range(T2)]).astype(np.int32)
        ref2 = layers[1].moe(x2.astype(np.float32), i2)
        s_tok, s_exp, s_k, starts, uniq = O.group_by_expert(i2)
        ng = len(uniq) - 1
        arrs = [np.ascontiguousarray(a, np.int32) for a in (s_tok, s_exp, s_k, starts, uniq)]
        o2 = np.full((T2, K, 2048), 7, np.float16)
        assert L.bakan_cpu_expert_mlp_prefill_f16(eng, 1, x2.ctypes.data_as(ctypes.c_void_p), T2, K, 2048,
                                                  *[a.ctypes.data_as(N.c_i32p) for a in arrs], ng,
                                                  o2.ctypes.data_as(ctypes.c_void_p)) == 0
        left_out = i2 == uniq[-1]
        assert left_out.any() and (~left_out).any()
        assert np.all(o2[left_out] == 7)
        assert rel_l2(o2[~left_out].astype(np.float32), ref2[~left_out]) < 2e-3
        # pread_batch reconstructs the BKEX bytes bit-exactly from HBM
        ids = np.array([5, 1], np.int32)
        esz = layers[0].expert_size()
        buf = np.zeros(2 * esz, np.uint8)
        assert L.bakan_cpu_expert_pread_batch(eng, 0, ids.ctypes.data_as(N.c_i32p), 2,
                                              buf.ctypes.data_as(ctypes.c_void_p)) == 0
        assert buf[:esz].tobytes() == layers[0].expert_blob(5)
        assert buf[esz:].tobytes() == layers[0].expert_blob(1)
        # error convention: -1 for a bad layer, a bad K, a bad expert id
        assert L.bakan_cpu_expert_mlp(eng, 2, x.ctypes.data_as(ctypes.c_void_p), idx.ctypes.data_as(N.c_i32p), 2,
                                      out.ctypes.data_as(ctypes.c_void_p)) == -1
        assert L.bakan_cpu_expert_mlp(eng, 0, x.ctypes.data_as(ctypes.c_void_p), idx.ctypes.data_as(N.c_i32p), 17,
                                      out.ctypes.data_as(ctypes.c_void_p)) == -1
        bad = np.array([6], np.int32)
        assert L.bakan_cpu_expert_mlp(eng, 0, x.ctypes.data_as(ctypes.c_void_p), bad.ctypes.data_as(N.c_i32p), 1,
                                      out.ctypes.data_as(ctypes.c_void_p)) == -1
    finally:
        L.bakan_cpu_expert_destroy(eng)


def test_single_token_graph_replays_and_reallocation(packed):
    """Single-token calls replay one CUDA graph per (layer, K, dtypes): new
    inputs each call, and correct results again after a batch call grew the
    device buffers (which drops the graphs)."""
    from kandiga_b200 import _native as N
    d, layers = packed
    L = N.load()
    eng = L.bakan_cpu_expert_init(d.encode(), 2)
    assert eng
    try:
        rng = np.random.RandomState(7)

        def one(layer, K):
            x = rng.randn(2048).astype(np.float16)
            idx = rng.choice(6, K, replace=False).astype(np.int32)
            out = np.zeros((K, 2048), np.float16)
            assert L.bakan_cpu_expert_mlp_f16(eng, layer, x.ctypes.data_as(ctypes.c_void_p),
                                              idx.ctypes.data_as(N.c_i32p), K,
                                              out.ctypes.data_as(ctypes.c_void_p)) == 0
            ref = layers[layer].moe(x.astype(np.float32)[None], idx[None])[0]
            assert rel_l2(out.astype(np.float32), ref) < 2e-3

        for i in range(6):
            one(i % 2, 1 + i % 3)
        T, K = 96, 4
        xb = rng.randn(T, 2048).astype(np.float16)
        ib = np.stack([rng.choice(6, K, replace=False) for _ in range(T)]).astype(np.int32)
        ob = np.zeros((T, K, 2048), np.float16)
        assert L.bakan_cpu_expert_mlp_batch_f16(eng, 0, xb.ctypes.data_as(ctypes.c_void_p),
                                                ib.ctypes.data_as(N.c_i32p), T, K,
                                                ob.ctypes.data_as(ctypes.c_void_p)) == 0
        assert rel_l2(ob.astype(np.float32), layers[0].moe(xb.astype(np.float32), ib)) < 2e-3
        for i in range(6):
            one(i % 2, 1 + i % 3)
    finally:
        L.bakan_cpu_expert_destroy(eng)


def test_init_missing_dir_returns_null(gpu, tmp_path):
    from kandiga_b200 import _native as N
    L = N.load()
    assert not L.bakan_cpu_expert_init(str(tmp_path / "nope").encode(), 1)
