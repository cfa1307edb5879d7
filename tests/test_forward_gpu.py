"""GPU parity of the MoE block engine (bakan_forward_*: the ABI declared in
kandiga/metal/bakan_forward.h) against the oracle composition of
kandiga/metal/moe_block.metal: RMSNorm -> quantized router -> softmax/top-K ->
routed experts -> shared expert + sigmoid gate -> blend + residual.
Tolerance: 2e-3 relative L2 of the block output."""
import ctypes

import numpy as np
import pytest

from oracle import oracle as O
from tests.test_bakan_gpu import rel_l2, write_bkex

pytestmark = pytest.mark.gpu
H, I, E, IS = 1024, 512, 32, 512
RTOL_L2 = 2e-3


@pytest.fixture(scope="module", params=["separate", "merged"])
def block(tmp_path_factory, gpu, request):
    """'separate': a 4-bit shared expert next to 3-bit routed experts (its own
    table, the separate gate kernel and combine); 'merged': a shared expert of
    the routed experts' shape, served as expert E of the routed table with the
    gate row inside the router GEMV (4 launches per block)."""
    shared_bits = 4 if request.param == "separate" else 3
    d = tmp_path_factory.mktemp("fwd")
    layers = [O.ExpertLayer.random(3, H, I, E, seed=60 + l, sb_dtype="bf16") for l in range(2)]
    write_bkex(str(d), layers)
    rng = np.random.RandomState(5)
    per = []
    for l in range(2):
        per.append(dict(
            norm=O.f32_to_bf16_bits((1.0 + 0.1 * rng.randn(H)).astype(np.float32)),
            router=O.quantize_affine((rng.randn(E, H) * 0.02).astype(np.float32), 4, 64, "bf16"),
            sgate=O.quantize_affine((rng.randn(1, H) * 0.02).astype(np.float32), 4, 64, "bf16"),
            shared=O.ExpertLayer.random(shared_bits, H, IS, 1, seed=80 + l, sb_dtype="bf16")))
    return str(d), layers, per


def put(L, eng, layer, wtype, arr, dtype):
    a = np.ascontiguousarray(arr)
    rows = a.shape[0] if a.ndim == 2 else 1
    cols = a.nbytes // (4 if dtype == 1 else 2) // rows
    return L.bakan_forward_set_weight(eng, layer, wtype, a.ctypes.data, a.nbytes, rows, cols, dtype)


def set_all(L, eng, layer, p):
    assert put(L, eng, layer, 0, p["norm"], 2) == 0
    for t0, (pk, s, b) in ((1, p["router"]), (4, p["sgate"])):
        assert put(L, eng, layer, t0, pk, 1) == 0
        assert put(L, eng, layer, t0 + 1, s, 2) == 0
        assert put(L, eng, layer, t0 + 2, b, 2) == 0
    sh = p["shared"]  # ExpertLayer matrices: 0 gate, 1 up, 2 down
    for t0, m in ((7, 1), (10, 0), (13, 2)):
        assert put(L, eng, layer, t0, sh.w[m][0], 1) == 0
        assert put(L, eng, layer, t0 + 1, sh.s[m][0], 2) == 0
        assert put(L, eng, layer, t0 + 2, sh.b[m][0], 2) == 0


def oracle_block(layer, p, h, normed_input, K=8, eps=1e-6):
    x = h if normed_input else O.rms_norm(h, O.bf16_bits_to_f32(p["norm"]), eps)
    xf = x.astype(np.float32)
    rpk, rs, rb = p["router"]
    logits = O.matvec(4, rpk, rs, rb, xf, "bf16")
    idx, w = O.router_topk(logits[None], K)
    y = layer.moe(xf[None], idx)
    gpk, gs, gb = p["sgate"]
    gate = O.shared_gate(xf[None], gpk, gs, gb, 4, "bf16")  # router and gate rows: 4-bit
    shared = p["shared"].moe(xf[None], np.zeros((1, 1), np.int32))[0, 0].astype(np.float16).astype(np.float32)
    res = None if normed_input else h.astype(np.float32)[None]
    return logits, O.combine(y, w, res, shared[None], gate)[0]


def routing_is_clear(logits, K):
    s = np.sort(logits)[::-1]
    return s[K - 1] - s[K] > 1e-3


def test_moe_block_matches_oracle(block):
    from kandiga_b200 import _native as N
    d, layers, per = block
    L = N.load()
    eng = L.bakan_forward_init(d.encode(), 2)
    assert eng
    try:
        assert L.bakan_forward_num_layers(eng) == 2
        for l in range(2):
            set_all(L, eng, l, per[l])
        rng = np.random.RandomState(11)
        checked = 0
        for it in range(8):  # repeated calls replay the layer's graph with new inputs
            l = it % 2
            h = rng.randn(H).astype(np.float16)
            for normed in (False, True):
                _, ref = oracle_block(layers[l], per[l], h, normed)
                logits = oracle_block(layers[l], per[l], h, normed)[0]
                if not routing_is_clear(logits, 8):
                    continue
                out = np.zeros(H, np.float16)
                fn = L.bakan_forward_moe_block_normed if normed else L.bakan_forward_moe_block
                assert fn(eng, l, h.ctypes.data, out.ctypes.data) == 0
                assert rel_l2(out.astype(np.float32), ref) < RTOL_L2
                checked += 1
        assert checked >= 8
        # top-K and epsilon are the block parameters the reference fixes
        assert L.kq_forward_set_params(eng, 4, ctypes.c_float(1e-5)) == 0
        h = rng.randn(H).astype(np.float16)
        logits, ref = oracle_block(layers[0], per[0], h, False, K=4, eps=1e-5)
        if routing_is_clear(logits, 4):
            out = np.zeros(H, np.float16)
            assert L.bakan_forward_moe_block(eng, 0, h.ctypes.data, out.ctypes.data) == 0
            assert rel_l2(out.astype(np.float32), ref) < RTOL_L2
        assert L.kq_forward_set_params(eng, 0, ctypes.c_float(1e-6)) == N.ERRORS_INV["KQ_ERR_ARG"]
    finally:
        L.bakan_forward_destroy(eng)


def test_moe_block_errors(block):
    from kandiga_b200 import _native as N
    d, layers, per = block
    L = N.load()
    eng = L.bakan_forward_init(d.encode(), 2)
    assert eng
    try:
        h = np.zeros(H, np.float16)
        out = np.zeros(H, np.float16)
        # no weights set yet, a bad layer, a bad weight type, a size that does not match the shape
        assert L.bakan_forward_moe_block(eng, 0, h.ctypes.data, out.ctypes.data) == -1
        assert L.bakan_forward_moe_block(eng, 2, h.ctypes.data, out.ctypes.data) == -1
        a = np.zeros(16, np.uint16)
        assert L.bakan_forward_set_weight(eng, 0, 16, a.ctypes.data, a.nbytes, 1, 16, 2) == -1
        assert L.bakan_forward_set_weight(eng, 0, 0, a.ctypes.data, a.nbytes - 2, 1, 16, 2) == -1
        # the normed variant needs no norm weight; the full block does
        p = dict(per[0])
        set_all(L, eng, 0, p)
        assert L.bakan_forward_moe_block_normed(eng, 0, h.ctypes.data, out.ctypes.data) == 0
        assert L.bakan_forward_moe_block(eng, 1, h.ctypes.data, out.ctypes.data) == -1
    finally:
        L.bakan_forward_destroy(eng)
    assert not L.bakan_forward_init(b"/nonexistent", 1)
