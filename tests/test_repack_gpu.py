"""GPU re-quantization (kq_requantize_mlx, kandiga_b200.repack) against the
oracle composition dequantize_affine -> round to the scale dtype ->
quantize_affine: codes, scales and biases bit-exact; whole BKEX layer files
repacked 4-bit -> 3-bit as scripts/repack_experts_3bit.py does."""
import os

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def oracle_requant(packed, s, b, cols, src_bits, dst_bits, sb="bf16"):
    v = O.dequantize_affine(packed, s, b, src_bits, cols, 64, sb)
    v = O.sb_to_f32(O.f32_to_sb(v, sb), sb)  # held in the scale dtype
    return O.quantize_affine(v, dst_bits, 64, sb)


@pytest.mark.parametrize("src,dst,sb", [(4, 3, "bf16"), (3, 4, "bf16"), (4, 3, "f16"), (4, 4, "bf16")])
def test_requantize_matches_oracle(gpu, src, dst, sb):
    from kandiga_b200.repack import requantize
    rng = np.random.RandomState(src * 10 + dst)
    rows, cols = 96, 1024
    w = (rng.randn(rows, cols) * 0.02).astype(np.float32)
    w[3, :64] = 0.5  # a constant group
    pk, s, b = O.quantize_affine(w, src, 64, sb)
    want = oracle_requant(pk, s, b, cols, src, dst, sb)
    got = requantize(torch.from_numpy(np.ascontiguousarray(pk).view(np.uint8)).cuda(),
                     torch.from_numpy(s.view(np.int16)).cuda(), torch.from_numpy(b.view(np.int16)).cuda(),
                     cols, src, dst, sb)
    assert np.array_equal(got[0].cpu().numpy(), np.ascontiguousarray(want[0]).view(np.uint8).reshape(rows, -1))
    assert np.array_equal(got[1].cpu().numpy().view(np.uint16), want[1])
    assert np.array_equal(got[2].cpu().numpy().view(np.uint16), want[2])


def test_repack_layer_files(gpu, tmp_path):
    from kandiga_b200.repack import parse_header, repack_dir
    from tests.test_bakan_gpu import write_bkex
    src = tmp_path / "packed"
    src.mkdir()
    layers = [O.ExpertLayer.random(4, 1024, 512, 5, seed=30 + l, sb_dtype="bf16") for l in range(2)]
    write_bkex(str(src), layers)
    out, sizes = repack_dir(str(src))
    assert os.path.basename(out) == "packed_3bit" and len(sizes) == 2
    for l, layer in enumerate(layers):
        data = open(os.path.join(out, f"layer_{l:02d}.bin"), "rb").read()
        n, esz, tensors = parse_header(data[:4096])
        assert n == 5 and esz == sizes[l] == 3 * 512 * 1024 * (3 / 8 + 4 / 64)
        by = {t["name"]: t for t in tensors}
        for e in range(5):
            blob = data[4096 + e * esz:4096 + (e + 1) * esz]
            for m, proj in enumerate(("gate_proj", "up_proj", "down_proj")):
                cols = layer.hidden if m < 2 else layer.inter
                want = oracle_requant(layer.w[m][e], layer.s[m][e], layer.b[m][e], cols, 4, 3)
                for k, arr in zip(("weight", "scales", "biases"), want):
                    t = by[f"{proj}.{k}"]
                    assert blob[t["offset"]:t["offset"] + t["nbytes"]] == np.ascontiguousarray(arr).tobytes()
    # the repacked files serve the reference ABI as a 3-bit layer
    from kandiga_b200 import _native as N
    import ctypes
    L = N.load()
    eng = L.bakan_cpu_expert_init(out.encode(), 2)
    assert eng
    try:
        ref = O.ExpertLayer(3, 1024, 512, *[[np.stack([oracle_requant(layers[0].w[m][e], layers[0].s[m][e],
                                                                       layers[0].b[m][e], 1024 if m < 2 else 512,
                                                                       4, 3)[i] for e in range(5)])
                                               for m in range(3)] for i in range(3)], sb_dtype="bf16")
        x = np.random.RandomState(2).randn(1024).astype(np.float16)
        idx = np.array([4, 0, 2], np.int32)
        o = np.zeros((3, 1024), np.float16)
        assert L.bakan_cpu_expert_mlp_f16(eng, 0, x.ctypes.data_as(ctypes.c_void_p), idx.ctypes.data_as(N.c_i32p),
                                          3, o.ctypes.data_as(ctypes.c_void_p)) == 0
        y = ref.moe(x.astype(np.float32)[None], idx[None])[0]
        from tests.test_bakan_gpu import rel_l2
        assert rel_l2(o.astype(np.float32), y) < 2e-3
    finally:
        L.bakan_cpu_expert_destroy(eng)
