"""Generate the golden fixtures in tests/golden/ from the reference itself.

Runs only where the reference tree is mounted ($KQ_REFERENCE_ROOT, or a
directory named `reference` beside this repository).  The fixtures it writes are committed; the GPU box and the
test suite never read the reference tree.

Fixtures:
  tq3_golden.npz      kandiga/tq3/quantize.py imported directly (pure numpy):
                      quantize_tensor blocks and dequantize_tensor output for
                      seeded weights, plus the 16-byte legacy block format.
  turboquant_golden.npz
                      kandiga/kv_compress.py TurboQuantCache run on a small
                      numpy-backed stand-in for mlx.core (MLX is not installed
                      here).  The stand-in maps each mx op the module uses to
                      the numpy op with the same documented semantics (round
                      half-to-even, fp32 matmul, etc.).
  bkex_header.bin     kandiga/_pack_experts.py _build_header for the 3-bit
                      H2048/I512/E256 layer, imported with the same stand-in
                      (the function itself uses only struct).
  expert_golden.npz   kandiga/metal/kandiga_cpu_expert.m scalar C (compiled by
                      oracle/build_ref.py): outputs of compute_single_expert_3bit
                      and compute_single_expert (4-bit) for seeded experts.

Usage: python tests/golden/make_golden.py
"""
from __future__ import annotations

import hashlib
import importlib.util
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
from oracle.build_ref import reference_root  # noqa: E402

REF = reference_root()


def _load(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _mlx_standin():
    """numpy-backed stand-in for the mlx.core ops kv_compress.py and
    _pack_experts.py touch."""
    core = types.ModuleType("mlx.core")
    core.float16, core.float32, core.int8, core.int32 = np.float16, np.float32, np.int8, np.int32
    core.uint32, core.bool_ = np.uint32, np.bool_
    core.bfloat16 = np.float32  # unused by the code paths exercised here
    core.array = lambda a, dtype=None: np.asarray(a, dtype=dtype)
    core.min = lambda a, axis=None, keepdims=False: np.min(a, axis=axis, keepdims=keepdims)
    core.max = lambda a, axis=None, keepdims=False: np.max(a, axis=axis, keepdims=keepdims)
    core.where = np.where
    core.ones_like = np.ones_like
    core.clip = np.clip
    core.round = np.round  # half-to-even, like mlx.core.round
    core.concatenate = lambda xs, axis=0: np.concatenate(xs, axis=axis)
    core.expand_dims = lambda a, axis: np.expand_dims(a, axis)
    core.eval = lambda *a, **k: None
    pkg = types.ModuleType("mlx")
    pkg.core = core
    sys.modules["mlx"] = pkg
    sys.modules["mlx.core"] = core
    return core


def make_tq3():
    q = _load("ref_tq3_quantize", os.path.join(REF, "kandiga", "tq3", "quantize.py"))
    rng = np.random.RandomState(1234)
    w = (rng.randn(8, 256) * 0.02).astype(np.float32)
    # include an all-zero block row and an outlier block
    w[3, :32] = 0.0
    w[5, 64:96] *= 50.0
    data, shape, nb = q.quantize_tensor(w)
    deq = q.dequantize_tensor(data, shape, nb)
    # legacy 16-byte blocks: d0, d1 fp16 + 12 B codes
    rng2 = np.random.RandomState(77)
    legacy = bytearray()
    for _ in range(6):
        d = rng2.rand(2).astype(np.float16)
        codes = q._pack_indices(rng2.randint(0, 8, 32).astype(np.uint8))
        legacy += d.tobytes() + codes.tobytes()
    deq16 = q.dequantize_tensor(bytes(legacy), (6 * 32,), 6)
    xw = rng.randn(32).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "tq3_golden.npz"), w=w,
                        blocks=np.frombuffer(data, np.uint8), num_blocks=nb, deq=deq,
                        legacy_blocks=np.frombuffer(bytes(legacy), np.uint8), legacy_deq=deq16,
                        wht_in=xw, wht_fwd=q._wht_forward(xw), wht_inv=q._wht_inverse(xw))
    print("tq3_golden.npz", nb, "blocks")


def make_turboquant():
    _mlx_standin()
    kv = _load("ref_kv_compress", os.path.join(REF, "kandiga", "kv_compress.py"))
    out = {}
    for tag, (D, H, S, seed, dseed) in {"a": (64, 4, 16, 123, 42), "b": (128, 2, 9, 42, 7)}.items():
        cache = kv.TurboQuantCache(head_dim=D, num_heads=H, seed=seed)
        rng = np.random.RandomState(dseed)
        k = rng.randn(1, H, S, D).astype(np.float32)
        v = rng.randn(1, H, S, D).astype(np.float32)
        k[..., 3] *= 8.0
        # two appends: S-1 tokens then 1 token (exercises concatenate)
        cache.update(k[:, :, :S - 1], v[:, :, :S - 1])
        cache.update(k[:, :, S - 1:], v[:, :, S - 1:])
        out.update({f"{tag}_k": k, f"{tag}_v": v, f"{tag}_rotation": np.asarray(cache.rotation),
                    f"{tag}_qjl": np.asarray(cache.qjl_proj), f"{tag}_kq": cache.k_quant,
                    f"{tag}_ks": cache.k_scales, f"{tag}_kz": cache.k_zeros,
                    f"{tag}_ksign": cache.k_qjl_signs, f"{tag}_vq": cache.v_quant,
                    f"{tag}_vs": cache.v_scales, f"{tag}_vz": cache.v_zeros,
                    f"{tag}_vsign": cache.v_qjl_signs, f"{tag}_keys": np.asarray(cache.keys),
                    f"{tag}_values": np.asarray(cache.values),
                    f"{tag}_meta": np.array([D, H, S, seed, cache.seq_len, cache.memory_bytes])})
    np.savez_compressed(os.path.join(HERE, "turboquant_golden.npz"), **out)
    print("turboquant_golden.npz")


def make_bkex():
    _mlx_standin()
    pk = _load("ref_pack_experts", os.path.join(REF, "kandiga", "_pack_experts.py"))
    H, I, bits, E = 2048, 512, 3, 256
    order = []
    for name, rows, cols in (("gate_proj", I, H), ("up_proj", I, H), ("down_proj", H, I)):
        wc = cols * bits // 32
        order.append((f"{name}.weight", (rows, wc), "uint32", rows * wc * 4))
        order.append((f"{name}.scales", (rows, cols // 64), "bfloat16", rows * cols // 64 * 2))
        order.append((f"{name}.biases", (rows, cols // 64), "bfloat16", rows * cols // 64 * 2))
    esz = sum(t[3] for t in order)
    hdr = pk._build_header(E, esz, order)
    with open(os.path.join(HERE, "bkex_header.bin"), "wb") as f:
        f.write(hdr)
    print("bkex_header.bin", esz)


def make_expert():
    from oracle import build_ref, oracle as O
    build_ref.build(REF)
    ref = O.ref_lib("small")
    out = {}
    for bits in (3, 4):
        layer = O.ExpertLayer.random(bits, 2048, 512, 3, seed=100 + bits, sb_dtype="bf16")
        rng = np.random.RandomState(200 + bits)
        x = rng.randn(2048).astype(np.float32)
        ys = []
        for e in range(layer.num_experts):
            blob = np.frombuffer(layer.expert_blob(e), np.uint8).copy()
            y = np.zeros(2048, np.float32)
            ref.ref_expert(bits, blob.ctypes.data, x.ctypes.data_as(O._f32p), y.ctypes.data_as(O._f32p))
            ys.append(y)
        digest = hashlib.sha256(layer.layer_blob()).hexdigest()
        out.update({f"b{bits}_x": x, f"b{bits}_y": np.stack(ys),
                    f"b{bits}_sha": np.frombuffer(digest.encode(), np.uint8)})
    np.savez_compressed(os.path.join(HERE, "expert_golden.npz"), **out)
    print("expert_golden.npz")


if __name__ == "__main__":
    make_tq3()
    make_turboquant()
    make_bkex()
    make_expert()
