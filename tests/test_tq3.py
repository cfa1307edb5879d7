"""TQ3_1S host logic on CPU: the product quantizer (torch float64) against the
numpy restatement pinned to kandiga/tq3/quantize.py, and the TQ31 file format."""
import numpy as np

from kandiga_b200 import tq3
from oracle import oracle as O


def test_quantizer_matches_oracle_blocks():
    rng = np.random.RandomState(0)
    w = (rng.randn(64, 256) * 0.02).astype(np.float32)
    data, shape, nb = tq3.quantize_tensor(w)
    ref, rshape, rnb = O.tq3_quantize(w)
    assert shape == rshape and nb == rnb == 64 * 256 // 32
    a = np.frombuffer(data, np.uint8).reshape(nb, 20)
    b = np.frombuffer(ref, np.uint8).reshape(nb, 20)
    same = np.mean(np.all(a == b, axis=1))
    assert same >= 0.999, same
    wa = O.tq3_dequantize(data, shape, nb)
    wb = O.tq3_dequantize(ref, shape, nb)
    assert np.max(np.abs(wa - wb)) < 1e-3


def test_pack_matches_oracle():
    rng = np.random.RandomState(1)
    idx = rng.randint(0, 8, (50, 32))
    import torch
    got = tq3._pack(torch.from_numpy(idx)).numpy()
    assert np.array_equal(got, O.tq3_pack_indices(idx.astype(np.uint8)))


def test_linear_file_roundtrip(tmp_path):
    rng = np.random.RandomState(2)
    w = (rng.randn(8, 64) * 0.05).astype(np.float32)
    bias = rng.randn(8).astype(np.float32)
    layer = tq3.TQ3Linear.from_linear(w, bias)
    p = str(tmp_path / "l.tq3")
    layer.save(p)
    back = tq3.TQ3Linear.load(p)
    assert back.shape == (8, 64) and back.num_blocks == 16 and back.weight_data == layer.weight_data
    assert np.allclose(back.bias, bias.astype(np.float16).astype(np.float32))
    assert layer.memory_bytes == len(layer.weight_data) + bias.nbytes
    assert abs(layer.compression_ratio - 8 * 64 * 2 / layer.memory_bytes) < 1e-12
