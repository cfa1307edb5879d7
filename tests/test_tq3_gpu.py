"""GPU parity of the TQ3_1S GEMV (kq_tq3_gemv) and reconstruction (kq_tq3_dequant)
against the numpy restatement pinned to kandiga/tq3/quantize.py: the kernel scores
the stored codes against the rotated input, so its output equals x @ W^T of the
oracle's reconstruction up to fp32 summation order (rel L2 < 1e-4)."""
import numpy as np
import pytest
import torch

from kandiga_b200 import tq3
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def rel_l2(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


def drop_means(data: bytes, nb: int) -> bytes:
    b = np.frombuffer(data, np.uint8).reshape(nb, 20)
    return np.concatenate([b[:, :4], b[:, 8:]], 1).tobytes()


@pytest.mark.parametrize("n,k,t,xdt", [(300, 2560, 1, torch.float16), (257, 2560, 5, torch.float32),
                                       (64, 9216, 2, torch.bfloat16), (1000, 1024, 4, torch.float16)])
def test_gemv_matches_oracle(gpu, n, k, t, xdt):
    rng = np.random.RandomState(n + k)
    w = (rng.randn(n, k) * 0.02).astype(np.float32)
    data, shape, nb = O.tq3_quantize(w)
    wd = O.tq3_dequantize(data, shape, nb).astype(np.float64)
    x = torch.from_numpy(rng.randn(t, k).astype(np.float32)).to(xdt)
    bias = rng.randn(n).astype(np.float32)
    m = tq3.TQ3Matrix(data, n, k)
    y = m.gemv(x.cuda(), torch.from_numpy(bias).cuda()).cpu().numpy()
    want = x.float().numpy().astype(np.float64) @ wd.T + bias
    assert rel_l2(y, want) < 1e-4


def test_sixteen_byte_blocks(gpu):
    rng = np.random.RandomState(3)
    n, k = 96, 512
    w = (rng.randn(n, k) * 0.02).astype(np.float32)
    data, shape, nb = O.tq3_quantize(w)
    d16 = drop_means(data, nb)
    wd = O.tq3_dequantize(d16, shape, nb).astype(np.float64)
    x = rng.randn(3, k).astype(np.float32)
    m = tq3.TQ3Matrix(d16, n, k, 16)
    y = m.gemv(torch.from_numpy(x).cuda()).cpu().numpy()
    assert rel_l2(y, x.astype(np.float64) @ wd.T) < 1e-4
    got = m.dequant().cpu().numpy()
    assert np.max(np.abs(got - wd)) <= 1e-6 * max(1.0, np.max(np.abs(wd)))


def test_dequantize_tensor_matches_oracle(gpu):
    rng = np.random.RandomState(4)
    w = (rng.randn(33, 70) * 0.05).astype(np.float32)  # ragged: blocks straddle rows, padded tail
    data, shape, nb = O.tq3_quantize(w)
    got = tq3.dequantize_tensor(data, shape, nb)
    want = O.tq3_dequantize(data, shape, nb)
    assert got.shape == w.shape
    assert np.max(np.abs(got - want)) <= 1e-6 * max(1.0, np.max(np.abs(want)))


def test_linear_forward(gpu):
    rng = np.random.RandomState(5)
    w = (rng.randn(128, 256) * 0.02).astype(np.float32)
    b = rng.randn(128).astype(np.float32)
    layer = tq3.TQ3Linear.from_linear(w, b)
    x = rng.randn(2, 7, 256).astype(np.float32)
    y = layer(torch.from_numpy(x).cuda()).cpu().numpy()
    wd = O.tq3_dequantize(layer.weight_data, layer.shape, layer.num_blocks).astype(np.float64)
    assert y.shape == (2, 7, 128)
    assert rel_l2(y, x.astype(np.float64) @ wd.T + b) < 1e-4
    cos = np.sum(w * wd) / (np.linalg.norm(w) * np.linalg.norm(wd))
    assert cos > 0.98  # TQ3 quality (kandiga README: cosine 0.990)
