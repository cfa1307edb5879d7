"""GPU parity of the dense quantized GEMV (shared / dense-layer path) against the
C oracle matvec (kandiga/metal/kandiga_cpu_expert.m:105-299 semantics) and a
torch fp32 reference for the fused RMSNorm prologue and SwiGLU pair."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


def qmat_from(bits, rows, cols, seed, sb="f16", pair=False):
    from kandiga_b200.experts import QuantizedLinear
    rng = np.random.RandomState(seed)
    mats = []
    for _ in range(2 if pair else 1):
        W = (rng.randn(rows, cols) * 0.02).astype(np.float32)
        mats.append(O.quantize_affine(W, bits, 64, sb))
    q = QuantizedLinear(rows, cols, bits, sb, pair)
    dev = [(torch.from_numpy(p.view(np.uint8).reshape(rows, -1)).cuda(), torch.from_numpy(s.view(np.int16)).cuda(),
            torch.from_numpy(b.view(np.int16)).cuda()) for p, s, b in mats]
    q.load_mlx(dev[0], dev[1] if pair else None)
    torch.cuda.synchronize()
    return q, mats


@pytest.mark.parametrize("bits,rows,cols,T", [(3, 512, 2560, 2), (4, 256, 2048, 2), (3, 2560, 9216, 2),
                                              (3, 4096, 2560, 2), (3, 6144, 2560, 2), (4, 4112, 2048, 3)])
def test_dense_gemv_matches_oracle(gpu, bits, rows, cols, T):
    """Launch shapes with 1, 2 and 4 row tiles per CTA; 4112 rows (257 row
    tiles) leave the last CTA of each token one row tile."""
    q, mats = qmat_from(bits, rows, cols, seed=rows + cols)
    p, s, b = mats[0]
    w, ss, bb = q.unpack_mlx(0)
    assert np.array_equal(w.cpu().numpy().reshape(-1), p.view(np.uint8).reshape(-1))
    assert np.array_equal(ss.cpu().numpy().view(np.uint16), s)
    x = np.random.RandomState(1).randn(T, cols).astype(np.float16)
    y = q(torch.from_numpy(x).cuda(), out_dtype=torch.float32).cpu().numpy()
    for t in range(T):
        ref = O.matvec(bits, p, s, b, x[t].astype(np.float32), "f16")
        assert rel_l2(y[t], ref) < 2e-3


def test_dense_pair_swiglu_and_rmsnorm(gpu):
    rows, cols = 512, 2560
    q, mats = qmat_from(3, rows, cols, seed=3, pair=True)
    rng = np.random.RandomState(2)
    x = rng.randn(1, cols).astype(np.float16)
    nw = (1 + 0.1 * rng.randn(cols)).astype(np.float16)
    y = q(torch.from_numpy(x).cuda(), norm_weight=torch.from_numpy(nw).cuda(), eps=1e-6,
          out_dtype=torch.float32).cpu().numpy()
    xf = x.astype(np.float32)[0]
    xn = xf / np.sqrt(np.mean(xf * xf) + 1e-6) * nw.astype(np.float32)
    g = O.matvec(3, *mats[0], xn, "f16")
    u = O.matvec(3, *mats[1], xn, "f16")
    ref = g / (1 + np.exp(-g)) * u
    assert rel_l2(y[0], ref) < 2e-3
