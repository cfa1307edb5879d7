"""GPU quantizer (kandiga_b200.quant.quantize_affine, torch on the device) against
the numpy restatement of MLX's affine quantizer (oracle.quantize_affine; call
sites scripts/repack_experts_3bit.py:91-94, scripts/convert_3bit.py:52-70):
packed codes, scales and biases bit-exact, in both modes, for ordinary,
constant, all-zero, one-signed and wide-range groups."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu


def weights(seed):
    rng = np.random.RandomState(seed)
    w = (rng.randn(96, 1024) * 0.02).astype(np.float32)
    w[0, :64] = 0.5                       # constant group
    w[1, :64] = 0.0                       # all-zero group
    w[2, :64] = np.abs(w[2, :64]) + 0.01  # one-signed, positive
    w[3, :64] = -np.abs(w[3, :64]) - 0.01 # one-signed, negative
    w[4, :64] *= 3000.0                   # wide range (fp16 scale still finite)
    w[5, :64] *= 1e-4                     # tiny values (fp16 subnormal scales)
    w[6, 64:128] = np.linspace(-1, 0.5, 64)
    return w


@pytest.mark.parametrize("mode", ["edge", "minmax"])
@pytest.mark.parametrize("bits,sb", [(3, "f16"), (4, "f16"), (3, "bf16"), (4, "bf16")])
def test_gpu_quantizer_matches_oracle(gpu, bits, sb, mode):
    from kandiga_b200.quant import dequantize_affine, quantize_affine
    w = weights(bits * 10 + (sb == "bf16"))
    p_ref, s_ref, b_ref = O.quantize_affine(w, bits, 64, sb, mode=mode)
    p, s, b = quantize_affine(torch.from_numpy(w).cuda(), bits, 64, sb, mode=mode)
    torch.cuda.synchronize()
    assert np.array_equal(p.cpu().numpy().view(np.uint8).reshape(-1),
                          np.ascontiguousarray(p_ref).view(np.uint8).reshape(-1))
    assert np.array_equal(s.view(torch.int16).cpu().numpy().view(np.uint16), s_ref)
    assert np.array_equal(b.view(torch.int16).cpu().numpy().view(np.uint16), b_ref)
    # and the device dequantization agrees with the oracle's
    deq = dequantize_affine(p, s, b, bits, w.shape[1]).cpu().numpy()
    want = O.dequantize_affine(p_ref, s_ref, b_ref, bits, w.shape[1], 64, sb)
    np.testing.assert_allclose(deq, want, rtol=1e-6, atol=1e-12)
