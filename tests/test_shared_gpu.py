"""GPU parity of the MoE block with a shared expert (kq_shared_gate + the routed
paths with K+1 assignments) against the oracle: router top-K, the reference's
gate sigmoid(w_gate . x) (kandiga/metal/moe_block.metal:335-404), the expert MLPs
and the blend res + sum w_k y_k + gate * shared (moe_block.metal:556-584).
Tolerance: 2e-3 relative L2 per token row."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.test_decode_gpu import get_layer, make_table, rel_l2

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("T,path,gbits,gsb", [(4, "decode", 4, "bf16"), (64, "prefill", 4, "f16"),
                                              (3, "decode", 3, "f16"), (96, "prefill", 3, "bf16")])
def test_moe_block_with_shared_expert(gpu, T, path, gbits, gsb):
    E, H, I, K = 16, 2048, 512, 8
    layer = get_layer(4, H, I, E + 1, "f16", seed=60 + gbits)  # expert E is the shared expert
    t = make_table(layer)
    rng = np.random.RandomState(T)
    x = rng.randn(T, H).astype(np.float16)
    logits = rng.randn(T, E).astype(np.float32)
    res = rng.randn(T, H).astype(np.float32)
    gp, gs, gb = O.quantize_affine((rng.randn(1, H) * 0.02).astype(np.float32), gbits, 64, gsb)
    dev = torch.device("cuda")
    gate_t = (torch.from_numpy(np.ascontiguousarray(gp).view(np.uint8)).to(dev),
              torch.from_numpy(gs.view(np.int16)).to(dev), torch.from_numpy(gb.view(np.int16)).to(dev))
    r = t.moe_block(0, torch.from_numpy(x).to(dev), torch.from_numpy(logits).to(dev), K, gate_t, gate_bits=gbits,
                    gate_sb=gsb, residual=torch.from_numpy(res).to(dev), out_dtype=torch.float32, path=path)
    idx, w = O.router_topk(logits, K)
    gate = O.shared_gate(x, gp, gs, gb, gbits, gsb)
    assert np.array_equal(r["idx"].cpu().numpy()[:, :K], idx)
    assert np.all(r["idx"].cpu().numpy()[:, K] == E)
    np.testing.assert_allclose(r["gate"].cpu().numpy(), gate, rtol=1e-4, atol=1e-6)
    idx2 = np.concatenate([idx, np.full((T, 1), E, np.int32)], 1)
    y = layer.moe(x.astype(np.float32), idx2)
    want = O.combine(y[:, :K], w, res, shared=y[:, K], gate=gate)
    got = r["out"].cpu().numpy()
    worst = max(rel_l2(got[i], want[i]) for i in range(T))
    assert worst < 2e-3, worst
    assert t.status() == 0
