"""Edge cases across the GPU paths: empty batches, top-1 and the largest top-K
the kernels take (32), a single-expert table, one token through the prefill
path, and a TurboQuant cache filled one token at a time against a bulk fill."""
import numpy as np
import pytest
import torch

from oracle import oracle as O
from tests.test_decode_gpu import get_layer, make_table, rel_l2

pytestmark = pytest.mark.gpu
RTOL_L2 = 2e-3


def per_k_ok(layer, x, idx, per_k):
    y = layer.moe(x.float().cpu().numpy(), idx)
    pk = per_k.float().cpu().numpy()
    return max(rel_l2(pk[i, k], y[i, k]) for i in range(idx.shape[0]) for k in range(idx.shape[1]))


def test_prefill_empty_batch(gpu):
    t = make_table(get_layer(4, 1024, 512, 8, "f16", seed=1))
    x = torch.empty(0, 1024, device="cuda", dtype=torch.float16)
    idx = torch.empty(0, 2, device="cuda", dtype=torch.int32)
    r = t.moe(0, x, idx=idx, per_k=True, combine=False, out_dtype=torch.float32, path="prefill")
    assert r["per_k"].shape == (0, 2, 1024) and t.status() == 0


@pytest.mark.parametrize("path", ["prefill", "decode"])
@pytest.mark.parametrize("K,E,T", [(1, 16, 40), (32, 64, 24)])
def test_top1_and_top32(gpu, path, K, E, T):
    layer = get_layer(3, 1024, 512, E, "bf16", seed=K + E)
    t = make_table(layer)
    rng = np.random.RandomState(K)
    x = torch.from_numpy(rng.randn(T, 1024).astype(np.float16)).cuda()
    logits = torch.from_numpy(rng.randn(T, E).astype(np.float32)).cuda()
    r = t.moe(0, x, logits=logits, top_k=K, per_k=True, combine=True, out_dtype=torch.float32, path=path)
    idx_ref, w_ref = O.router_topk(logits.cpu().numpy(), K)
    assert np.array_equal(r["idx"].cpu().numpy(), idx_ref)
    assert per_k_ok(layer, x, idx_ref, r["per_k"]) < RTOL_L2
    want = O.combine(layer.moe(x.float().cpu().numpy(), idx_ref), r["weights"].cpu().numpy())
    assert rel_l2(r["out"].cpu().numpy(), want) < RTOL_L2
    assert t.status() == 0


def test_single_expert_table_and_single_token_prefill(gpu):
    layer = get_layer(4, 1024, 512, 1, "f16", seed=3)
    t = make_table(layer)
    x = torch.randn(1, 1024, device="cuda").half()
    idx = torch.zeros(1, 1, dtype=torch.int32, device="cuda")
    for path in ("prefill", "decode"):
        r = t.moe(0, x, idx=idx, per_k=True, combine=False, out_dtype=torch.float32, path=path)
        assert per_k_ok(layer, x, idx.cpu().numpy(), r["per_k"]) < RTOL_L2
    assert t.status() == 0


def test_turbo_token_by_token_equals_bulk(gpu):
    """Per-vector quantization: 300 one-token appends give the same codes, scales
    and attention as one 300-token append."""
    from kandiga_b200.kv_compress import TurboQuantCache
    g = torch.Generator(device="cuda").manual_seed(8)
    k = torch.randn(1, 2, 300, 128, generator=g, device="cuda").half()
    v = torch.randn(1, 2, 300, 128, generator=g, device="cuda").half()
    bulk = TurboQuantCache(128, 2, capacity=16)
    bulk.update(k, v)
    step = TurboQuantCache(128, 2, capacity=1)
    step.update(k[:, :, :0], v[:, :, :0])  # an empty append is a no-op
    assert step.seq_len == 0
    for i in range(300):
        step.update(k[:, :, i:i + 1], v[:, :, i:i + 1])
    assert step.seq_len == bulk.seq_len == 300
    for a, b in zip(step.state(), bulk.state()):
        assert torch.equal(a, b)
    q = torch.randn(1, 4, 128, generator=g, device="cuda").half()  # grouped-query: 2 query heads per KV head
    assert torch.equal(step.attend(q), bulk.attend(q))
