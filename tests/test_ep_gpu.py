"""Expert-parallel MoE over NCCL on 2 GPUs (tests/ep_gpu_worker.py) against the
full layer on one GPU; rel L2 < 2e-3 per call.  Skipped on boxes with one GPU."""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_ep_two_gpus(gpu):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    here = os.path.dirname(os.path.abspath(__file__))
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={port}", os.path.join(here, "ep_gpu_worker.py")]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    print(r.stdout[-3000:], r.stderr[-3000:])
    assert r.returncode == 0


def test_one_rank_fast_path_matches_exchange_path(gpu):
    """With one rank the routed MLP runs on the local table without permuting the
    T*K rows; it agrees with the generic per-row path."""
    import torch
    from kandiga_b200.ep import ExpertParallelMoE, ExpertPlacement, table_compute, table_local_moe, zipf_bias
    from tests.test_decode_gpu import get_layer, make_table, rel_l2
    E, K, T = 32, 4, 80
    layer = get_layer(3, 1024, 512, E, "f16", seed=21)
    tab = make_table(layer)
    pl = ExpertPlacement.balanced(np.exp(zipf_bias(E, 1.1, 3)), 1)
    order = torch.from_numpy(pl.experts_of(0).astype(np.int64))
    local = make_table(type(layer)(layer.bits, layer.hidden, layer.inter,
                                   [w[order.numpy()] for w in layer.w], [s[order.numpy()] for s in layer.s],
                                   [b[order.numpy()] for b in layer.b], sb_dtype=layer.sb_dtype))
    g = torch.Generator(device="cuda").manual_seed(2)
    x = torch.randn(T, 1024, generator=g, device="cuda").half()
    logits = torch.randn(T, E, generator=g, device="cuda")
    res = torch.randn(T, 1024, generator=g, device="cuda").half()
    fast = ExpertParallelMoE(pl, 0, K, table_compute(local), local_moe=table_local_moe(local))
    slow = ExpertParallelMoE(pl, 0, K, table_compute(local))
    a = fast.forward(0, x, logits, residual=res, out_dtype=torch.float16)
    b = slow.forward(0, x, logits, residual=res, out_dtype=torch.float16)
    full = tab.moe(0, x, logits=logits, top_k=K, combine=True, residual=res, out_dtype=torch.float16)["out"]
    assert rel_l2((a - res).float().cpu().numpy(), (full - res).float().cpu().numpy()) < 2e-3
    assert rel_l2((b - res).float().cpu().numpy(), (full - res).float().cpu().numpy()) < 2e-3
