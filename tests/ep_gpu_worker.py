"""One rank of the 2-GPU expert-parallel check (run by tests/test_ep_gpu.py under
torch.distributed.run): EP forward over NCCL, then over the peer-memory
exchange (kq_ep), against the full layer on one GPU."""
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
from kandiga_b200.ep import ExpertParallelMoE, ExpertPlacement, table_compute, zipf_bias  # noqa: E402
from kandiga_b200.experts import ExpertTable  # noqa: E402
from kandiga_b200.quant import quantize_affine  # noqa: E402

E, H, I, K = 32, 2048, 512, 8


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    lr = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(lr)
    dev = torch.device("cuda", lr)
    dist.init_process_group("nccl", device_id=dev)
    g = torch.Generator(device=dev).manual_seed(1)
    mats = []
    for rows, cols in ((I, H), (I, H), (H, I)):
        w = torch.randn(E * rows, cols, generator=g, device=dev) * 0.02
        p, s, b = quantize_affine(w, 3, 64, "f16")
        mats.append((p.reshape(E, rows, -1).contiguous(), s.reshape(E, rows, -1).view(torch.int16).contiguous(),
                     b.reshape(E, rows, -1).view(torch.int16).contiguous()))
    full = ExpertTable(1, E, H, I, 3, "f16")
    full.load_mlx(0, *mats)
    pl = ExpertPlacement.balanced(np.exp(zipf_bias(E, 1.1, 7)), world)
    mine = torch.from_numpy(pl.experts_of(rank)).to(dev)
    local = ExpertTable(1, len(mine), H, I, 3, "f16")
    local.load_mlx(0, *[(m[0][mine].contiguous(), m[1][mine].contiguous(), m[2][mine].contiguous()) for m in mats])
    ok = True
    for T in (3, 40):
        gt = torch.Generator(device=dev).manual_seed(100 + rank + T)
        x = torch.randn(T, H, generator=gt, device=dev).half()
        logits = torch.randn(T, E, generator=gt, device=dev) + torch.from_numpy(zipf_bias(E, 1.1, 7)).to(dev)
        res = torch.randn(T, H, generator=gt, device=dev)
        ep = ExpertParallelMoE(pl, rank, K, table_compute(local))
        out = ep.forward(0, x, logits, residual=res, out_dtype=torch.float32)
        ref = full.moe(0, x, logits=logits, top_k=K, combine=True, residual=res, out_dtype=torch.float32,
                       path="decode")["out"]
        err = (torch.linalg.norm(out - ref) / torch.linalg.norm(ref)).item()
        print(f"rank {rank} T {T} rel_l2 {err:.3e}", flush=True)
        ok &= err < 2e-3 and local.status() == 0
    # the same layer through the peer-memory exchange (kq_ep over CUDA IPC)
    from kandiga_b200.ep import PeerExchange, PeerExpertParallelMoE
    ex = PeerExchange(rank, world, 40, H, K, torch.float16)
    ex.connect()
    pm = PeerExpertParallelMoE(pl, rank, K, local, ex)
    for T in (3, 40, 0, 17):
        gt = torch.Generator(device=dev).manual_seed(200 + rank + T)
        x = torch.randn(T, H, generator=gt, device=dev).half()
        logits = torch.randn(T, E, generator=gt, device=dev) + torch.from_numpy(zipf_bias(E, 1.1, 7)).to(dev)
        res = torch.randn(T, H, generator=gt, device=dev)
        out = pm.forward(0, x, logits=logits, residual=res, out_dtype=torch.float32)
        st, site = ex.status()
        if T == 0:
            ok &= st == 0 and out.shape[0] == 0
            continue
        ref = full.moe(0, x, logits=logits, top_k=K, combine=True, residual=res, out_dtype=torch.float32,
                       path="decode")["out"]
        err = (torch.linalg.norm(out - ref) / torch.linalg.norm(ref - res)).item()
        print(f"rank {rank} peer T {T} rel_l2 {err:.3e} status {st} site {site}", flush=True)
        ok &= err < 2e-3 and st == 0 and local.status() == 0
    torch.cuda.synchronize()
    dist.barrier()
    ex.close()
    flag = torch.tensor([0 if ok else 1], device=dev)
    dist.all_reduce(flag)
    dist.destroy_process_group()
    sys.exit(int(flag.item() != 0))


if __name__ == "__main__":
    main()
