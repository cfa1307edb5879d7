"""kq_moe_decode_static: the decode entry point for callers that cannot allocate
device memory (runtimes that give a plugin only its inputs and outputs, plain-FFI
hosts without a device allocator).  Its scratch is a fixed array inside libkq.so.

Checked through the C ABI against kq_moe_decode with a caller workspace, on two
calls in a row with different shapes (the second call must not see the first
call's leftovers).  This file is collected last (its name sorts after every
other test file): the entry point is the most recent addition, so a run that
stops at the first failure has already run the whole established suite, and
it exercises the shared static array after other kernels have run in the
same process.  It also passes run alone in a fresh process."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle as O

pytestmark = pytest.mark.gpu
RTOL_L2 = 2e-3


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


def test_static_decode_matches_workspace_decode(gpu):
    from kandiga_b200 import _native as N
    from kandiga_b200.experts import ExpertTable
    lib = N.load()
    E, H, I = 16, 2048, 512
    layer = O.ExpertLayer.random(3, H, I, E, seed=31, sb_dtype="f16")
    t = ExpertTable(1, E, H, I, 3, "f16")
    t.load_mlx(0, *[(torch.from_numpy(layer.w[m].reshape(E, layer.w[m].shape[1], -1)).cuda(),
                     torch.from_numpy(layer.s[m].view(np.int16)).cuda(),
                     torch.from_numpy(layer.b[m].view(np.int16)).cuda()) for m in range(3)])
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = lambda a: ctypes.c_void_p(a.data_ptr()) if a is not None else None
    rng = np.random.RandomState(9)
    for T, K in ((3, 8), (1, 4)):
        x = torch.from_numpy(rng.randn(T, H).astype(np.float16)).cuda()
        logits = torch.from_numpy(rng.randn(T, E).astype(np.float32)).cuda()
        res = torch.from_numpy(rng.randn(T, H).astype(np.float32)).cuda()  # residual is in out_dtype
        ref = t.moe(0, x, logits=logits, top_k=K, per_k=True, combine=True, residual=res,
                    out_dtype=torch.float32)
        idx = torch.empty(T, K, dtype=torch.int32, device="cuda")
        w = torch.empty(T, K, dtype=torch.float32, device="cuda")
        pk = torch.empty(T, K, H, dtype=torch.float32, device="cuda")
        out = torch.empty(T, H, dtype=torch.float32, device="cuda")
        rc = lib.kq_moe_decode_static(t.handle, 0, p(x), N.DT_F16, T, p(logits), p(idx), p(w), K, p(pk), p(out),
                                      N.DT_F32, p(res), stream)
        assert rc == 0
        torch.cuda.synchronize()
        assert torch.equal(idx, ref["idx"])
        assert rel_l2(pk.cpu().numpy(), ref["per_k"].cpu().numpy()) < RTOL_L2
        assert rel_l2(out.cpu().numpy(), ref["out"].cpu().numpy()) < RTOL_L2
        # and against the oracle
        y = layer.moe(x.float().cpu().numpy(), idx.cpu().numpy())
        want = O.combine(y, w.cpu().numpy(), res.float().cpu().numpy())
        assert rel_l2(out.cpu().numpy(), want) < RTOL_L2


def test_static_decode_rejects_oversize(gpu):
    from kandiga_b200 import _native as N
    from kandiga_b200.experts import ExpertTable
    lib = N.load()
    t = ExpertTable(1, 16, 2048, 512, 3, "f16")
    # 1024 tokens x 16 experts needs far more scratch than the static array holds
    rc = lib.kq_moe_decode_static(t.handle, 0, ctypes.c_void_p(1), N.DT_F16, 1024, None, ctypes.c_void_p(1), None,
                                  16, ctypes.c_void_p(1), None, N.DT_F16, None, None)
    assert rc == 7  # KQ_ERR_WORKSPACE, before any device work


def test_static_decode_status_reports_bad_expert(gpu):
    """An expert id outside the table, passed as input routing, latches
    KQ_DEV_BAD_EXPERT; kq_moe_decode_static_status reports it and clears it."""
    from kandiga_b200 import _native as N
    from kandiga_b200.experts import ExpertTable
    lib = N.load()
    E, H, I, K = 8, 2048, 512, 2
    layer = O.ExpertLayer.random(3, H, I, E, seed=32, sb_dtype="f16")
    t = ExpertTable(1, E, H, I, 3, "f16")
    t.load_mlx(0, *[(torch.from_numpy(layer.w[m].reshape(E, layer.w[m].shape[1], -1)).cuda(),
                     torch.from_numpy(layer.s[m].view(np.int16)).cuda(),
                     torch.from_numpy(layer.b[m].view(np.int16)).cuda()) for m in range(3)])
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    p = lambda a: ctypes.c_void_p(a.data_ptr())  # noqa: E731
    x = torch.randn(1, H, device="cuda").half()
    idx = torch.tensor([[1, 99]], dtype=torch.int32, device="cuda")
    w = torch.tensor([[0.5, 0.5]], dtype=torch.float32, device="cuda")
    out = torch.empty(1, H, dtype=torch.float32, device="cuda")
    st = ctypes.c_uint32(0)
    assert lib.kq_moe_decode_static(t.handle, 0, p(x), N.DT_F16, 1, None, p(idx), p(w), K, None, p(out),
                                    N.DT_F32, None, stream) == 0
    assert lib.kq_moe_decode_static_status(ctypes.byref(st), stream) == 0
    assert st.value & N.DEV_BAD_EXPERT
    assert lib.kq_moe_decode_static_status(ctypes.byref(st), stream) == 0 and st.value == 0  # cleared
    idx = torch.tensor([[1, 3]], dtype=torch.int32, device="cuda")
    assert lib.kq_moe_decode_static(t.handle, 0, p(x), N.DT_F16, 1, None, p(idx), p(w), K, None, p(out),
                                    N.DT_F32, None, stream) == 0
    assert lib.kq_moe_decode_static_status(ctypes.byref(st), stream) == 0 and st.value == 0
