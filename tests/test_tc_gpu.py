"""GPU check of the tcgen05 building block (kq_gemm_f16_tc) against a torch
fp32 matmul of the same fp16 operands."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K", [(128, 16, 64), (256, 32, 128), (128, 256, 512), (384, 48, 2048)])
def test_gemm_f16_tc_matches_torch(gpu, M, N, K):
    from kandiga_b200 import _native as N_
    lib = N_.load()
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    A = torch.randn(M, K, device="cuda", generator=g).half()
    B = torch.randn(N, K, device="cuda", generator=g).half()
    C = torch.empty(M, N, device="cuda", dtype=torch.float32)
    rc = lib.kq_gemm_f16_tc(ctypes.c_void_p(A.data_ptr()), ctypes.c_void_p(B.data_ptr()),
                            ctypes.c_void_p(C.data_ptr()), M, N, K,
                            ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0
    torch.cuda.synchronize()
    ref = A.float() @ B.float().T
    rel = (C - ref).norm() / ref.norm()
    assert rel < 1e-5, float(rel)


def test_gemm_f16_tc_rejects_bad_shapes(gpu):
    from kandiga_b200 import _native as N_
    lib = N_.load()
    assert lib.kq_gemm_f16_tc(ctypes.c_void_p(1), ctypes.c_void_p(1), ctypes.c_void_p(1), 100, 16, 64, None) == 1
    assert lib.kq_gemm_f16_tc(ctypes.c_void_p(1), ctypes.c_void_p(1), ctypes.c_void_p(1), 128, 24, 64, None) == 1
