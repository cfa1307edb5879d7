// kq_gemm_tc.cu -- dense fp16 GEMM C = A * B^T on tcgen05 (TMEM accumulator).
//
// The building block of the prefill expert GEMM, exposed on its own so the
// operand layout, descriptors, tensor-memory allocation and MMA completion path
// can be checked against a plain reference.  One CTA (4 warps) per 128-row
// block: threads stage one 64-wide K-chunk of A (128 rows) and B (N rows) into
// 128-byte-swizzled shared memory, one thread issues four K=16 MMAs into a
// TMEM accumulator of 128 lanes x N fp32 columns and commits them to an
// mbarrier (bounded wait), and after the last chunk each warp reads its 32
// lanes back with tcgen05.ld.
#include "kq_internal.h"
#include "kq_tc.cuh"

namespace kq {

constexpr int GEMM_TC_THREADS = 128;

__global__ void __launch_bounds__(GEMM_TC_THREADS) gemm_f16_tc_kernel(const __half* __restrict__ A,
                                                                      const __half* __restrict__ B,
                                                                      float* __restrict__ C, int M, int N,
                                                                      int K, uint32_t ncols,
                                                                      uint32_t* status) {
    extern __shared__ uint8_t smem_raw[];
    // 1024-byte aligned in the shared window; an offset from smem_raw keeps the
    // shared address space, so accesses through it compile to shared-memory ops
    uint8_t* smem = smem_raw + ((1024u - ((uint32_t)__cvta_generic_to_shared(smem_raw) & 1023u)) & 1023u);
    uint8_t* sA = smem;                 // 128 x 128 B
    uint8_t* sB = smem + 128 * 128;     // N x 128 B
    __shared__ uint64_t bar;
    __shared__ uint32_t tmem_slot;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int m0 = blockIdx.x * 128;

    if (warp == 0) {
        tc::tmem_alloc(&tmem_slot, ncols);
        tc::tmem_relinquish();
    }
    if (tid == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = tmem_slot;
    const uint32_t idesc = tc::idesc_f16(128, N, false);

    uint32_t phase = 0;
    for (int kc = 0; kc < K / 64; ++kc) {
        // stage A rows (one per thread) and B rows into the swizzled layout
        {
            const uint4* src = reinterpret_cast<const uint4*>(A + (size_t)(m0 + tid) * K + kc * 64);
#pragma unroll
            for (int c = 0; c < 8; ++c)
                *reinterpret_cast<uint4*>(sA + tc::sw128_offset(tid, c * 8)) = src[c];
        }
        for (int r = tid; r < N; r += GEMM_TC_THREADS) {
            const uint4* src = reinterpret_cast<const uint4*>(B + (size_t)r * K + kc * 64);
#pragma unroll
            for (int c = 0; c < 8; ++c)
                *reinterpret_cast<uint4*>(sB + tc::sw128_offset(r, c * 8)) = src[c];
        }
        fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
        __syncthreads();
        if (tid == 0) {
            tc::fence_after_sync();
            const uint64_t da = tc::smem_desc_sw128(sA), db = tc::smem_desc_sw128(sB);
#pragma unroll
            for (int s = 0; s < 4; ++s)
                tc::mma_f16_ss(tmem, tc::desc_advance(da, 32 * s), tc::desc_advance(db, 32 * s), idesc,
                               kc > 0 || s > 0);
            tc::mma_commit(&bar);
        }
        mbar_wait(&bar, phase, status);  // the MMAs have read shared memory; it may be refilled
        phase ^= 1u;
    }
    tc::fence_after_sync();
    // epilogue: warp w owns TMEM lanes 32w..32w+31 (rows m0 + 32w + lane)
    const int row = m0 + warp * 32 + lane;
    for (int col = 0; col < N; col += 16) {
        uint32_t r[16];
        tc::tmem_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)col, r);
        tc::tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) C[(size_t)row * N + col + j] = __uint_as_float(r[j]);
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) tc::tmem_dealloc(tmem, ncols);
}

}  // namespace kq

using namespace kq;

extern "C" int kq_gemm_f16_tc(const void* A, const void* B, float* C, int M, int N, int K, void* stream) {
    if (!A || !B || !C) return KQ_ERR_ARG;
    if (M <= 0 || M % 128 || N < 16 || N > 256 || N % 16 || K <= 0 || K % 64) return KQ_ERR_ARG;
    uint32_t ncols = 32;
    while (ncols < (uint32_t)N) ncols <<= 1;
    const size_t smem = 1024 + 128 * 128 + (size_t)N * 128;
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return KQ_ERR_CUDA;
    if ((size_t)configured[dev] < smem) {
        if (cudaFuncSetAttribute(gemm_f16_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
            cudaSuccess)
            return KQ_ERR_CUDA;
        configured[dev] = (int)smem;
    }
    gemm_f16_tc_kernel<<<M / 128, GEMM_TC_THREADS, smem, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __half*>(A), static_cast<const __half*>(B), C, M, N, K, ncols, nullptr);
    return cudaGetLastError() == cudaSuccess ? KQ_OK : KQ_ERR_CUDA;
}
