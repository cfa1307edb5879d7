// kq_tq3.cu -- TQ3_1S (Walsh-Hadamard rotated 3-bit) dense GEMV on sm_100a.
//
// Format (kandiga/tq3/quantize.py:122-145, 390-461): a row-major weight
// [rows][cols] is cut into blocks of 32; block = fp16 d0, d1 (and m0, m1 in the
// 20-byte variant) then 12 bytes holding 32 3-bit Lloyd-Max indices (four
// little-endian 24-bit groups of 8).  Dequantized, half h of a block is
// r = C[idx] d_h + m_h and the weights are w = S . H(r) / sqrt(32)
// (kandiga/tq3/quantize.py:464-516).  H and S are orthonormal up to the
// 1/sqrt(32), so  w . x = r . WHT(x)  with WHT(x) = H(S . x) / sqrt(32), the
// identity the reference GEMV uses (kandiga/tq3/fused_kernel.py:289-341).
//
// The matrix stays in HBM as the reference's own byte stream (bit-exact with
// its files).  tq3_gemv_kernel: each CTA rotates x into shared memory once
// (warp-shuffle butterfly per block, padded stride so that a warp reading 32
// different blocks hits distinct banks), then one warp per row: lane l takes
// blocks l, l+32, ...; pairs of indices (6-bit fields) look up a 64-entry
// table of centroid pairs, so a pair of weights costs one bit-field extract,
// one shared load and two FMAs.  The table is held in 16 interleaved copies,
// copy c in bank pair c, and lane l reads copy l % 16: a half-warp's 8-byte
// lookups (one shared-memory wavefront) never conflict, whatever the indices.
#include <algorithm>
#include <cstdio>
#include <cstring>

#include "kq_internal.h"
#include "kq_common.cuh"

namespace kq {

constexpr int TQ3_THREADS = 256;
constexpr int TQ3_XSTRIDE = 36;  // floats per rotated 32-block in shared memory (16-byte aligned, bank-staggered)
constexpr int TQ3_LUT_COPIES = 16;  // centroid-pair table copies: one per lane of a half-warp

// kandiga/tq3/quantize.py:29-47 (centroids of the 3-bit Lloyd-Max quantizer; block sign pattern)
__constant__ float tq3_centroids[8] = {-1.996684f, -1.291398f, -0.740341f, -0.247508f,
                                       0.230106f,  0.725222f,  1.277503f,  1.988943f};
__constant__ float tq3_signs[32] = {+1, -1, +1, -1, +1, +1, -1, +1, -1, -1, +1, -1, +1, +1, -1, +1,
                                    -1, -1, +1, -1, +1, -1, -1, +1, -1, +1, +1, -1, +1, -1, -1, +1};

template <int BB, int TT>
__global__ void __launch_bounds__(TQ3_THREADS) tq3_gemv_kernel(const uint8_t* __restrict__ blocks, int rows,
                                                                int cols, const void* __restrict__ x, int x_dtype,
                                                                int T, const float* __restrict__ bias, void* y,
                                                                int y_dtype) {
    extern __shared__ float4 tq3_sm[];
    const int nb = cols / 32;
    float* xr = reinterpret_cast<float*>(tq3_sm);        // [TT][nb][TQ3_XSTRIDE]
    float* hs = xr + (size_t)TT * nb * TQ3_XSTRIDE;       // [TT][2 nb] half-block sums
    float2* lut = reinterpret_cast<float2*>(hs + (size_t)TT * 2 * nb);  // [64][16]: (C[lo], C[hi]) per copy
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int i = tid; i < 64 * TQ3_LUT_COPIES; i += TQ3_THREADS) {
        const int e = i / TQ3_LUT_COPIES;
        lut[i] = make_float2(tq3_centroids[e & 7], tq3_centroids[e >> 3]);
    }
    const float2* lutl = lut + (lane % TQ3_LUT_COPIES);  // this lane's copy: entry e at lutl[e * 16]
    const float inv = sqrtf(32.f);
    // rotate x: warp per (token, block) of the T real tokens, lane = element;
    // XB blocks' loads in flight per warp (rows of slots t >= T are never stored)
    constexpr int NWARP = TQ3_THREADS / 32, XB = 16;
    const int jobs = min(T, TT) * nb;
    for (int j0 = warp; j0 < jobs; j0 += XB * NWARP) {
        float v[XB];
#pragma unroll
        for (int u = 0; u < XB; ++u) {
            const int job = j0 + u * NWARP;
            const int t = job / nb, b = job % nb;
            v[u] = job < jobs ? load_as_float(x, x_dtype, (size_t)t * cols + (size_t)b * 32 + lane) : 0.f;
        }
#pragma unroll
        for (int u = 0; u < XB; ++u) {
            const int job = j0 + u * NWARP;
            if (job >= jobs) break;
            const int t = job / nb, b = job % nb;
            float w = v[u] * tq3_signs[lane];
#pragma unroll
            for (int step = 1; step < 32; step <<= 1) {
                const float o = __shfl_xor_sync(0xffffffffu, w, step);
                w = (lane & step) ? o - w : w + o;
            }
            w = __fdiv_rn(w, inv);
            xr[((size_t)t * nb + b) * TQ3_XSTRIDE + lane] = w;
            float h = w;
#pragma unroll
            for (int o = 8; o > 0; o >>= 1) h += __shfl_xor_sync(0xffffffffu, h, o);
            if ((lane & 15) == 0) hs[(size_t)t * 2 * nb + 2 * b + (lane >> 4)] = h;
        }
    }
    __syncthreads();
    const size_t row_bytes = (size_t)nb * BB;
    for (int row = blockIdx.x * (TQ3_THREADS / 32) + warp; row < rows; row += gridDim.x * (TQ3_THREADS / 32)) {
        const uint8_t* rb = blocks + (size_t)row * row_bytes;
        float acc[TT];
#pragma unroll
        for (int t = 0; t < TT; ++t) acc[t] = 0.f;
        // RB blocks per lane are loaded before any is used: one memory round trip per RB blocks
        constexpr int RB = 4;
        for (int b0 = lane; b0 < nb; b0 += 32 * RB) {
            uint32_t wr[RB][BB / 4];
#pragma unroll
            for (int u = 0; u < RB; ++u) {
                const int b = b0 + 32 * u;
                const uint32_t* bw = reinterpret_cast<const uint32_t*>(rb + (size_t)(b < nb ? b : 0) * BB);
#pragma unroll
                for (int i = 0; i < BB / 4; ++i) wr[u][i] = b < nb ? __ldg(bw + i) : 0u;
            }
#pragma unroll
            for (int u = 0; u < RB; ++u) {
                const int b = b0 + 32 * u;
                if (b >= nb) break;
                const uint32_t* w = wr[u];
                const __half2 d01 = *reinterpret_cast<const __half2*>(&w[0]);
                const float d0 = __low2float(d01), d1 = __high2float(d01);
                float m0 = 0.f, m1 = 0.f;
                constexpr int CW = BB == 20 ? 2 : 1;  // first word of the codes
                if constexpr (BB == 20) {
                    const __half2 m01 = *reinterpret_cast<const __half2*>(&w[1]);
                    m0 = __low2float(m01);
                    m1 = __high2float(m01);
                }
                uint32_t grp[4];
                grp[0] = w[CW] & 0xFFFFFFu;
                grp[1] = (w[CW] >> 24) | ((w[CW + 1] & 0xFFFFu) << 8);
                grp[2] = (w[CW + 1] >> 16) | ((w[CW + 2] & 0xFFu) << 16);
                grp[3] = w[CW + 2] >> 8;
    #pragma unroll
                for (int t = 0; t < TT; ++t) {
                    const float* xb = xr + ((size_t)t * nb + b) * TQ3_XSTRIDE;
                    float a0 = 0.f, a1 = 0.f;
    #pragma unroll
                    for (int g = 0; g < 4; ++g) {
    #pragma unroll
                        for (int r = 0; r < 8; r += 4) {
                            const float4 xv = *reinterpret_cast<const float4*>(xb + g * 8 + r);
                            const float2 c0 = lutl[((grp[g] >> (3 * r)) & 63u) * TQ3_LUT_COPIES];
                            const float2 c1 = lutl[((grp[g] >> (3 * r + 6)) & 63u) * TQ3_LUT_COPIES];
                            float& a = g < 2 ? a0 : a1;
                            a = fmaf(c0.x, xv.x, a);
                            a = fmaf(c0.y, xv.y, a);
                            a = fmaf(c1.x, xv.z, a);
                            a = fmaf(c1.y, xv.w, a);
                        }
                    }
                    const float* hb = hs + (size_t)t * 2 * nb + 2 * b;
                    acc[t] += fmaf(d0, a0, fmaf(m0, hb[0], fmaf(d1, a1, m1 * hb[1])));
                }
            }
        }
#pragma unroll
        for (int t = 0; t < TT; ++t) {
            const float v = warp_sum(acc[t]);
            if (lane == 0 && t < T) store_from_float(y, y_dtype, (size_t)t * rows + row, bias ? v + bias[row] : v);
        }
    }
}

// w[row][32 b + i] = (S . H(r) / sqrt(32))[i]: reconstruction for checks
template <int BB>
__global__ void tq3_dequant_kernel(const uint8_t* __restrict__ blocks, long nblocks, float* __restrict__ w) {
    const long blk = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (blk >= nblocks) return;
    const uint8_t* bp = blocks + blk * BB;
    const float d = __half2float(*reinterpret_cast<const __half*>(bp + 2 * (lane >> 4)));
    const float m = BB == 20 ? __half2float(*reinterpret_cast<const __half*>(bp + 4 + 2 * (lane >> 4))) : 0.f;
    const uint8_t* q = bp + (BB == 20 ? 8 : 4) + 3 * (lane >> 3);
    const uint32_t word = (uint32_t)q[0] | ((uint32_t)q[1] << 8) | ((uint32_t)q[2] << 16);
    float v = fmaf(tq3_centroids[(word >> (3 * (lane & 7))) & 7u], d, m);
#pragma unroll
    for (int step = 1; step < 32; step <<= 1) {
        const float o = __shfl_xor_sync(0xffffffffu, v, step);
        v = (lane & step) ? o - v : v + o;
    }
    w[blk * 32 + lane] = __fdiv_rn(v * tq3_signs[lane], sqrtf(32.f));
}

template <int BB, int TT>
static cudaError_t launch_tq3(const kq_tq3_mat* m, const void* x, int x_dtype, int T, const float* bias, void* y,
                              int y_dtype, cudaStream_t s) {
    static int configured[64] = {0};
    const int nb = m->cols / 32;
    const size_t smem = ((size_t)TT * nb * TQ3_XSTRIDE + (size_t)TT * 2 * nb) * 4 + 64 * TQ3_LUT_COPIES * 8 + 16;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if ((size_t)configured[dev] < smem) {
        cudaError_t e =
            cudaFuncSetAttribute(tq3_gemv_kernel<BB, TT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        configured[dev] = (int)smem;
    }
    int nsm = 148;
    cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    const int rows_per_cta = TQ3_THREADS / 32;
    const int grid = std::min((m->rows + rows_per_cta - 1) / rows_per_cta, nsm * 4);
    tq3_gemv_kernel<BB, TT><<<grid, TQ3_THREADS, smem, s>>>(m->data, m->rows, m->cols, x, x_dtype, T, bias, y,
                                                             y_dtype);
    return cudaGetLastError();
}

// tokens per launch: every CTA keeps TT rotated inputs in shared memory
static int tq3_tokens_per_launch(int cols) {
    const size_t per_token = ((size_t)(cols / 32) * TQ3_XSTRIDE + (size_t)2 * (cols / 32)) * 4;
    if (per_token * 4 <= 96 * 1024) return 4;
    if (per_token * 2 <= 96 * 1024) return 2;
    return 1;
}

}  // namespace kq

using namespace kq;

extern "C" int kq_tq3_create(int rows, int cols, int block_bytes, const void* host_blocks, size_t nbytes,
                             kq_tq3_mat** out) {
    if (!out) return KQ_ERR_ARG;
    *out = nullptr;
    if (rows <= 0 || cols <= 0 || cols % 32 || (block_bytes != 16 && block_bytes != 20) || !host_blocks)
        return KQ_ERR_ARG;
    const size_t need = (size_t)rows * (cols / 32) * block_bytes;
    if (nbytes != need) return KQ_ERR_FORMAT;
    kq_tq3_mat* m = new (std::nothrow) kq_tq3_mat();
    if (!m) return KQ_ERR_ALLOC;
    m->rows = rows;
    m->cols = cols;
    m->block_bytes = block_bytes;
    m->bytes = need;
    if (cudaMalloc(&m->data, need) != cudaSuccess) {
        delete m;
        return KQ_ERR_ALLOC;
    }
    if (cudaMemcpy(m->data, host_blocks, need, cudaMemcpyHostToDevice) != cudaSuccess) {
        cudaFree(m->data);
        delete m;
        return KQ_ERR_CUDA;
    }
    *out = m;
    return KQ_OK;
}

extern "C" int kq_tq3_destroy(kq_tq3_mat* m) {
    if (!m) return KQ_OK;
    cudaFree(m->data);
    delete m;
    return KQ_OK;
}

extern "C" size_t kq_tq3_bytes(const kq_tq3_mat* m) { return m ? m->bytes : 0; }

extern "C" int kq_tq3_gemv(const kq_tq3_mat* m, const void* x, int x_dtype, int T, const float* bias, void* y,
                           int y_dtype, void* stream) {
    if (!m || T < 0) return KQ_ERR_ARG;
    if (x_dtype != KQ_DT_F16 && x_dtype != KQ_DT_BF16 && x_dtype != KQ_DT_F32) return KQ_ERR_ARG;
    if (y_dtype != KQ_DT_F16 && y_dtype != KQ_DT_BF16 && y_dtype != KQ_DT_F32) return KQ_ERR_ARG;
    if (T == 0) return KQ_OK;
    if (!x || !y) return KQ_ERR_ARG;
    // one rotated input row must fit shared memory
    if ((size_t)(m->cols / 32) * TQ3_XSTRIDE * 4 + (size_t)(m->cols / 32) * 8 > 200 * 1024) return KQ_ERR_UNSUPPORTED;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int tt = tq3_tokens_per_launch(m->cols);
    const size_t xe = x_dtype == KQ_DT_F32 ? 4 : 2, ye = y_dtype == KQ_DT_F32 ? 4 : 2;
    for (int t0 = 0; t0 < T; t0 += tt) {
        const int n = std::min(tt, T - t0);
        const void* xt = static_cast<const uint8_t*>(x) + (size_t)t0 * m->cols * xe;
        void* yt = static_cast<uint8_t*>(y) + (size_t)t0 * m->rows * ye;
        cudaError_t e;
        if (m->block_bytes == 20)
            e = n > 2 ? launch_tq3<20, 4>(m, xt, x_dtype, n, bias, yt, y_dtype, s)
                      : (n == 2 ? launch_tq3<20, 2>(m, xt, x_dtype, n, bias, yt, y_dtype, s)
                                : launch_tq3<20, 1>(m, xt, x_dtype, n, bias, yt, y_dtype, s));
        else
            e = n > 2 ? launch_tq3<16, 4>(m, xt, x_dtype, n, bias, yt, y_dtype, s)
                      : (n == 2 ? launch_tq3<16, 2>(m, xt, x_dtype, n, bias, yt, y_dtype, s)
                                : launch_tq3<16, 1>(m, xt, x_dtype, n, bias, yt, y_dtype, s));
        if (e != cudaSuccess) return KQ_ERR_CUDA;
    }
    return KQ_OK;
}

extern "C" int kq_tq3_dequant(const kq_tq3_mat* m, float* w, void* stream) {
    if (!m || !w) return KQ_ERR_ARG;
    const long nblocks = (long)m->rows * (m->cols / 32);
    const int threads = 256;
    const long grid = (nblocks * 32 + threads - 1) / threads;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (m->block_bytes == 20)
        tq3_dequant_kernel<20><<<(unsigned)grid, threads, 0, s>>>(m->data, nblocks, w);
    else
        tq3_dequant_kernel<16><<<(unsigned)grid, threads, 0, s>>>(m->data, nblocks, w);
    return cudaGetLastError() == cudaSuccess ? KQ_OK : KQ_ERR_CUDA;
}
