// kq_turbo.cu -- TurboQuant KV cache (PolarQuant 3-bit + 1-bit QJL) on sm_100a.
//
// The reference (kandiga/kv_compress.py:22-168) keeps int8 codes, int8 signs
// and fp32 scales/zeros in MLX arrays, grows them with a concatenate per
// append, and dequantizes the whole cache for every attention call.  Here:
//
//   tq_append_kernel   one pass per new vector: x R (D x D fp32, R and P staged
//                      in shared memory, 8 vectors per warp share every R/P
//                      load), per-vector min/max, 3-bit codes, residual,
//                      residual P, signs; packed as one nibble per element
//                      (code << 1 | sign) into a preallocated cache.  Used for
//                      storage width 64 and for small appends.
//   tq_append_tc_kernel the same for bulk appends at width 128, the two products
//                      on the tensor cores (see below).
//   tq_dequant_kernel  the reference's reconstruction ((q s + z) +- s/4) R^T
//                      -> fp16, for the `keys` / `values` accessors.
//   tq_attend_kernel   single-query attention straight on the codes, split
//                      over the sequence (flash-decoding): with q' = q R and
//                      v = c + sigma/2 (half the stored nibble),
//                      q.K_t = s_t (q'.v_t) + (z_t - s_t/4) sum(q'),
//                      values accumulated in the rotated domain the same way;
//   tq_combine_kernel  merges the per-chunk softmax partials and un-rotates
//                      once per query head: out = (sum p V~) R^T.
//
// Any head_dim up to 128 is stored at a width D of 64 or 128: R is extended by
// the identity and P by zeros on the added dimensions, inputs are read and
// outputs written at the caller's stride Dr with zeros in the added
// dimensions, and each vector's min / max run over its Dr dimensions only, so
// the Dr real codes, scales, zeros, signs, scores and outputs are those of the
// unpadded arithmetic (an added dimension of x R is 0 and meets a zero row of
// P, and q R is 0 there, so it enters no score or output).
//
// Arithmetic that the reference fixes (kandiga/kv_compress.py:75-88) is done
// with explicitly rounded operations (no contraction): scale = (max - min) / 7,
// q = clip(round_half_even((r - min) / scale), 0, 7), dequant = q * scale + min,
// residual = r - dequant.  The two D x D products use fp32 FMA chains, whose
// summation order differs from a BLAS sgemm: codes can differ from a CPU
// restatement only where a value sits on a rounding boundary.
#include <cstdio>
#include <cstring>

#include "kq_internal.h"
#include "kq_common.cuh"
#include "kq_tc.cuh"

namespace kq {

constexpr int TQ_VPW = 8;    // vectors per warp per pass (append / dequant)
constexpr int TQ_WARPS = 8;  // warps per CTA (append / dequant)

struct TqVecParams {
    const void* src[2];  // append: keys, values [B][H][T][D]
    int dtype;
    int B, H, T, cap, len;  // append: T new tokens written at len; dequant: T = len
    int Dr;                 // caller's head_dim (<= D; input / output stride)
    const float* R;
    const float* RT;
    const float* P;
    uint8_t* packed[2];
    float* scale[2];
    float* zero[2];
    __half* out;  // dequant output [B][H][len][D]
    int which;    // dequant: 0 = K, 1 = V
    uint32_t* status;
    const uint8_t* tc_ops;  // tensor-core append: the B operand images
};

__device__ __forceinline__ float warp_min(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fminf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// acc[v][c] = sum_d xs[v][d] * M[d][lane * CPL + c], M row-major D x D in shared memory
template <int D, int NV>
__device__ __forceinline__ void warp_matvec(const float* M, const float* xs, int lane, float (&acc)[NV][D / 32]) {
    constexpr int CPL = D / 32;
#pragma unroll
    for (int v = 0; v < NV; ++v)
#pragma unroll
        for (int c = 0; c < CPL; ++c) acc[v][c] = 0.f;
#pragma unroll 4
    for (int d = 0; d < D; ++d) {
        float r[CPL];
        if constexpr (CPL == 4) {
            const float4 t = *reinterpret_cast<const float4*>(M + d * D + lane * 4);
            r[0] = t.x;
            r[1] = t.y;
            r[2] = t.z;
            r[3] = t.w;
        } else {
            const float2 t = *reinterpret_cast<const float2*>(M + d * D + lane * 2);
            r[0] = t.x;
            r[1] = t.y;
        }
#pragma unroll
        for (int v = 0; v < NV; ++v) {
            const float xv = xs[v * D + d];
#pragma unroll
            for (int c = 0; c < CPL; ++c) acc[v][c] = fmaf(xv, r[c], acc[v][c]);
        }
    }
}

template <int D>
__global__ void __launch_bounds__(TQ_WARPS * 32, 1) tq_append_kernel(TqVecParams p) {
    constexpr int CPL = D / 32;
    extern __shared__ float4 tq_sm[];
    float* sR = reinterpret_cast<float*>(tq_sm);
    float* sP = sR + D * D;
    float* xs = sP + D * D + (threadIdx.x >> 5) * TQ_VPW * D;
#pragma unroll 8
    for (int i = threadIdx.x; i < D * D / 4; i += blockDim.x) {  // loads of several rows in flight
        reinterpret_cast<float4*>(sR)[i] = reinterpret_cast<const float4*>(p.R)[i];
        reinterpret_cast<float4*>(sP)[i] = reinterpret_cast<const float4*>(p.P)[i];
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long per = (long)p.B * p.H * p.T;
    const long nvec = 2 * per;
    const long stride = (long)gridDim.x * TQ_WARPS * TQ_VPW;
    for (long v0 = ((long)blockIdx.x * TQ_WARPS + warp) * TQ_VPW; v0 < nvec; v0 += stride) {
#pragma unroll
        for (int v = 0; v < TQ_VPW; ++v) {
            const long vi = v0 + v;
            if (vi < nvec) {
                const int which = vi >= per ? 1 : 0;
                const size_t base = (size_t)(vi - which * per) * p.Dr;
                const void* src = which ? p.src[1] : p.src[0];
                for (int d = lane; d < D; d += 32) xs[v * D + d] = d < p.Dr ? load_as_float(src, p.dtype, base + d) : 0.f;
            } else {
                for (int d = lane; d < D; d += 32) xs[v * D + d] = 0.f;
            }
        }
        __syncwarp();
        float acc[TQ_VPW][CPL];
        warp_matvec<D, TQ_VPW>(sR, xs, lane, acc);  // rotated = x R
        __syncwarp();
        float vscale[TQ_VPW], vmin[TQ_VPW];
        uint32_t codes[TQ_VPW];
#pragma unroll
        for (int v = 0; v < TQ_VPW; ++v) {
            float mn = INFINITY, mx = -INFINITY;  // over the head_dim real dimensions
#pragma unroll
            for (int c = 0; c < CPL; ++c) {
                if (lane * CPL + c < p.Dr) {
                    mn = fminf(mn, acc[v][c]);
                    mx = fmaxf(mx, acc[v][c]);
                }
            }
            mn = warp_min(mn);
            mx = warp_max(mx);
            float scale = __fdiv_rn(__fsub_rn(mx, mn), 7.f);
            if (scale == 0.f) scale = 1.f;
            uint32_t cw = 0;
#pragma unroll
            for (int c = 0; c < CPL; ++c) {
                float q = rintf(__fdiv_rn(__fsub_rn(acc[v][c], mn), scale));
                q = fminf(fmaxf(q, 0.f), 7.f);
                const float deq = __fadd_rn(__fmul_rn(q, scale), mn);
                xs[v * D + lane * CPL + c] = __fsub_rn(acc[v][c], deq);  // residual
                cw |= (uint32_t)q << (4 * c + 1);
            }
            codes[v] = cw;
            vscale[v] = scale;
            vmin[v] = mn;
        }
        __syncwarp();
        warp_matvec<D, TQ_VPW>(sP, xs, lane, acc);  // residual P
#pragma unroll
        for (int v = 0; v < TQ_VPW; ++v) {
            const long vi = v0 + v;
            if (vi >= nvec) break;
            const int which = vi >= per ? 1 : 0;
            const long r = vi - which * per;  // (b H + h) T + t
            const size_t slot = (size_t)(r / p.T) * p.cap + p.len + (size_t)(r % p.T);
            uint32_t cw = codes[v];
#pragma unroll
            for (int c = 0; c < CPL; ++c)
                if (acc[v][c] > 0.f) cw |= 1u << (4 * c);
            uint8_t* dst = (which ? p.packed[1] : p.packed[0]) + slot * (D / 2) + lane * (CPL / 2);
            if constexpr (CPL == 4)
                *reinterpret_cast<uint16_t*>(dst) = (uint16_t)cw;
            else
                *dst = (uint8_t)cw;
            if (lane == 0) {
                (which ? p.scale[1] : p.scale[0])[slot] = vscale[v];
                (which ? p.zero[1] : p.zero[0])[slot] = vmin[v];
            }
        }
        __syncwarp();
    }
}

// ---- append on the tensor cores (storage width 128) -----------------------------------------
//
// One CTA of 128 threads per tile of 128 vectors (persistent over tiles).  The
// two D x D products run as tcgen05 MMAs in fp16 with two limbs per operand:
// v = v_hi + v_lo (v_hi = fp16(v), v_lo = fp16(v - v_hi)), likewise M, and
// v M ~ v_hi M_hi + v_hi M_lo + v_lo M_hi (the dropped v_lo M_lo is ~2^-22 of
// the product), accumulated in fp32 in tensor memory: about 22 bits, so a code
// or a sign differs from an fp32 evaluation only where a value sits on a
// rounding boundary.  R^T and P^T (B operands: B[n][k] = M[k][n]) sit in shared
// memory as fp16 limb pairs for the whole launch; the A stage holds the tile's
// inputs, then its residuals.  Thread i owns vector i of the tile (TMEM lane i)
// and does the quantisation with the same explicitly rounded operations as
// tq_append_kernel.
constexpr int TQTC_THREADS = 128;
constexpr int TQTC_D = 128;
constexpr int TQTC_OP = TQTC_D * TQTC_D * 2;  // one 128 x 128 fp16 operand (two 64-wide K blocks)

__host__ __device__ constexpr size_t tq_tc_smem() { return 1024 + (size_t)6 * TQTC_OP; }

// element (r, k) of a 128 x 128 fp16 operand stored as two swizzled [128 x 64] K blocks
__device__ __forceinline__ uint32_t tq_op_offset(int r, int k) {
    return (uint32_t)((k >> 6) * (TQTC_D * 128)) + tc::sw128_offset(r, k & 63);
}


// 8 consecutive values (k0 % 8 == 0) of row r as fp16 hi / lo limbs: one 16-byte store each
__device__ __forceinline__ void split_store8(uint8_t* hi, uint8_t* lo, int r, int k0, const float* v) {
    uint32_t h[4], l[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const __half2 hh = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
        const float2 hf = __half22float2(hh);
        const __half2 ll = __floats2half2_rn(v[2 * i] - hf.x, v[2 * i + 1] - hf.y);
        h[i] = *reinterpret_cast<const uint32_t*>(&hh);
        l[i] = *reinterpret_cast<const uint32_t*>(&ll);
    }
    *reinterpret_cast<uint4*>(hi + tq_op_offset(r, k0)) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4*>(lo + tq_op_offset(r, k0)) = make_uint4(l[0], l[1], l[2], l[3]);
}

// The four B operand images (R^T hi, R^T lo, P^T hi, P^T lo; each 128 x 128 fp16
// in the swizzled two-block layout), built once per cache.
__global__ void tq_tc_ops_kernel(const float* __restrict__ RT, const float* __restrict__ P, uint8_t* ops) {
    const int n = blockIdx.x, k0 = threadIdx.x * 8;  // 128 blocks x 16 threads
    float r[8], q[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        r[i] = RT[(size_t)n * TQTC_D + k0 + i];       // R^T[n][k] = R[k][n]
        q[i] = P[(size_t)(k0 + i) * TQTC_D + n];     // P^T[n][k] = P[k][n]
    }
    split_store8(ops, ops + TQTC_OP, n, k0, r);
    split_store8(ops + 2 * TQTC_OP, ops + 3 * TQTC_OP, n, k0, q);
}

// D[lane][n] (+)= sum_k A[lane][k] B[n][k] with the three limb products, one thread issuing
__device__ __forceinline__ void limb_mma(uint32_t d_tmem, const uint8_t* a_hi, const uint8_t* a_lo,
                                         const uint8_t* b_hi, const uint8_t* b_lo) {
    constexpr uint32_t idesc = tc::idesc_f16(128, TQTC_D, false);
#pragma unroll
    for (int kc = 0; kc < 2; ++kc) {
        const uint32_t off = (uint32_t)kc * (TQTC_D * 128);
        const uint64_t ah = tc::smem_desc_sw128(a_hi + off), al = tc::smem_desc_sw128(a_lo + off);
        const uint64_t bh = tc::smem_desc_sw128(b_hi + off), bl = tc::smem_desc_sw128(b_lo + off);
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            const uint32_t o = 32u * s;
            tc::mma_f16_ss(d_tmem, tc::desc_advance(ah, o), tc::desc_advance(bh, o), idesc, kc > 0 || s > 0);
            tc::mma_f16_ss(d_tmem, tc::desc_advance(ah, o), tc::desc_advance(bl, o), idesc, true);
            tc::mma_f16_ss(d_tmem, tc::desc_advance(al, o), tc::desc_advance(bh, o), idesc, true);
        }
    }
}

__global__ void __launch_bounds__(TQTC_THREADS, 1) tq_append_tc_kernel(TqVecParams p) {
    extern __shared__ uint8_t tqtc_raw[];
    uint8_t* sm = tqtc_raw + ((1024u - ((uint32_t)__cvta_generic_to_shared(tqtc_raw) & 1023u)) & 1023u);
    uint8_t* sRh = sm;  // R^T limbs
    uint8_t* sRl = sm + TQTC_OP;
    uint8_t* sPh = sm + 2 * TQTC_OP;  // P^T limbs
    uint8_t* sPl = sm + 3 * TQTC_OP;
    uint8_t* sAh = sm + 4 * TQTC_OP;  // inputs, then residuals
    uint8_t* sAl = sm + 5 * TQTC_OP;
    __shared__ uint64_t bar;
    __shared__ uint32_t tmem_slot;
    const int tid = threadIdx.x, warp = tid >> 5;
    if (warp == 0) {
        tc::tmem_alloc(&tmem_slot, 256);
        tc::tmem_relinquish();
    }
    if (tid == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    __syncthreads();  // the barrier is initialised
    // the B operand images, once per launch: four 32 KB bulk copies on one mbarrier
    if (tid == 0) {
        mbar_expect_tx(&bar, 4 * TQTC_OP);
        const uint64_t pol = policy_evict_first();
        for (int i = 0; i < 4; ++i) bulk_g2s(sm + (size_t)i * TQTC_OP, p.tc_ops + (size_t)i * TQTC_OP, TQTC_OP, &bar, pol);
    }
    mbar_wait(&bar, 0, p.status);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = tmem_slot;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    const long per = (long)p.B * p.H * p.T;
    const long nvec = 2 * per;
    const long ntiles = (nvec + 127) / 128;
    uint32_t phase = 1;  // phase 0 was the operand copy
    for (long tile = blockIdx.x; tile < ntiles; tile += gridDim.x) {
        const long vi = tile * 128 + tid;
        const bool live = vi < nvec;
        const int which = live && vi >= per ? 1 : 0;
        const long r = vi - which * per;  // (b H + h) T + t
        // stage this thread's vector (zeros past head_dim and past the last vector),
        // 8 values per step; 16-byte loads when the row allows them
        {
            const void* src = which ? p.src[1] : p.src[0];
            const size_t base = live ? (size_t)r * p.Dr : 0;
            const int esz = p.dtype == KQ_DT_F32 ? 4 : 2;
            const bool vec = live && p.Dr == TQTC_D && p.dtype != KQ_DT_F32 &&
                             ((reinterpret_cast<uintptr_t>(src) + base * esz) & 15) == 0;
#pragma unroll 2
            for (int k0 = 0; k0 < TQTC_D; k0 += 8) {
                float v[8];
                if (vec) {
                    const uint4 u = *reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(src) + (base + k0) * 2);
                    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float2 f = p.dtype == KQ_DT_F16
                                             ? __half22float2(*reinterpret_cast<const __half2*>(&w[i]))
                                             : __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
                        v[2 * i] = f.x;
                        v[2 * i + 1] = f.y;
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        v[i] = live && k0 + i < p.Dr ? load_as_float(src, p.dtype, base + k0 + i) : 0.f;
                }
                split_store8(sAh, sAl, tid, k0, v);
            }
        }
        fence_proxy_async_smem();
        __syncthreads();
        if (tid == 0) {
            tc::fence_after_sync();
            limb_mma(tmem, sAh, sAl, sRh, sRl);  // rotated = x R  -> columns [0, 128)
            tc::mma_commit(&bar);
        }
        mbar_wait(&bar, phase, p.status);
        phase ^= 1u;
        tc::fence_after_sync();
        // min / max over the head_dim real dimensions
        float mn = INFINITY, mx = -INFINITY;
        for (int c0 = 0; c0 < TQTC_D; c0 += 16) {
            uint32_t a[16];
            tc::tmem_ld16(tmem + lane_base + (uint32_t)c0, a);
            tc::tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (c0 + j < p.Dr) {
                    mn = fminf(mn, __uint_as_float(a[j]));
                    mx = fmaxf(mx, __uint_as_float(a[j]));
                }
        }
        float scale = __fdiv_rn(__fsub_rn(mx, mn), 7.f);
        if (scale == 0.f) scale = 1.f;
        // codes and residuals (the residual overwrites the staged input)
        uint32_t cw[TQTC_D / 8];
#pragma unroll
        for (int c0 = 0; c0 < TQTC_D; c0 += 16) {
            uint32_t a[16];
            tc::tmem_ld16(tmem + lane_base + (uint32_t)c0, a);
            tc::tmem_ld_wait();
            uint32_t w0 = 0, w1 = 0;
            float res[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const float v = __uint_as_float(a[j]);
                float q = rintf(__fdiv_rn(__fsub_rn(v, mn), scale));
                q = fminf(fmaxf(q, 0.f), 7.f);
                const float deq = __fadd_rn(__fmul_rn(q, scale), mn);
                res[j] = __fsub_rn(v, deq);
                if (j < 8) w0 |= (uint32_t)q << (4 * j + 1);
                else w1 |= (uint32_t)q << (4 * (j - 8) + 1);
            }
            split_store8(sAh, sAl, tid, c0, res);
            split_store8(sAh, sAl, tid, c0 + 8, res + 8);
            cw[c0 / 8] = w0;
            cw[c0 / 8 + 1] = w1;
        }
        tc::fence_before_sync();
        fence_proxy_async_smem();
        __syncthreads();
        if (tid == 0) {
            tc::fence_after_sync();
            limb_mma(tmem + 128, sAh, sAl, sPh, sPl);  // residual P -> columns [128, 256)
            tc::mma_commit(&bar);
        }
        mbar_wait(&bar, phase, p.status);
        phase ^= 1u;
        tc::fence_after_sync();
#pragma unroll
        for (int c0 = 0; c0 < TQTC_D; c0 += 16) {
            uint32_t a[16];
            tc::tmem_ld16(tmem + lane_base + 128u + (uint32_t)c0, a);
            tc::tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 16; ++j)
                if (__uint_as_float(a[j]) > 0.f) cw[(c0 + j) / 8] |= 1u << (4 * ((c0 + j) & 7));
        }
        if (live) {
            const size_t slot = (size_t)(r / p.T) * p.cap + p.len + (size_t)(r % p.T);
            uint4* dst = reinterpret_cast<uint4*>((which ? p.packed[1] : p.packed[0]) + slot * (TQTC_D / 2));
#pragma unroll
            for (int i = 0; i < TQTC_D / 32; ++i) dst[i] = make_uint4(cw[4 * i], cw[4 * i + 1], cw[4 * i + 2], cw[4 * i + 3]);
            (which ? p.scale[1] : p.scale[0])[slot] = scale;
            (which ? p.zero[1] : p.zero[0])[slot] = mn;
        }
        tc::fence_before_sync();
        __syncthreads();  // the A stage and the accumulators are free for the next tile
        tc::fence_after_sync();
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 0) tc::tmem_dealloc(tmem, 256);
}

template <int D>
__global__ void __launch_bounds__(TQ_WARPS * 32, 1) tq_dequant_kernel(TqVecParams p) {
    constexpr int CPL = D / 32;
    extern __shared__ float4 tq_sm[];
    float* sRT = reinterpret_cast<float*>(tq_sm);  // R^T
    float* xs = sRT + D * D + (threadIdx.x >> 5) * TQ_VPW * D;
#pragma unroll 8
    for (int i = threadIdx.x; i < D * D / 4; i += blockDim.x)
        reinterpret_cast<float4*>(sRT)[i] = reinterpret_cast<const float4*>(p.RT)[i];
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long nvec = (long)p.B * p.H * p.len;
    const long stride = (long)gridDim.x * TQ_WARPS * TQ_VPW;
    const uint8_t* packed = p.which ? p.packed[1] : p.packed[0];
    const float* scale = p.which ? p.scale[1] : p.scale[0];
    const float* zero = p.which ? p.zero[1] : p.zero[0];
    for (long v0 = ((long)blockIdx.x * TQ_WARPS + warp) * TQ_VPW; v0 < nvec; v0 += stride) {
#pragma unroll
        for (int v = 0; v < TQ_VPW; ++v) {
            const long vi = v0 + v;
            if (vi < nvec) {
                const size_t slot = (size_t)(vi / p.len) * p.cap + (size_t)(vi % p.len);
                const uint8_t* src = packed + slot * (D / 2) + lane * (CPL / 2);
                const uint32_t cw = CPL == 4 ? (uint32_t)*reinterpret_cast<const uint16_t*>(src) : (uint32_t)*src;
                const float s = scale[slot], z = zero[slot];
                const float corr = __fdiv_rn(s, 4.f);
#pragma unroll
                for (int c = 0; c < CPL; ++c) {
                    const uint32_t nib = (cw >> (4 * c)) & 15u;
                    const float deq = __fadd_rn(__fmul_rn((float)(nib >> 1), s), z);
                    xs[v * D + lane * CPL + c] = __fadd_rn(deq, (nib & 1u) ? corr : -corr);
                }
            } else {
#pragma unroll
                for (int c = 0; c < CPL; ++c) xs[v * D + lane * CPL + c] = 0.f;
            }
        }
        __syncwarp();
        float acc[TQ_VPW][CPL];
        warp_matvec<D, TQ_VPW>(sRT, xs, lane, acc);  // corrected R^T
#pragma unroll
        for (int v = 0; v < TQ_VPW; ++v) {
            const long vi = v0 + v;
            if (vi >= nvec) break;
            __half* o = p.out + (size_t)vi * p.Dr;
#pragma unroll
            for (int c = 0; c < CPL; ++c)
                if (lane * CPL + c < p.Dr) o[lane * CPL + c] = __float2half_rn(acc[v][c]);
        }
        __syncwarp();
    }
}

__global__ void tq_export_kernel(const uint8_t* __restrict__ packed, const float* __restrict__ scale,
                                 const float* __restrict__ zero, int D, int Dr, int BH, int cap, int len,
                                 int8_t* codes, int8_t* signs, float* scales, float* zeros) {
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;  // element index [BH][len][Dr]
    const long n = (long)BH * len * Dr;
    if (i >= n) return;
    const long vec = i / Dr;
    const int d = (int)(i % Dr);
    const size_t slot = (size_t)(vec / len) * cap + (size_t)(vec % len);
    const uint32_t nib = (packed[slot * (D / 2) + d / 2] >> (4 * (d & 1))) & 15u;
    if (codes) codes[i] = (int8_t)(nib >> 1);
    if (signs) signs[i] = (int8_t)(nib & 1u);
    if (d == 0) {
        if (scales) scales[vec] = scale[slot];
        if (zeros) zeros[vec] = zero[slot];
    }
}

// ---- attention ---------------------------------------------------------------------------------

// Nibble k of w (2c + sigma) as the float 1 + (c + sigma/2)/8: the four bits
// placed in the mantissa under the exponent of 1.0 (no int-to-float convert).
__device__ __forceinline__ float nib_1p(uint32_t w, int k) {
    const uint32_t b = k <= 4 ? (w << (19 - 4 * k)) : (w >> (4 * k - 19));
    return __uint_as_float(and_or(b, 0x00780000u, 0x3F800000u));  // one lop3, not an AND and an OR
}

#ifndef KQ_TQ_ATT_THREADS
#define KQ_TQ_ATT_THREADS 128
#endif
#ifndef KQ_TQ_CHUNK
#define KQ_TQ_CHUNK 256
#endif
constexpr int TQ_ATT_THREADS = KQ_TQ_ATT_THREADS;
constexpr int TQ_CHUNK = KQ_TQ_CHUNK;  // tokens per CTA
constexpr int TQ_MAXG = 8;     // query heads per KV head

struct TqAttParams {
    const uint8_t* packed[2];
    const float* scale[2];
    const float* zero[2];
    const float* R;
    const float* RT;
    const void* q;
    int q_dtype;
    int B, H, G, cap, len, nchunk;
    int Dr;         // head_dim (q / out stride, softmax scale)
    float* qrot;    // [B][Hq][D + 1]: q R and its sum
    float* part;    // [B][Hq][nchunk][D + 2]: sum p V~ (rotated), chunk max, sum p
    float* scores;  // [B][Hq][len] or null
    float* out;     // [B][Hq][D]
    uint32_t* status;
};

// q' = q R and sum(q'), once per query head: 256 threads, thread (half, j)
// sums half of the rows of column j
template <int D>
__global__ void __launch_bounds__(256) tq_rotate_q_kernel(TqAttParams p) {
    constexpr int SPLIT = 256 / D;
    __shared__ float qs[D];
    __shared__ float part[SPLIT][D];
    __shared__ float red[D / 32];
    const int qh = blockIdx.x, b = blockIdx.y, tid = threadIdx.x;
    const int j = tid % D, half = tid / D;
    const int Hq = p.H * p.G;
    pdl_launch_dependents();  // the attend kernel may start its copies now
    const size_t qoff = ((size_t)b * Hq + qh) * p.Dr;
    if (tid < D) qs[tid] = tid < p.Dr ? load_as_float(p.q, p.q_dtype, qoff + tid) : 0.f;
    __syncthreads();
    // all of this thread's R loads are issued before the first FMA: one memory round trip
    const int d0 = half * (D / SPLIT);
    float r[D / SPLIT];
#pragma unroll
    for (int d = 0; d < D / SPLIT; ++d) r[d] = __ldg(p.R + (size_t)(d0 + d) * D + j);
    float a = 0.f;
#pragma unroll
    for (int d = 0; d < D / SPLIT; ++d) a = fmaf(qs[d0 + d], r[d], a);
    part[half][j] = a;
    __syncthreads();
    if (tid < D) {
        float v = 0.f;
        for (int h2 = 0; h2 < SPLIT; ++h2) v += part[h2][tid];
        float* dst = p.qrot + ((size_t)b * Hq + qh) * (D + 1);
        dst[tid] = v;
        const float w = warp_sum(v);
        if ((tid & 31) == 0) red[tid >> 5] = w;
    }
    __syncthreads();
    if (tid == 0) {
        float t = 0.f;
        for (int i = 0; i < D / 32; ++i) t += red[i];
        p.qrot[((size_t)b * Hq + qh) * (D + 1) + D] = t;
    }
}

template <int D>
__host__ __device__ constexpr size_t tq_att_smem(int G) {
    // K, V codes + K, V scale/zero + scores + per-slot value partials + q' + barrier
    return (size_t)2 * TQ_CHUNK * (D / 2) + (size_t)4 * TQ_CHUNK * 4 + (size_t)G * TQ_CHUNK * 4 +
           (size_t)(TQ_ATT_THREADS / (D / 16)) * D * 4 + (size_t)G * (D + 1) * 4 + 64;
}

// One CTA per (chunk of TQ_CHUNK tokens, KV head, batch).  Thread 0 brings the
// chunk's codes, scales and zeros of K and V into shared memory with bulk
// copies on one mbarrier; every thread then works from shared memory.
template <int D>
__global__ void __launch_bounds__(TQ_ATT_THREADS) tq_attend_kernel(TqAttParams p) {
    constexpr int TPT = D / 16;                // threads per token (16 elements = 8 packed bytes each)
    constexpr int TPP = TQ_ATT_THREADS / TPT;  // tokens per pass
    constexpr int NW = TQ_ATT_THREADS / 32;
    constexpr int CB = D / 2;                  // packed bytes per vector
    extern __shared__ __align__(128) uint8_t att_sm[];
    const int G = p.G, Hq = p.H * G;
    uint8_t* kc = att_sm;                                           // [TQ_CHUNK][CB]
    uint8_t* vc = kc + TQ_CHUNK * CB;
    float* ksc = reinterpret_cast<float*>(vc + TQ_CHUNK * CB);      // [TQ_CHUNK]
    float* kze = ksc + TQ_CHUNK;
    float* vsc = kze + TQ_CHUNK;
    float* vze = vsc + TQ_CHUNK;
    float* sc = vze + TQ_CHUNK;                                     // [G][TQ_CHUNK]
    float* accs = sc + G * TQ_CHUNK;                                // [TPP][D]
    float* qr = accs + TPP * D;                                     // [G][D + 1]
    uint64_t* bar = reinterpret_cast<uint64_t*>(qr + G * (D + 1) + 1);  // 8-byte aligned below
    bar = reinterpret_cast<uint64_t*>((reinterpret_cast<uintptr_t>(bar) + 7) & ~uintptr_t(7));
    __shared__ float red[NW];
    __shared__ float cmax[TQ_MAXG], csum[TQ_MAXG];
    const int chunk = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int sub = tid % TPT, slot = tid / TPT;
    const int t0 = chunk * TQ_CHUNK, t1 = min(t0 + TQ_CHUNK, p.len);
    const int n = t1 - t0;
    const size_t row = ((size_t)b * p.H + h) * p.cap + t0;
    if (tid == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
        const uint32_t cbytes = (uint32_t)n * CB;              // multiple of 16
        const uint32_t fbytes = (uint32_t)((n + 3) & ~3) * 4;  // scale / zero rows carry tail padding
        mbar_expect_tx(bar, 2 * cbytes + 4 * fbytes);
        const uint64_t pol = policy_evict_first();
        bulk_g2s(kc, p.packed[0] + row * CB, cbytes, bar, pol);
        bulk_g2s(vc, p.packed[1] + row * CB, cbytes, bar, pol);
        bulk_g2s(ksc, p.scale[0] + row, fbytes, bar, pol);
        bulk_g2s(kze, p.zero[0] + row, fbytes, bar, pol);
        bulk_g2s(vsc, p.scale[1] + row, fbytes, bar, pol);
        bulk_g2s(vze, p.zero[1] + row, fbytes, bar, pol);
    }
    pdl_wait();  // q R is complete and visible (the chunk's copies are already in flight)
    pdl_launch_dependents();
    for (int i = tid; i < G * (D + 1); i += TQ_ATT_THREADS)
        qr[i] = p.qrot[((size_t)b * Hq + (size_t)h * G) * (D + 1) + i];
    __syncthreads();
    mbar_wait(bar, 0, p.status);
    const float sqrt_d = sqrtf((float)p.Dr);

    // scores on the codes; a thread's 16 query elements stay in registers for all its tokens
    const int npass = (n + TPP - 1) / TPP;
    for (int g = 0; g < G; ++g) {
        float qv[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) qv[e] = qr[g * (D + 1) + sub * 16 + e];
        const float qs = qr[g * (D + 1) + D];
        for (int i = 0; i < npass; ++i) {
            const int tl = i * TPP + slot;
            const int tc = tl < n ? tl : 0;
            const uint2 pk = *reinterpret_cast<const uint2*>(kc + tc * CB + sub * 8);
            const float s = ksc[tc], lo = kze[tc];
            // a = sum q (1 + v/8) with v = c + sigma/2; q.v = 8 (a - sum q)
            float a = 0.f;
#pragma unroll
            for (int e = 0; e < 16; ++e) a = fmaf(qv[e], nib_1p(e < 8 ? pk.x : pk.y, e & 7), a);
#pragma unroll
            for (int o = TPT / 2; o > 0; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
            const float score = __fdiv_rn(fmaf(s, 8.f * (a - qs), (lo - 0.25f * s) * qs), sqrt_d);
            if (tl < n && sub == 0) {
                sc[g * TQ_CHUNK + tl] = score;
                if (p.scores) p.scores[((size_t)b * Hq + (size_t)h * G + g) * p.len + t0 + tl] = score;
            }
        }
    }
    __syncthreads();

    for (int g = 0; g < G; ++g) {
        float* sg = sc + g * TQ_CHUNK;
        float m = -INFINITY;
        for (int i = tid; i < n; i += TQ_ATT_THREADS) m = fmaxf(m, sg[i]);
        m = warp_max(m);
        if (lane == 0) red[wid] = m;
        __syncthreads();
        m = red[0];
        for (int w = 1; w < NW; ++w) m = fmaxf(m, red[w]);
        float l = 0.f;
        for (int i = tid; i < n; i += TQ_ATT_THREADS) {
            const float e = expf(sg[i] - m);
            sg[i] = e;
            l += e;
        }
        l = warp_sum(l);
        __syncthreads();
        if (lane == 0) red[wid] = l;
        __syncthreads();
        if (tid == 0) {
            float ll = 0.f;
            for (int w = 0; w < NW; ++w) ll += red[w];
            cmax[g] = m;
            csum[g] = ll;
        }
        __syncthreads();
    }

    // values in the rotated domain: sum_t p_t (s_t c_t + z_t + (s_t/4)(2 sigma_t - 1))
    for (int g = 0; g < G; ++g) {
        const float* sg = sc + g * TQ_CHUNK;
        float acc[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) acc[e] = 0.f;
        float plo = 0.f;
        for (int i = 0; i < npass; ++i) {
            const int tl = i * TPP + slot;
            if (tl >= n) break;
            const uint2 pk = *reinterpret_cast<const uint2*>(vc + tl * CB + sub * 8);
            const float pt = sg[tl];
            // p (s c + z + (s/4)(2 sigma - 1)) = p s v + p (z - s/4) = 8 p s (1 + v/8) + p (z - s/4 - 8 s)
            const float w1 = 8.f * pt * vsc[tl];
#pragma unroll
            for (int e = 0; e < 16; ++e) acc[e] = fmaf(w1, nib_1p(e < 8 ? pk.x : pk.y, e & 7), acc[e]);
            if (sub == 0) plo = fmaf(pt, fmaf(-8.25f, vsc[tl], vze[tl]), plo);
        }
        __syncthreads();  // accs / red of the previous head are consumed
#pragma unroll
        for (int e = 0; e < 16; ++e) accs[slot * D + sub * 16 + e] = acc[e];
        const float pl = warp_sum(plo);
        if (lane == 0) red[wid] = pl;
        __syncthreads();
        float plsum = 0.f;
        for (int w = 0; w < NW; ++w) plsum += red[w];
        float* part = p.part + (((size_t)b * Hq + (size_t)h * G + g) * p.nchunk + chunk) * (D + 2);
        for (int d = tid; d < D; d += TQ_ATT_THREADS) {
            float a = plsum;
            for (int sl = 0; sl < TPP; ++sl) a += accs[sl * D + d];
            part[d] = a;
        }
        if (tid == 0) {
            part[D] = cmax[g];
            part[D + 1] = csum[g];
        }
    }
}

// Merge the chunk partials of one query head and un-rotate: out = (sum p V~ / sum p) R^T.
// 256 threads: warp w sums chunks c % 8 == w, lane covers dims lane + 32 i.
template <int D>
__global__ void __launch_bounds__(256) tq_combine_kernel(TqAttParams p) {
    constexpr int NWC = 8, DPL = D / 32;
    __shared__ float orot[D];
    __shared__ float pacc[NWC][D];
    __shared__ float pl[NWC], pm[NWC];
    const int qh = blockIdx.x, b = blockIdx.y, tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int Hq = p.H * p.G;
    const float* part = p.part + ((size_t)b * Hq + qh) * p.nchunk * (D + 2);
    pdl_wait();  // every chunk's partials are complete and visible
    float M = -INFINITY;
    for (int c = tid; c < p.nchunk; c += 256) M = fmaxf(M, part[(size_t)c * (D + 2) + D]);
    M = warp_max(M);
    if (lane == 0) pm[w] = M;
    __syncthreads();
    M = pm[0];
    for (int i = 1; i < NWC; ++i) M = fmaxf(M, pm[i]);
    float L = 0.f, A[DPL];
#pragma unroll
    for (int i = 0; i < DPL; ++i) A[i] = 0.f;
    // warp w merges chunks w, w + NWC, ...: a batch of CB chunks' loads is issued
    // before its arithmetic, in the same chunk order as one chunk at a time
    constexpr int CB = 8;
    for (int c0 = w; c0 < p.nchunk; c0 += NWC * CB) {
        float mv[CB], lv[CB], av[CB][DPL];
#pragma unroll
        for (int u = 0; u < CB; ++u) {
            const int c = c0 + u * NWC;
            const float* pc = part + (size_t)(c < p.nchunk ? c : 0) * (D + 2);
            mv[u] = c < p.nchunk ? pc[D] : -INFINITY;
            lv[u] = pc[D + 1];
#pragma unroll
            for (int i = 0; i < DPL; ++i) av[u][i] = pc[lane + 32 * i];
        }
#pragma unroll
        for (int u = 0; u < CB; ++u) {
            if (c0 + u * NWC >= p.nchunk) break;
            const float f = expf(mv[u] - M);
            L = fmaf(lv[u], f, L);
#pragma unroll
            for (int i = 0; i < DPL; ++i) A[i] = fmaf(av[u][i], f, A[i]);
        }
    }
#pragma unroll
    for (int i = 0; i < DPL; ++i) pacc[w][lane + 32 * i] = A[i];
    if (lane == 0) pl[w] = L;
    __syncthreads();
    if (tid < D) {
        float a = 0.f, l = 0.f;
        for (int i = 0; i < NWC; ++i) {
            a += pacc[i][tid];
            l += pl[i];
        }
        orot[tid] = a / l;
    }
    __syncthreads();
    // un-rotate: out[d] = sum_k orot[k] R^T[k][d]; thread (d, half) takes half of k,
    // its R^T loads issued together
    constexpr int KS = 256 / D;
    const int d = tid % D, hk = tid / D, k0 = hk * (D / KS);
    float rt[D / KS];
#pragma unroll
    for (int k = 0; k < D / KS; ++k) rt[k] = __ldg(p.RT + (size_t)(k0 + k) * D + d);
    float o = 0.f;
#pragma unroll
    for (int k = 0; k < D / KS; ++k) o = fmaf(orot[k0 + k], rt[k], o);
    pacc[hk][d] = o;  // pacc is free again: its sums were read before the barrier above
    __syncthreads();
    if (tid < p.Dr) {
        float v = 0.f;
        for (int h2 = 0; h2 < KS; ++h2) v += pacc[h2][tid];
        p.out[((size_t)b * Hq + qh) * p.Dr + tid] = v;
    }
}

// ---- host ----------------------------------------------------------------------------------------

static void free_planes(kq_tq_cache* c) {
    for (int w = 0; w < 2; ++w) {
        cudaFree(c->packed[w]);
        cudaFree(c->scale[w]);
        cudaFree(c->zero[w]);
        c->packed[w] = nullptr;
        c->scale[w] = c->zero[w] = nullptr;
    }
}

static bool alloc_planes(const kq_tq_cache* c, int cap, uint8_t* (&packed)[2], float* (&scale)[2],
                         float* (&zero)[2]) {
    const size_t nv = (size_t)c->B * c->H * (size_t)(cap > 0 ? cap : 1) + 16;  // tail padding
    for (int w = 0; w < 2; ++w) {
        packed[w] = nullptr;
        scale[w] = zero[w] = nullptr;
    }
    for (int w = 0; w < 2; ++w) {
        if (cudaMalloc(&packed[w], nv * (c->D / 2)) != cudaSuccess || cudaMalloc(&scale[w], nv * 4) != cudaSuccess ||
            cudaMalloc(&zero[w], nv * 4) != cudaSuccess) {
            for (int v = 0; v < 2; ++v) {
                cudaFree(packed[v]);
                cudaFree(scale[v]);
                cudaFree(zero[v]);
            }
            return false;
        }
    }
    return true;
}

// capacities are multiples of 4 vectors so every row of scales / zeros starts 16-byte aligned
static int round_cap(int cap) { return (cap + 3) & ~3; }

static int sm_count() {
    int dev = 0, n = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n;
}

template <typename K>
static cudaError_t smem_attr_once(K kern, size_t smem, int* configured) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if ((size_t)configured[dev] >= smem) return cudaSuccess;
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess) configured[dev] = (int)smem;
    return e;
}

template <int D>
static cudaError_t launch_append(const TqVecParams& p, cudaStream_t s) {
    static int configured[64] = {0};
    const size_t smem = ((size_t)2 * D * D + (size_t)TQ_WARPS * TQ_VPW * D) * 4;
    cudaError_t e = smem_attr_once(tq_append_kernel<D>, smem, configured);
    if (e != cudaSuccess) return e;
    const long nvec = 2L * p.B * p.H * p.T;
    const long per_cta = (long)TQ_WARPS * TQ_VPW;
    const int grid = (int)std::min<long>((nvec + per_cta - 1) / per_cta, (long)sm_count());
    tq_append_kernel<D><<<grid, TQ_WARPS * 32, smem, s>>>(p);
    return cudaGetLastError();
}

static cudaError_t launch_append_tc(const TqVecParams& p, cudaStream_t s) {
    static int configured[64] = {0};
    cudaError_t e = smem_attr_once(tq_append_tc_kernel, tq_tc_smem(), configured);
    if (e != cudaSuccess) return e;
    const long ntiles = (2L * p.B * p.H * p.T + 127) / 128;
    const int grid = (int)std::min<long>(ntiles, (long)sm_count());
    tq_append_tc_kernel<<<grid, TQTC_THREADS, tq_tc_smem(), s>>>(p);
    return cudaGetLastError();
}

template <int D>
static cudaError_t launch_dequant(const TqVecParams& p, cudaStream_t s) {
    static int configured[64] = {0};
    const size_t smem = ((size_t)D * D + (size_t)TQ_WARPS * TQ_VPW * D) * 4;
    cudaError_t e = smem_attr_once(tq_dequant_kernel<D>, smem, configured);
    if (e != cudaSuccess) return e;
    const long nvec = (long)p.B * p.H * p.len;
    const long per_cta = (long)TQ_WARPS * TQ_VPW;
    const int grid = (int)std::min<long>((nvec + per_cta - 1) / per_cta, (long)sm_count());
    tq_dequant_kernel<D><<<grid, TQ_WARPS * 32, smem, s>>>(p);
    return cudaGetLastError();
}

template <int D>
static cudaError_t launch_attend(const TqAttParams& p, dim3 grid, dim3 cgrid, cudaStream_t s) {
    static int configured[64] = {0};
    const size_t smem = tq_att_smem<D>(TQ_MAXG);
    cudaError_t e = smem_attr_once(tq_attend_kernel<D>, smem, configured);
    if (e != cudaSuccess) return e;
    // rotate-q -> attend -> combine as programmatic dependents: each kernel
    // starts (the attend CTAs issue their chunk copies) while its predecessor
    // finishes, and waits for it before reading its output
    tq_rotate_q_kernel<D><<<cgrid, 256, 0, s>>>(p);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    if ((e = launch_dep(tq_attend_kernel<D>, grid, dim3(TQ_ATT_THREADS), tq_att_smem<D>(p.G), s, p)) != cudaSuccess)
        return e;
    return launch_dep(tq_combine_kernel<D>, cgrid, dim3(256), (size_t)0, s, p);
}

}  // namespace kq

using namespace kq;

extern "C" int kq_tq_create(int head_dim, int num_heads, int batch, int capacity, const float* rotation,
                            const float* qjl, kq_tq_cache** out) {
    if (!out) return KQ_ERR_ARG;
    *out = nullptr;
    if (head_dim <= 0 || num_heads <= 0 || batch <= 0 || capacity < 0 || !rotation || !qjl) return KQ_ERR_ARG;
    if (head_dim > 128) return KQ_ERR_UNSUPPORTED;
    const int Dr = head_dim;
    head_dim = Dr <= 64 ? 64 : 128;  // storage width
    kq_tq_cache* c = new (std::nothrow) kq_tq_cache();
    if (!c) return KQ_ERR_ALLOC;
    c->D = head_dim;
    c->Dr = Dr;
    c->H = num_heads;
    c->B = batch;
    capacity = round_cap(capacity);
    const size_t mb = (size_t)head_dim * head_dim * 4;
    if (cudaMalloc(&c->R, mb) != cudaSuccess || cudaMalloc(&c->RT, mb) != cudaSuccess ||
        cudaMalloc(&c->P, mb) != cudaSuccess || cudaMalloc(&c->status, 4) != cudaSuccess ||
        cudaMemset(c->status, 0, 4) != cudaSuccess || !alloc_planes(c, capacity, c->packed, c->scale, c->zero)) {
        cudaFree(c->R);
        cudaFree(c->RT);
        cudaFree(c->P);
        cudaFree(c->status);
        delete c;
        return KQ_ERR_ALLOC;
    }
    c->cap = capacity;
    // R and P at the storage width: R extended by the identity, P by zeros
    const size_t nn = (size_t)head_dim * head_dim;
    float* host = new (std::nothrow) float[3 * nn];
    if (!host) {
        kq_tq_destroy(c);
        return KQ_ERR_ALLOC;
    }
    float *r = host, *rt = host + nn, *pj = host + 2 * nn;
    for (int i = 0; i < head_dim; ++i)
        for (int j = 0; j < head_dim; ++j) {
            const bool in = i < Dr && j < Dr;
            r[(size_t)i * head_dim + j] = in ? rotation[(size_t)i * Dr + j] : (i == j ? 1.f : 0.f);
            pj[(size_t)i * head_dim + j] = in ? qjl[(size_t)i * Dr + j] : 0.f;
        }
    for (int i = 0; i < head_dim; ++i)
        for (int j = 0; j < head_dim; ++j) rt[(size_t)j * head_dim + i] = r[(size_t)i * head_dim + j];
    const bool up = cudaMemcpy(c->R, r, mb, cudaMemcpyHostToDevice) == cudaSuccess &&
                    cudaMemcpy(c->RT, rt, mb, cudaMemcpyHostToDevice) == cudaSuccess &&
                    cudaMemcpy(c->P, pj, mb, cudaMemcpyHostToDevice) == cudaSuccess;
    delete[] host;
    if (!up) {
        kq_tq_destroy(c);
        return KQ_ERR_CUDA;
    }
    if (head_dim == TQTC_D) {  // the tensor-core append's operand images
        if (cudaMalloc(&c->tc_ops, 4 * (size_t)TQTC_OP) != cudaSuccess) {
            c->tc_ops = nullptr;
            kq_tq_destroy(c);
            return KQ_ERR_ALLOC;
        }
        tq_tc_ops_kernel<<<TQTC_D, TQTC_D / 8>>>(c->RT, c->P, c->tc_ops);
        if (cudaGetLastError() != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
            kq_tq_destroy(c);
            return KQ_ERR_CUDA;
        }
    }
    *out = c;
    return KQ_OK;
}

extern "C" int kq_tq_destroy(kq_tq_cache* c) {
    if (!c) return KQ_OK;
    free_planes(c);
    cudaFree(c->R);
    cudaFree(c->RT);
    cudaFree(c->P);
    cudaFree(c->status);
    cudaFree(c->tc_ops);
    delete c;
    return KQ_OK;
}

extern "C" int kq_tq_status(const kq_tq_cache* c, uint32_t* status_out, void* stream) {
    if (!c || !status_out) return KQ_ERR_ARG;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (cudaMemcpyAsync(status_out, c->status, 4, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return KQ_ERR_CUDA;
    return KQ_OK;
}

extern "C" int kq_tq_seq_len(const kq_tq_cache* c) { return c ? c->len : -1; }
extern "C" int kq_tq_storage_dim(const kq_tq_cache* c) { return c ? c->D : -1; }
extern "C" int kq_tq_capacity(const kq_tq_cache* c) { return c ? c->cap : -1; }

extern "C" int kq_tq_reserve(kq_tq_cache* c, int capacity, void* stream) {
    if (!c || capacity < 0) return KQ_ERR_ARG;
    if (capacity <= c->cap) return KQ_OK;
    capacity = round_cap(capacity);
    uint8_t* packed[2];
    float *scale[2], *zero[2];
    if (!alloc_planes(c, capacity, packed, scale, zero)) return KQ_ERR_ALLOC;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t rows = (size_t)c->B * c->H;
    bool ok = true;
    if (c->len > 0) {
        for (int w = 0; w < 2 && ok; ++w) {
            const size_t pb = (size_t)c->D / 2;
            ok = cudaMemcpy2DAsync(packed[w], capacity * pb, c->packed[w], c->cap * pb, c->len * pb, rows,
                                   cudaMemcpyDeviceToDevice, s) == cudaSuccess &&
                 cudaMemcpy2DAsync(scale[w], capacity * 4, c->scale[w], c->cap * 4ull, c->len * 4ull, rows,
                                   cudaMemcpyDeviceToDevice, s) == cudaSuccess &&
                 cudaMemcpy2DAsync(zero[w], capacity * 4, c->zero[w], c->cap * 4ull, c->len * 4ull, rows,
                                   cudaMemcpyDeviceToDevice, s) == cudaSuccess;
        }
    }
    if (ok) ok = cudaStreamSynchronize(s) == cudaSuccess;
    if (!ok) {
        for (int w = 0; w < 2; ++w) {
            cudaFree(packed[w]);
            cudaFree(scale[w]);
            cudaFree(zero[w]);
        }
        return KQ_ERR_CUDA;
    }
    free_planes(c);
    for (int w = 0; w < 2; ++w) {
        c->packed[w] = packed[w];
        c->scale[w] = scale[w];
        c->zero[w] = zero[w];
    }
    c->cap = capacity;
    return KQ_OK;
}

extern "C" int kq_tq_append(kq_tq_cache* c, const void* keys, const void* values, int dtype, int T, void* stream) {
    if (!c || T < 0) return KQ_ERR_ARG;
    if (dtype != KQ_DT_F16 && dtype != KQ_DT_BF16 && dtype != KQ_DT_F32) return KQ_ERR_ARG;
    if (T == 0) return KQ_OK;
    if (!keys || !values) return KQ_ERR_ARG;
    if ((long)c->len + T > c->cap) return KQ_ERR_CAPACITY;
    TqVecParams p{};
    p.src[0] = keys;
    p.src[1] = values;
    p.dtype = dtype;
    p.B = c->B;
    p.H = c->H;
    p.T = T;
    p.cap = c->cap;
    p.len = c->len;
    p.Dr = c->Dr;
    p.R = c->R;
    p.RT = c->RT;  // the tensor-core path stages R^T as its B operand
    p.P = c->P;
    for (int w = 0; w < 2; ++w) {
        p.packed[w] = c->packed[w];
        p.scale[w] = c->scale[w];
        p.zero[w] = c->zero[w];
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    p.status = c->status;
    p.tc_ops = c->tc_ops;
    // Below 2048 vectors (a decode step's few tokens) the FMA kernel's shorter
    // start-up wins; bulk appends go to the tensor cores.
    const long nvec = 2L * c->B * c->H * T;
    const cudaError_t e = c->D == 128 ? (nvec >= 2048 ? launch_append_tc(p, s) : launch_append<128>(p, s))
                                      : launch_append<64>(p, s);
    if (e != cudaSuccess) return KQ_ERR_CUDA;
    c->len += T;
    return KQ_OK;
}

extern "C" int kq_tq_dequant(const kq_tq_cache* c, int which, void* out_f16, void* stream) {
    if (!c || (which != 0 && which != 1)) return KQ_ERR_ARG;
    if (c->len == 0) return KQ_OK;
    if (!out_f16) return KQ_ERR_ARG;
    TqVecParams p{};
    p.B = c->B;
    p.H = c->H;
    p.cap = c->cap;
    p.len = c->len;
    p.Dr = c->Dr;
    p.R = c->R;
    p.RT = c->RT;
    for (int w = 0; w < 2; ++w) {
        p.packed[w] = c->packed[w];
        p.scale[w] = c->scale[w];
        p.zero[w] = c->zero[w];
    }
    p.out = static_cast<__half*>(out_f16);
    p.which = which;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const cudaError_t e = c->D == 128 ? launch_dequant<128>(p, s) : launch_dequant<64>(p, s);
    return e == cudaSuccess ? KQ_OK : KQ_ERR_CUDA;
}

extern "C" int kq_tq_export(const kq_tq_cache* c, int which, int8_t* codes, int8_t* signs, float* scales,
                            float* zeros, void* stream) {
    if (!c || (which != 0 && which != 1)) return KQ_ERR_ARG;
    if (c->len == 0) return KQ_OK;
    const long n = (long)c->B * c->H * c->len * c->Dr;
    const int threads = 256;
    tq_export_kernel<<<(int)((n + threads - 1) / threads), threads, 0, static_cast<cudaStream_t>(stream)>>>(
        c->packed[which], c->scale[which], c->zero[which], c->D, c->Dr, c->B * c->H, c->cap, c->len, codes, signs,
        scales, zeros);
    return cudaGetLastError() == cudaSuccess ? KQ_OK : KQ_ERR_CUDA;
}

// Compact copies of the packed storage (session persistence): rows of the
// cache are `cap` vectors apart, rows of the saved arrays `len` apart.
extern "C" int kq_tq_save(const kq_tq_cache* c, int which, uint8_t* packed, float* scales, float* zeros,
                          void* stream) {
    if (!c || (which != 0 && which != 1)) return KQ_ERR_ARG;
    if (c->len == 0) return KQ_OK;
    if (!packed || !scales || !zeros) return KQ_ERR_ARG;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t rows = (size_t)c->B * c->H, vb = (size_t)c->D / 2;
    const bool ok =
        cudaMemcpy2DAsync(packed, c->len * vb, c->packed[which], (size_t)c->cap * vb, c->len * vb, rows,
                          cudaMemcpyDeviceToDevice, s) == cudaSuccess &&
        cudaMemcpy2DAsync(scales, c->len * 4, c->scale[which], (size_t)c->cap * 4, c->len * 4, rows,
                          cudaMemcpyDeviceToDevice, s) == cudaSuccess &&
        cudaMemcpy2DAsync(zeros, c->len * 4, c->zero[which], (size_t)c->cap * 4, c->len * 4, rows,
                          cudaMemcpyDeviceToDevice, s) == cudaSuccess;
    return ok ? KQ_OK : KQ_ERR_CUDA;
}

extern "C" int kq_tq_restore(kq_tq_cache* c, int len, const uint8_t* k_packed, const float* k_scales,
                             const float* k_zeros, const uint8_t* v_packed, const float* v_scales,
                             const float* v_zeros, void* stream) {
    if (!c || len < 0) return KQ_ERR_ARG;
    if (len > 0 && (!k_packed || !k_scales || !k_zeros || !v_packed || !v_scales || !v_zeros)) return KQ_ERR_ARG;
    if (len > c->cap) {
        const int rc = kq_tq_reserve(c, len, stream);
        if (rc != KQ_OK) return rc;
    }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t rows = (size_t)c->B * c->H, vb = (size_t)c->D / 2;
    const uint8_t* pk[2] = {k_packed, v_packed};
    const float* sc[2] = {k_scales, v_scales};
    const float* zr[2] = {k_zeros, v_zeros};
    for (int w = 0; w < 2 && len > 0; ++w) {
        if (cudaMemcpy2DAsync(c->packed[w], (size_t)c->cap * vb, pk[w], (size_t)len * vb, (size_t)len * vb, rows,
                              cudaMemcpyDeviceToDevice, s) != cudaSuccess ||
            cudaMemcpy2DAsync(c->scale[w], (size_t)c->cap * 4, sc[w], (size_t)len * 4, (size_t)len * 4, rows,
                              cudaMemcpyDeviceToDevice, s) != cudaSuccess ||
            cudaMemcpy2DAsync(c->zero[w], (size_t)c->cap * 4, zr[w], (size_t)len * 4, (size_t)len * 4, rows,
                              cudaMemcpyDeviceToDevice, s) != cudaSuccess)
            return KQ_ERR_CUDA;
    }
    c->len = len;
    return KQ_OK;
}

extern "C" size_t kq_tq_attend_workspace_size(const kq_tq_cache* c, int q_heads) {
    if (!c || q_heads <= 0) return 0;
    const size_t nchunk = ((size_t)(c->cap > 0 ? c->cap : 1) + TQ_CHUNK - 1) / TQ_CHUNK;
    return 16 + (size_t)c->B * q_heads * ((c->D + 1) + nchunk * (c->D + 2)) * 4;
}

extern "C" int kq_tq_attend(const kq_tq_cache* c, const void* q, int q_dtype, int q_heads, float* out,
                            float* scores, void* workspace, size_t workspace_bytes, void* stream) {
    if (!c || !q || !out || q_heads <= 0 || q_heads % c->H) return KQ_ERR_ARG;
    if (q_dtype != KQ_DT_F16 && q_dtype != KQ_DT_BF16 && q_dtype != KQ_DT_F32) return KQ_ERR_ARG;
    const int G = q_heads / c->H;
    if (G > TQ_MAXG) return KQ_ERR_UNSUPPORTED;
    if (c->len == 0) return KQ_ERR_ARG;  // softmax over an empty sequence
    const int nchunk = (c->len + TQ_CHUNK - 1) / TQ_CHUNK;
    const size_t need = 16 + (size_t)c->B * q_heads * ((c->D + 1) + (size_t)nchunk * (c->D + 2)) * 4;
    if (!workspace || workspace_bytes < need) return KQ_ERR_WORKSPACE;
    TqAttParams p{};
    for (int w = 0; w < 2; ++w) {
        p.packed[w] = c->packed[w];
        p.scale[w] = c->scale[w];
        p.zero[w] = c->zero[w];
    }
    p.R = c->R;
    p.RT = c->RT;
    p.q = q;
    p.q_dtype = q_dtype;
    p.B = c->B;
    p.H = c->H;
    p.G = G;
    p.cap = c->cap;
    p.len = c->len;
    p.nchunk = nchunk;
    p.Dr = c->Dr;
    // workspace: status word (16 B), q R, chunk partials
    p.status = static_cast<uint32_t*>(workspace);
    p.qrot = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + 16);
    p.part = p.qrot + (size_t)c->B * q_heads * (c->D + 1);
    p.scores = scores;
    p.out = out;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const dim3 grid(nchunk, c->H, c->B), cgrid(q_heads, c->B);
    cudaError_t e = c->D == 128 ? launch_attend<128>(p, grid, cgrid, s) : launch_attend<64>(p, grid, cgrid, s);
    if (e != cudaSuccess) return KQ_ERR_CUDA;
    return cudaGetLastError() == cudaSuccess ? KQ_OK : KQ_ERR_CUDA;
}
