// kq_full.cu -- whole-model single-token decode step behind the reference's
// bakan_full_* ABI (kandiga/metal/full_forward.h:43-220).
//
// The reference hard-codes one model's constants (full_forward_lg.m:39-109)
// and encodes every step as Metal command buffers.  Here the model shape comes
// from its config.json, and one decode step is two CUDA graphs replayed
// back to back (body: embedding + all layers; head: final norm + LM head), with
// the token id, position and KV length in device memory, so a step costs two
// graph launches and the copies of the token in and the logits out.
//
// Per attention layer (full_forward_lg.m:1140-1354):
//   kq_dense_gemv        input RMSNorm + stacked q|k|v projection (one pass)
//   attn_chunk_kernel    per-head RMSNorm of q and k (q_norm / k_norm), RoPE from
//                        the step's table, K and V appended to the fp16 cache,
//                        GQA attention over one context chunk per CTA (one per
//                        SM; all q heads of a kv head share each K/V row; the
//                        cached rows are requested before the wait on the
//                        projection)
//   attn_merge_kernel    chunk merge per (q head, 32 dims), sigmoid output gate
//   kq_dense_gemv        o_proj with the residual added in its epilogue
// Per GatedDeltaNet layer (full_forward_lg.m:1361-1508): kq_dense_gemv (input
// RMSNorm + q|k|v|z|b|a), gdn_conv_kernel (ring buffer + conv1d + SiLU),
// gdn_state_kernel (q/k norm and scale, gated delta rule on the fp32 state,
// RMSNormGated of the head), kq_dense_gemv (out_proj + residual).
// MLP: the MoE block engine of kq_forward.cu (routed experts from the BKEX
// files, shared expert, gate, blend) or a dense MLP: RMSNorm + gate/up pair
// with SwiGLU in one pass, then down with the residual.  Rounding points follow the reference's kernels: every buffer
// between kernels is fp16 (attention.metal writes half after each step).
#include "kq_internal.h"
#include "kq_common.cuh"

#include <cctype>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <new>
#include <string>
#include <vector>

namespace kq {
namespace full {

constexpr int ATTN_WARPS = 8;
constexpr int ATTN_CTAS = 148;  // attention chunk CTAs per layer (one per SM), split over the kv heads

struct Cfg {
    int hidden = 0, inter = 0, layers = 0, nq = 0, nkv = 0, hd = 0, rope_dim = 0, vocab = 0, max_seq = 4096;
    float eps = 1e-6f, theta = 10000.f;
    int group = 64;
    int act = KQ_ACT_SILU;
    std::vector<char> linear;  // per layer: 1 = GatedDeltaNet, 0 = full attention
    int lnk = 0, lnv = 0, lkd = 0, lvd = 0, conv_k = 4;  // GatedDeltaNet heads and dims
    int num_experts = 0;       // > 0: MoE MLP, experts from the BKEX layer files
    int conv_dim() const { return 2 * lnk * lkd + lnv * lvd; }
    int lin_proj_rows() const { return conv_dim() + lnv * lvd + 2 * lnv; }
};

// ---- kernels ------------------------------------------------------------------------

// One embedding row: MLX-affine quantized (bits 2..8, codes LSB-first as a bit
// stream, value = q * scale + bias; kandiga/metal/attention.metal:190-224) or
// plain fp16/bf16.  The token id is read from device memory.
// Block 0 also writes this position's RoPE table, rope[i] = (cos, sin) of
// pos * theta^(-2i / rope_dim) for i < rope_dim / 2 (attention.metal:697-734),
// which every layer's attention reads.
__global__ void embed_kernel(const int* __restrict__ dev_i, int vocab, const uint8_t* __restrict__ w,
                             const uint16_t* __restrict__ s, const uint16_t* __restrict__ b, int bits, int sb_dtype,
                             int kind, int H, int group, __half* __restrict__ out, int rope_dim, float theta,
                             float2* __restrict__ rope, uint32_t* status) {
    if (blockIdx.x == 0) {
        const int pos = dev_i[1];
        for (int r = threadIdx.x; r < rope_dim / 2; r += blockDim.x) {
            const float freq = 1.f / powf(theta, (float)(2 * r) / (float)rope_dim);
            const float ang = (float)pos * freq;
            rope[r] = make_float2(cosf(ang), sinf(ang));
        }
    }
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= H) return;
    const int tok = dev_i[0];
    if (tok < 0 || tok >= vocab) {
        if (i == 0) set_status(status, KQ_DEV_BAD_INDEX);
        out[i] = __float2half(0.f);
        return;
    }
    float v;
    if (kind == 0) {
        const size_t row_bytes = (size_t)H * bits / 8;
        const uint8_t* row = w + (size_t)tok * row_bytes;
        const size_t bit = (size_t)i * bits;
        const size_t by = bit >> 3;
        const uint32_t lo = row[by], hi = (by + 1 < row_bytes) ? row[by + 1] : 0u;
        const uint32_t q = ((lo | (hi << 8)) >> (bit & 7)) & ((1u << bits) - 1u);
        const int gpr = H / group;
        const float sc = load_as_float(s, sb_dtype, (size_t)tok * gpr + i / group);
        const float bi = load_as_float(b, sb_dtype, (size_t)tok * gpr + i / group);
        v = fmaf((float)q, sc, bi);
    } else {
        v = load_as_float(w, kind == 1 ? KQ_DT_F16 : KQ_DT_BF16, (size_t)tok * H + i);
    }
    out[i] = __float2half(v);
}

__device__ __forceinline__ float block_sum(float v, float* red) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.f;
    for (int w = 0; w < nw; ++w) t += red[w];
    return t;
}

template <int DPL>
__device__ __forceinline__ void load_row(const __half* p, float* f) {
    if constexpr (DPL == 8) {
        const uint4 u = *reinterpret_cast<const uint4*>(p);
        const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float2 t = __half22float2(h[j]);
            f[2 * j] = t.x;
            f[2 * j + 1] = t.y;
        }
    } else if constexpr (DPL == 4) {
        const uint2 u = *reinterpret_cast<const uint2*>(p);
        const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const float2 t = __half22float2(h[j]);
            f[2 * j] = t.x;
            f[2 * j + 1] = t.y;
        }
    } else {
        const float2 t = __half22float2(*reinterpret_cast<const __half2*>(p));
        f[0] = t.x;
        f[1] = t.y;
    }
}

// DPL halves kept packed (DPL / 2 words) until used
template <int DPL>
__device__ __forceinline__ void load_raw(const __half* p, uint32_t* r) {
    if constexpr (DPL == 8) {
        const uint4 u = *reinterpret_cast<const uint4*>(p);
        r[0] = u.x;
        r[1] = u.y;
        r[2] = u.z;
        r[3] = u.w;
    } else if constexpr (DPL == 4) {
        const uint2 u = *reinterpret_cast<const uint2*>(p);
        r[0] = u.x;
        r[1] = u.y;
    } else {
        r[0] = *reinterpret_cast<const uint32_t*>(p);
    }
}

template <int DPL>
__device__ __forceinline__ void unpack_raw(const uint32_t* r, float* f) {
#pragma unroll
    for (int j = 0; j < DPL / 2; ++j) {
        const float2 t = __half22float2(*reinterpret_cast<const __half2*>(&r[j]));
        f[2 * j] = t.x;
        f[2 * j + 1] = t.y;
    }
}

template <int DPL>
__device__ __forceinline__ void store_row(__half* p, const float* f) {
#pragma unroll
    for (int j = 0; j < DPL; j += 2)
        *reinterpret_cast<__half2*>(p + j) = __floats2half2_rn(f[j], f[j + 1]);
}

struct AttnArgs {
    const __half* qkv;     // [q (| gate per head) | k | v] of this token, fp16
    const __half* q_norm;  // [hd] or null
    const __half* k_norm;
    __half* kc;            // [nkv][max_seq][hd]
    __half* vc;
    const int* dev_i;      // token, position, kv length
    const float2* rope;    // [rope_dim / 2] (cos, sin) at this position
    float* pm;             // [nq][nch]
    float* pl;
    float* pacc;           // [nq][nch][hd]
    __half* out;           // [nq][hd]
    uint32_t* status;
    int nq, nkv, max_seq, gate, rope_dim, nch;
    float eps;
};

// Prepare one head row in warp-owned shared memory: fp16 values, then the
// per-head RMSNorm with weight (attention.metal:898-949) and RoPE on dims
// [0, rope_dim) with pairs (i, i + rope_dim/2) (attention.metal:697-734), each
// rounded to fp16 as the reference writes half after every kernel.
template <int DPL>
__device__ __forceinline__ void prep_row(const __half* src, const __half* nw, float eps, int rope_dim,
                                         const float2* __restrict__ rope, float* row) {
    constexpr int HD = 32 * DPL;
    const int lane = threadIdx.x & 31;
    float v[DPL];
    load_row<DPL>(src + lane * DPL, v);
    if (nw) {
        float ss = 0.f;
#pragma unroll
        for (int j = 0; j < DPL; ++j) ss += v[j] * v[j];
        const float sc = 1.f / sqrtf(warp_sum(ss) / (float)HD + eps);
        float w[DPL];
        load_row<DPL>(nw + lane * DPL, w);
#pragma unroll
        for (int j = 0; j < DPL; ++j) v[j] = __half2float(__float2half((v[j] * sc) * w[j]));
    }
#pragma unroll
    for (int j = 0; j < DPL; ++j) row[lane * DPL + j] = v[j];
    __syncwarp();
    const int hr = rope_dim / 2;
    for (int i = lane; i < hr; i += 32) {
        const float2 cs = rope[i];
        const float c = cs.x, s = cs.y;
        const float x0 = row[i], x1 = row[i + hr];
        row[i] = __half2float(__float2half(x0 * c - x1 * s));
        row[i + hr] = __half2float(__float2half(x0 * s + x1 * c));
    }
    __syncwarp();
}

// Decode attention of one layer, part 1: softmax(q K^T / sqrt(hd)) V
// (attention.metal:752-849) for the G q heads of kv head blockIdx.x over
// token chunk blockIdx.y (the context split over gridDim.y CTAs, one per SM).
//   0. warp w owns tokens t0 + w, t0 + w + 8, ...; lane l owns dims
//      [l*DPL, l*DPL + DPL).  The K and V rows of the warp's first TB tokens are
//      requested before griddepcontrol.wait: cached rows do not depend on the
//      q|k|v projection still running, so their fetch overlaps it (the new
//      position's row is read after the wait);
//   1. the warps prepare the G q rows (norm, RoPE) in shared memory; the CTA
//      whose chunk holds the new position also prepares k and appends k and v;
//   2. online softmax per q head over the warp's tokens, TB rows in flight;
//   3. the warps are merged in shared memory and the chunk's (max, sum,
//      unnormalised acc) per q head written out for attn_merge_kernel.
template <int DPL, int G>
__global__ void __launch_bounds__(ATTN_WARPS * 32, 1) attn_chunk_kernel(const AttnArgs a) {
    constexpr int HD = 32 * DPL;
    constexpr int TB = G * DPL >= 64 ? 4 : 8;  // tokens whose rows are in flight per warp
    extern __shared__ __align__(16) float sm[];
    float* sq = sm;                            // [G][HD] prepared q rows
    float* sk = sq + G * HD;                   // [HD] new k row
    float* s_acc = sk + HD;                    // [ATTN_WARPS][G][HD]
    float* s_m = s_acc + ATTN_WARPS * G * HD;  // [ATTN_WARPS][G]
    float* s_l = s_m + ATTN_WARPS * G;
    float* s_f = s_l + ATTN_WARPS * G;         // [ATTN_WARPS][G] warp weights
    float* s_L = s_f + ATTN_WARPS * G;         // [G]
    const int kvh = blockIdx.x, c = blockIdx.y, nch = gridDim.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // dev_i was written before the step's first kernel: readable before the wait
    const int pos = a.dev_i[1];
    const int kv_len = min(a.dev_i[2], a.max_seq);
    const int per = (kv_len + nch - 1) / nch;
    const int t0 = c * per, t1 = min(kv_len, t0 + per);
    const bool owns_pos = pos >= t0 && pos < t1 && pos < a.max_seq;
    const __half* kb = a.kc + (size_t)kvh * a.max_seq * HD + lane * DPL;
    const __half* vb = a.vc + (size_t)kvh * a.max_seq * HD + lane * DPL;

    // 0. first batch of cached rows, before the wait
    uint32_t kr[TB][DPL / 2], vr[TB][DPL / 2];
#pragma unroll
    for (int i = 0; i < TB; ++i) {
        const int t = t0 + warp + i * ATTN_WARPS;
        if (t < t1 && t != pos) {
            load_raw<DPL>(kb + (size_t)t * HD, kr[i]);
            load_raw<DPL>(vb + (size_t)t * HD, vr[i]);
        }
    }
    pdl_wait();
    pdl_launch_dependents();
    const int qstride = a.gate ? 2 * HD : HD;
    const size_t qtot = (size_t)a.nq * qstride;

    // 1. q rows (and the new k / v rows)
    for (int job = warp; job <= G; job += ATTN_WARPS) {
        if (job < G) {
            prep_row<DPL>(a.qkv + (size_t)(kvh * G + job) * qstride, a.q_norm, a.eps, a.rope_dim, a.rope,
                          sq + job * HD);
        } else if (owns_pos) {
            prep_row<DPL>(a.qkv + qtot + (size_t)kvh * HD, a.k_norm, a.eps, a.rope_dim, a.rope, sk);
            float kv[DPL];
#pragma unroll
            for (int j = 0; j < DPL; ++j) kv[j] = sk[lane * DPL + j];
            store_row<DPL>(a.kc + ((size_t)kvh * a.max_seq + pos) * HD + lane * DPL, kv);
            load_row<DPL>(a.qkv + qtot + (size_t)a.nkv * HD + (size_t)kvh * HD + lane * DPL, kv);
            store_row<DPL>(a.vc + ((size_t)kvh * a.max_seq + pos) * HD + lane * DPL, kv);
        }
    }
    if (a.dev_i[1] >= a.max_seq && kvh == 0 && c == 0 && threadIdx.x == 0) set_status(a.status, KQ_DEV_BAD_INDEX);
    __syncthreads();  // q rows ready; the new K / V rows are visible to this CTA

    // 2. this CTA's tokens
    float qf[G][DPL];
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int j = 0; j < DPL; ++j) qf[g][j] = sq[g * HD + lane * DPL + j];
    float m[G], l[G], acc[G][DPL];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
#pragma unroll
        for (int j = 0; j < DPL; ++j) acc[g][j] = 0.f;
    }
    const float inv_sqrt = 1.f / sqrtf((float)HD);
    for (int tb = t0 + warp; tb < t1; tb += TB * ATTN_WARPS) {
        if (tb != t0 + warp) {  // later batches: fetched now
#pragma unroll
            for (int i = 0; i < TB; ++i) {
                const int t = tb + i * ATTN_WARPS;
                if (t < t1 && t != pos) {
                    load_raw<DPL>(kb + (size_t)t * HD, kr[i]);
                    load_raw<DPL>(vb + (size_t)t * HD, vr[i]);
                }
            }
        }
#pragma unroll
        for (int i = 0; i < TB; ++i) {
            const int t = tb + i * ATTN_WARPS;
            if (t >= t1) break;
            if (t == pos) {  // the row appended in step 1
                load_raw<DPL>(kb + (size_t)t * HD, kr[i]);
                load_raw<DPL>(vb + (size_t)t * HD, vr[i]);
            }
            float kf[DPL], vf[DPL];
            unpack_raw<DPL>(kr[i], kf);
            unpack_raw<DPL>(vr[i], vf);
            float s[G];
#pragma unroll
            for (int g = 0; g < G; ++g) {
                float d = 0.f;
#pragma unroll
                for (int j = 0; j < DPL; ++j) d = fmaf(qf[g][j], kf[j], d);
                s[g] = d;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1)
#pragma unroll
                for (int g = 0; g < G; ++g) s[g] += __shfl_xor_sync(0xffffffffu, s[g], o);
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float sc = s[g] * inv_sqrt;
                const float mn = fmaxf(m[g], sc);
                const float corr = expf(m[g] - mn), p = expf(sc - mn);
                l[g] = l[g] * corr + p;
#pragma unroll
                for (int j = 0; j < DPL; ++j) acc[g][j] = fmaf(acc[g][j], corr, p * vf[j]);
                m[g] = mn;
            }
        }
    }

    // 3. merge the warps (weights computed once per (warp, head)); the chunk's partial
#pragma unroll
    for (int g = 0; g < G; ++g) {
#pragma unroll
        for (int j = 0; j < DPL; ++j) s_acc[((size_t)warp * G + g) * HD + lane * DPL + j] = acc[g][j];
        if (lane == 0) {
            s_m[warp * G + g] = m[g];
            s_l[warp * G + g] = l[g];
        }
    }
    __syncthreads();
    if (threadIdx.x < G) {
        const int g = threadIdx.x;
        float M = -INFINITY;
        for (int w = 0; w < ATTN_WARPS; ++w) M = fmaxf(M, s_m[w * G + g]);
        float L = 0.f;
        for (int w = 0; w < ATTN_WARPS; ++w) {
            const float mw = s_m[w * G + g];
            const float f = mw == -INFINITY ? 0.f : expf(mw - M);  // a warp without tokens weighs 0
            s_f[w * G + g] = f;
            L = fmaf(s_l[w * G + g], f, L);
        }
        s_L[g] = L;
        const size_t ph = (size_t)(kvh * G + g) * nch + c;
        a.pm[ph] = M;
        a.pl[ph] = L;
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < G * HD; idx += ATTN_WARPS * 32) {
        const int g = idx / HD, d = idx % HD;
        float A = 0.f;
#pragma unroll
        for (int w = 0; w < ATTN_WARPS; ++w) A = fmaf(s_acc[((size_t)w * G + g) * HD + d], s_f[w * G + g], A);
        a.pacc[((size_t)(kvh * G + g) * nch + c) * HD + d] = A;
    }
}

constexpr int MERGE_WARPS = 4;

// Part 2: merge the chunks of q head blockIdx.x, dims [32 * blockIdx.y, + 32):
// warp w takes chunks w, w + 4, ..., every one of its loads in flight at
// once; out = half(acc / sum), then the sigmoid output gate when present
// (attention.metal:1005-1017).
template <int MAXC>
__global__ void __launch_bounds__(MERGE_WARPS * 32) attn_merge_kernel(const AttnArgs a, int hd) {
    __shared__ float s_a[MERGE_WARPS][32];
    __shared__ float s_sum[MERGE_WARPS];
    pdl_wait();
    pdl_launch_dependents();
    const int h = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int d = blockIdx.y * 32 + lane;
    const int nch = a.nch;
    const float* m = a.pm + (size_t)h * nch;
    const float* l = a.pl + (size_t)h * nch;
    // one round trip: the warp's partials, their maxima and sums, and (lanes)
    // every chunk's maximum for the global one (nch <= 160 chunks)
    float v[MAXC], mk[MAXC], lk[MAXC];
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
        const int k = warp + i * MERGE_WARPS;
        v[i] = (k < nch && d < hd) ? a.pacc[((size_t)h * nch + k) * hd + d] : 0.f;
        mk[i] = k < nch ? m[k] : -INFINITY;
        lk[i] = k < nch ? l[k] : 0.f;
    }
    float mm = -INFINITY;
#pragma unroll
    for (int r = 0; r < 5; ++r)
        if (lane + 32 * r < nch) mm = fmaxf(mm, m[lane + 32 * r]);
    const float M = warp_max(mm);
    float L = 0.f, A = 0.f;
    float f[MAXC];
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
        f[i] = mk[i] == -INFINITY ? 0.f : expf(mk[i] - M);
        L = fmaf(lk[i], f[i], L);
    }
#pragma unroll
    for (int i = 0; i < MAXC; ++i) A = fmaf(v[i], f[i], A);
    s_a[warp][lane] = A;
    if (lane == 0) s_sum[warp] = L;
    __syncthreads();
    if (warp != 0 || d >= hd) return;
    float At = 0.f, Lt = 0.f;
#pragma unroll
    for (int w = 0; w < MERGE_WARPS; ++w) {
        At += s_a[w][lane];
        Lt += s_sum[w];
    }
    float o = __half2float(__float2half(At * (Lt > 0.f ? 1.f / Lt : 0.f)));
    if (a.gate) {
        const int qstride = 2 * hd;
        const float gv = __half2float(a.qkv[(size_t)h * qstride + hd + d]);
        o = o * (1.f / (1.f + expf(-gv)));
    }
    a.out[(size_t)h * hd + d] = __float2half(o);
}

// ---- GatedDeltaNet (linear attention) layer ------------------------------------------
// Restates kandiga/metal/attention.metal:1055-1370 as dispatched by
// kandiga/metal/full_forward_lg.m:1361-1508 (conv buffer update, conv1d + SiLU,
// split q|k|v, per-head RMSNorm of q and k without weight, q * 1/kd and
// k * 1/sqrt(kd), gated delta state update, RMSNormGated, out_proj).

// Conv ring buffer [channel][ks]: shift left, append this token's projection
// (conv1d_buffer_update), then silu(sum_k buf * w) -> fp16 (depthwise_conv1d_silu).
__global__ void gdn_conv_kernel(const __half* __restrict__ proj, __half* __restrict__ state,
                                const float* __restrict__ w, int conv_dim, int ks, __half* __restrict__ out) {
    pdl_wait();
    pdl_launch_dependents();
    const int ch = blockIdx.x * blockDim.x + threadIdx.x;
    if (ch >= conv_dim) return;
    __half* st = state + (size_t)ch * ks;
    float acc = 0.f;
    for (int k = 0; k < ks; ++k) {
        const __half v = k + 1 < ks ? st[k + 1] : proj[ch];
        st[k] = v;
        acc = fmaf(__half2float(v), w[(size_t)ch * ks + k], acc);
    }
    out[ch] = __float2half(acc / (1.f + expf(-acc)));
}

// One CTA per value head hv (8 warps): q and k of key head hv / (nv / nk)
// normalised and scaled in shared memory, the decay g = exp(-exp(A_log) *
// softplus(a + dt_bias)) and beta = sigmoid(b); then per value row dv (lane l
// owning key dims [l*KPL, l*KPL + KPL), 64 / KPL rows in flight per warp): S *= g;
// delta = (v - S.k) * beta; S += delta k; o = S.q (attention.metal:1108-1178,
// state fp32 [nv][vd][kd]).  The head's o rows, rounded to fp16, then go
// through RMSNormGated in the same CTA: half(silu(z) * (o * rsqrt(mean(o^2) +
// eps) * w)) (rmsnorm_gated_kernel, attention.metal:1197-1260).
template <int KPL>
__global__ void __launch_bounds__(256) gdn_state_kernel(const __half* __restrict__ conv, const __half* __restrict__ proj,
                                                        const float* __restrict__ a_log,
                                                        const float* __restrict__ dt_bias,
                                                        const float* __restrict__ gnorm, float* __restrict__ state,
                                                        int nk, int nv, int vd, int conv_dim, int vtot, float eps,
                                                        __half* __restrict__ out) {
    constexpr int KD = 32 * KPL;
    constexpr int RB = 64 / KPL;  // rows in flight per warp (16 at kd 128: a warp's rows in one batch)
    extern __shared__ float so[];  // [vd] o rows of this head
    __shared__ float sq[KD], sk[KD];
    __shared__ float s_g, s_beta;
    __shared__ float red[32];
    pdl_wait();
    pdl_launch_dependents();
    const int hv = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int hk = hv / (nv / nk);
    if (warp < 2) {  // warp 0: q, warp 1: k -- rmsnorm_per_head_no_weight, then the scale, each to fp16
        const __half* src = conv + (size_t)warp * nk * KD + (size_t)hk * KD;
        float v[KPL], ss = 0.f;
#pragma unroll
        for (int j = 0; j < KPL; ++j) {
            v[j] = __half2float(src[lane * KPL + j]);
            ss += v[j] * v[j];
        }
        const float sc = 1.f / sqrtf(warp_sum(ss) / (float)KD + eps);
        const float inv = 1.f / sqrtf((float)KD);
        const float mul = warp == 0 ? inv * inv : inv;
        float* dst = warp == 0 ? sq : sk;
#pragma unroll
        for (int j = 0; j < KPL; ++j)
            dst[lane * KPL + j] = __half2float(__float2half(__half2float(__float2half(v[j] * sc)) * mul));
    } else if (threadIdx.x == 64) {
        const float av = __half2float(proj[conv_dim + vtot + nv + hv]);  // a follows b in the projection
        const float bv = __half2float(proj[conv_dim + vtot + hv]);
        const float sp = logf(1.f + expf(av + dt_bias[hv]));
        s_g = expf(-expf(a_log[hv]) * sp);
        s_beta = 1.f / (1.f + expf(-bv));
    }
    __syncthreads();
    const float g = s_g, beta = s_beta;
    float kf[KPL], qf[KPL];
#pragma unroll
    for (int j = 0; j < KPL; ++j) {
        kf[j] = sk[lane * KPL + j];
        qf[j] = sq[lane * KPL + j];
    }
    const __half* vsrc = conv + (size_t)2 * nk * KD + (size_t)hv * vd;
    for (int r0 = warp * RB; r0 < vd; r0 += 8 * RB) {
        float sv[RB][KPL], kv[RB];
#pragma unroll
        for (int b = 0; b < RB; ++b) {
            const int dv = r0 + b;
            const float* srow = state + ((size_t)hv * vd + (dv < vd ? dv : 0)) * KD + lane * KPL;
#pragma unroll
            for (int j = 0; j < KPL; ++j) sv[b][j] = dv < vd ? srow[j] : 0.f;
        }
#pragma unroll
        for (int b = 0; b < RB; ++b) {
            kv[b] = 0.f;
#pragma unroll
            for (int j = 0; j < KPL; ++j) {
                sv[b][j] *= g;
                kv[b] = fmaf(sv[b][j], kf[j], kv[b]);
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int b = 0; b < RB; ++b) kv[b] += __shfl_xor_sync(0xffffffffu, kv[b], o);
        float ov[RB];
#pragma unroll
        for (int b = 0; b < RB; ++b) {
            const int dv = r0 + b;
            const float delta = ((dv < vd ? __half2float(vsrc[dv]) : 0.f) - kv[b]) * beta;
            ov[b] = 0.f;
#pragma unroll
            for (int j = 0; j < KPL; ++j) {
                sv[b][j] = fmaf(delta, kf[j], sv[b][j]);
                ov[b] = fmaf(sv[b][j], qf[j], ov[b]);
            }
            if (dv < vd) {
                float* srow = state + ((size_t)hv * vd + dv) * KD + lane * KPL;
#pragma unroll
                for (int j = 0; j < KPL; ++j) srow[j] = sv[b][j];
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int b = 0; b < RB; ++b) ov[b] += __shfl_xor_sync(0xffffffffu, ov[b], o);
        if (lane == 0)
#pragma unroll
            for (int b = 0; b < RB; ++b)
                if (r0 + b < vd) so[r0 + b] = __half2float(__float2half(ov[b]));
    }
    __syncthreads();
    // RMSNormGated over the head's vd outputs
    float ss = 0.f;
    for (int d = threadIdx.x; d < vd; d += blockDim.x) ss += so[d] * so[d];
    const float sc = 1.f / sqrtf(block_sum(ss, red) / (float)vd + eps);
    for (int d = threadIdx.x; d < vd; d += blockDim.x) {
        const float normed = so[d] * sc * gnorm[d];
        const float z = __half2float(proj[conv_dim + (size_t)hv * vd + d]);
        out[(size_t)hv * vd + d] = __float2half((z / (1.f + expf(-z))) * normed);
    }
}

// float tensors of any 16/32-bit float type -> fp32 (conv weights, A_log, dt_bias, norm)
__global__ void to_f32_kernel(const void* __restrict__ src, int dtype, size_t n, float* __restrict__ dst) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        dst[i] = load_as_float(src, dtype, i);
}

// norm weights of any 16/32-bit float type -> fp16 (the GEMV prologue's dtype)
__global__ void to_f16_kernel(const void* __restrict__ src, int dtype, size_t n, __half* __restrict__ dst) {
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        dst[i] = __float2half(load_as_float(src, dtype, i));
}

// ---- host engine ------------------------------------------------------------------------

struct Weight {
    void* p = nullptr;
    size_t bytes = 0;
    std::vector<int64_t> shape;
    int dtype = -1;  // ABI code: 0 fp16, 1 bf16, 2 fp32, 3 packed uint32
};

struct Layer {
    bool linear = false;  // GatedDeltaNet
    kq_qmat* qkv = nullptr;   // attention: q|k|v; GatedDeltaNet: q|k|v|z|b|a
    kq_qmat* o = nullptr;     // o_proj / out_proj
    float* conv_w = nullptr;  // [conv_dim][conv_k]
    float* a_log = nullptr;   // [nv]
    float* dt_bias = nullptr; // [nv]
    float* gnorm = nullptr;   // [vd]
    __half* conv_state = nullptr;  // [conv_dim][conv_k]
    float* state = nullptr;        // [nv][vd][kd]
    kq_qmat* gate_up = nullptr;
    kq_qmat* down = nullptr;
    __half* in_norm = nullptr;
    __half* post_norm = nullptr;
    __half* q_norm = nullptr;
    __half* k_norm = nullptr;
    __half* kc = nullptr;
    __half* vc = nullptr;
    int gate = 0;
};

struct Engine {
    Cfg c;
    std::string dir;
    std::map<std::string, Weight> w;
    std::vector<Layer> L;
    std::vector<void*> allocs;
    std::vector<kq_qmat*> mats;
    bool built = false;
    int debug = 0;
    cudaStream_t s = nullptr;
    cudaGraphExec_t g_body = nullptr, g_head = nullptr;
    // embedding
    const void* emb_w = nullptr;
    const void* emb_s = nullptr;
    const void* emb_b = nullptr;
    int emb_kind = 0, emb_bits = 0, emb_sb = KQ_DT_BF16;
    kq_qmat* lm = nullptr;
    __half* final_norm = nullptr;
    // activations
    __half *h = nullptr, *qkv = nullptr, *attn = nullptr, *act = nullptr;
    float2* rope = nullptr;       // RoPE (cos, sin) of the current position
    float *logits = nullptr, *pm = nullptr, *pl = nullptr, *pacc = nullptr;
    int* dev_i = nullptr;         // token, position, kv length
    uint32_t* status = nullptr;
    int* host_i = nullptr;        // pinned staging of dev_i
    float* host_logits = nullptr; // pinned
    uint32_t* host_status = nullptr;
    int nchunk = 0;
    int position = 0;
    // GatedDeltaNet activations
    __half *lproj = nullptr, *lconv = nullptr, *lnorm = nullptr;
    // MoE MLP: the MoE block engine over the BKEX files, hidden state ping-pong
    void* moe = nullptr;
    __half* h2 = nullptr;
    __half* hfinal = nullptr;  // buffer holding the last layer's output
    uint32_t* host_moe_status = nullptr;
};

static void err(const char* what) { fprintf(stderr, "[kandiga] ERROR: bakan_full: %s\n", what); }

template <typename T>
static T* dalloc(Engine* e, size_t n) {
    void* p = nullptr;
    if (cudaMalloc(&p, n * sizeof(T) + 16) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    e->allocs.push_back(p);
    cudaMemset(p, 0, n * sizeof(T) + 16);
    return static_cast<T*>(p);
}

static bool json_num(const std::string& js, const char* key, double* out) {
    const std::string k = std::string("\"") + key + "\"";
    size_t pos = 0;
    while ((pos = js.find(k, pos)) != std::string::npos) {
        size_t c = pos + k.size();
        while (c < js.size() && isspace((unsigned char)js[c])) ++c;
        if (c < js.size() && js[c] == ':') {
            ++c;
            while (c < js.size() && isspace((unsigned char)js[c])) ++c;
            char* end = nullptr;
            const double v = strtod(js.c_str() + c, &end);
            if (end != js.c_str() + c) {
                *out = v;
                return true;
            }
        }
        pos = c;
    }
    return false;
}

static int jint(const std::string& js, const char* key, int dflt) {
    double v;
    return json_num(js, key, &v) ? (int)v : dflt;
}

// "layer_types": [...] strings -> 1 for "linear_attention"; false if absent
static bool json_layer_types(const std::string& js, int n, std::vector<char>* out) {
    size_t p = js.find("\"layer_types\"");
    if (p == std::string::npos) return false;
    p = js.find('[', p);
    const size_t q = js.find(']', p);
    if (p == std::string::npos || q == std::string::npos) return false;
    out->clear();
    size_t i = p;
    while ((i = js.find('"', i + 1)) != std::string::npos && i < q) {
        const size_t j = js.find('"', i + 1);
        if (j == std::string::npos || j > q) break;
        out->push_back(js.compare(i + 1, j - i - 1, "linear_attention") == 0 ? 1 : 0);
        i = j;
    }
    out->resize(n, 0);
    return true;
}

static bool parse_cfg(const std::string& js, int num_layers, Cfg* c) {
    c->hidden = jint(js, "hidden_size", 0);
    c->inter = jint(js, "intermediate_size", 0);
    c->layers = jint(js, "num_hidden_layers", num_layers);
    if (num_layers > 0 && num_layers < c->layers) c->layers = num_layers;
    c->lnk = jint(js, "linear_num_key_heads", 0);
    c->lnv = jint(js, "linear_num_value_heads", 0);
    c->lkd = jint(js, "linear_key_head_dim", 0);
    c->lvd = jint(js, "linear_value_head_dim", 0);
    c->conv_k = jint(js, "linear_conv_kernel_dim", 4);
    c->num_experts = jint(js, "num_experts", 0);
    if (c->layers > 0 && !json_layer_types(js, c->layers, &c->linear)) {
        const int every = c->lnv > 0 ? jint(js, "full_attention_interval", 4) : 1;
        c->linear.assign(c->layers, 0);
        for (int l = 0; l < c->layers; ++l) c->linear[l] = every > 1 && (l + 1) % every != 0;
    }
    c->nq = jint(js, "num_attention_heads", 0);
    c->nkv = jint(js, "num_key_value_heads", c->nq);
    c->hd = jint(js, "head_dim", c->nq ? c->hidden / c->nq : 0);
    c->vocab = jint(js, "vocab_size", 0);
    c->max_seq = jint(js, "max_cache_len", 4096);
    c->group = jint(js, "group_size", 64);
    double v;
    if (json_num(js, "rms_norm_eps", &v)) c->eps = (float)v;
    if (json_num(js, "rope_theta", &v)) c->theta = (float)v;
    double prf = 1.0;
    json_num(js, "partial_rotary_factor", &prf);
    c->rope_dim = (int)(c->hd * prf);
    c->rope_dim -= c->rope_dim % 2;
    if (js.find("\"gelu") != std::string::npos) c->act = KQ_ACT_GELU_TANH;
    bool any_lin = false;
    for (char x : c->linear) any_lin = any_lin || x;
    const bool lin_ok = !any_lin || (c->lnk > 0 && c->lnv > 0 && c->lnv % c->lnk == 0 && c->lkd > 0 && c->lvd > 0 &&
                                     c->conv_k > 0 && c->conv_k <= 8);
    return c->hidden > 0 && (c->inter > 0 || c->num_experts > 0) && c->layers > 0 && c->nq > 0 && c->nkv > 0 &&
           c->nq % c->nkv == 0 && c->hd > 0 && c->vocab > 0 && c->max_seq > 0 && lin_ok;
}

static const Weight* find(Engine* e, const std::string& name) {
    auto it = e->w.find(name);
    return it == e->w.end() ? nullptr : &it->second;
}

static std::string lname(int l, const char* suffix) { return "layers." + std::to_string(l) + "." + suffix; }

// fp16 copy of a 1-D float tensor (norm weight); nullptr if absent or wrong size
static __half* norm_f16(Engine* e, const std::string& name, int n, bool required, bool* ok) {
    const Weight* wt = find(e, name);
    if (!wt) {
        if (required) {
            fprintf(stderr, "[kandiga] ERROR: bakan_full: %s not set\n", name.c_str());
            *ok = false;
        }
        return nullptr;
    }
    const int dt = wt->dtype == 0 ? KQ_DT_F16 : wt->dtype == 1 ? KQ_DT_BF16 : wt->dtype == 2 ? KQ_DT_F32 : -1;
    const size_t es = dt == KQ_DT_F32 ? 4 : 2;
    if (dt < 0 || wt->bytes != (size_t)n * es) {
        fprintf(stderr, "[kandiga] ERROR: bakan_full: %s has %zu bytes, expected %d values\n", name.c_str(), wt->bytes,
                n);
        *ok = false;
        return nullptr;
    }
    __half* d = dalloc<__half>(e, n);
    if (!d) {
        *ok = false;
        return nullptr;
    }
    to_f16_kernel<<<(n + 255) / 256, 256, 0, e->s>>>(wt->p, dt, (size_t)n, d);
    return d;
}

// fp32 copy of a float tensor of n values (conv weights, A_log, dt_bias, norms)
static float* f32_of(Engine* e, const std::string& name, size_t n, bool* ok) {
    const Weight* wt = find(e, name);
    const int dt = !wt ? -1 : wt->dtype == 0 ? KQ_DT_F16 : wt->dtype == 1 ? KQ_DT_BF16 : wt->dtype == 2 ? KQ_DT_F32 : -1;
    if (dt < 0 || wt->bytes != n * (dt == KQ_DT_F32 ? 4 : 2)) {
        fprintf(stderr, "[kandiga] ERROR: bakan_full: %s not set as %zu float values\n", name.c_str(), n);
        *ok = false;
        return nullptr;
    }
    float* d = dalloc<float>(e, n);
    if (!d) {
        *ok = false;
        return nullptr;
    }
    to_f32_kernel<<<(unsigned)std::min<size_t>((n + 255) / 256, 1024), 256, 0, e->s>>>(wt->p, dt, n, d);
    return d;
}

// A quantized linear [rows][cols] from name.{weight,scales,biases}; with
// `parts`, the named matrices are stacked along rows (q|k|v).
static kq_qmat* qlinear(Engine* e, const std::vector<std::string>& parts, int cols, int* rows_out, bool* ok,
                        const std::string& pair_b = "") {
    int rows = 0, bits = 0, sbdt = -1;
    for (const auto& pn : parts) {
        const Weight* wt = find(e, pn + ".weight");
        const Weight* sc = find(e, pn + ".scales");
        const Weight* bi = find(e, pn + ".biases");
        if (!wt || !sc || !bi || wt->shape.size() != 2 || sc->shape.size() != 2) {
            fprintf(stderr, "[kandiga] ERROR: bakan_full: quantized linear %s not set\n", pn.c_str());
            *ok = false;
            return nullptr;
        }
        const int r = (int)wt->shape[0];
        const int b = (int)(wt->shape[1] * 32 / cols);
        const int sd = sc->dtype == 0 ? KQ_DT_F16 : KQ_DT_BF16;
        if (sc->shape[1] * e->c.group != cols || sc->shape[0] != r || (bits && b != bits) ||
            (sbdt >= 0 && sd != sbdt) || (b != 3 && b != 4) || (sc->dtype != 0 && sc->dtype != 1)) {
            fprintf(stderr, "[kandiga] ERROR: bakan_full: %s: shape does not match %d columns at 3/4 bits\n",
                    pn.c_str(), cols);
            *ok = false;
            return nullptr;
        }
        rows += r;
        bits = b;
        sbdt = sd;
    }
    auto stacked = [&](const char* comp, size_t* bytes_out) -> const void* {
        if (parts.size() == 1) {
            const Weight* wt = find(e, parts[0] + comp);
            *bytes_out = wt->bytes;
            return wt->p;
        }
        size_t total = 0;
        for (const auto& pn : parts) total += find(e, pn + comp)->bytes;
        uint8_t* d = dalloc<uint8_t>(e, total);
        if (!d) return nullptr;
        size_t off = 0;
        for (const auto& pn : parts) {
            const Weight* wt = find(e, pn + comp);
            cudaMemcpyAsync(d + off, wt->p, wt->bytes, cudaMemcpyDeviceToDevice, e->s);
            off += wt->bytes;
        }
        *bytes_out = total;
        return d;
    };
    size_t wb, sb, bb;
    kq_mlx_matrix a{};
    a.weight = stacked(".weight", &wb);
    a.scales = stacked(".scales", &sb);
    a.biases = stacked(".biases", &bb);
    if (!a.weight || !a.scales || !a.biases) {
        *ok = false;
        return nullptr;
    }
    kq_mlx_matrix bm{};
    const bool pair = !pair_b.empty();
    if (pair) {
        const Weight* wt = find(e, pair_b + ".weight");
        const Weight* sc = find(e, pair_b + ".scales");
        const Weight* bi = find(e, pair_b + ".biases");
        if (!wt || !sc || !bi || wt->bytes != wb || sc->bytes != sb) {
            fprintf(stderr, "[kandiga] ERROR: bakan_full: %s missing or not shaped like its pair\n", pair_b.c_str());
            *ok = false;
            return nullptr;
        }
        bm.weight = wt->p;
        bm.scales = sc->p;
        bm.biases = bi->p;
    }
    kq_qmat* m = nullptr;
    if (kq_qmat_create(rows, cols, bits, sbdt, pair ? 1 : 0, &m) != KQ_OK) {
        *ok = false;
        return nullptr;
    }
    e->mats.push_back(m);
    if (kq_qmat_load_mlx(m, &a, pair ? &bm : nullptr, e->s) != KQ_OK) {
        *ok = false;
        return nullptr;
    }
    if (rows_out) *rows_out = rows;
    return m;
}

// Launch as a programmatic dependent of the previous kernel on the stream:
// the kernel starts with griddepcontrol.wait, so it may be scheduled while
// its predecessor drains.
template <typename... KArgs, typename... Args>
static cudaError_t pdl_launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

static cudaError_t smem_opt_in(const void* fn, size_t bytes) {
    return bytes > 48 * 1024 ? raise_smem_limit(fn, bytes) : cudaSuccess;
}

// launch = false: only raise the kernel's shared-memory limit (done once,
// before the step is captured)
template <int DPL, int G>
static cudaError_t launch_attn(Engine* e, const Layer* ly, bool launch) {
    constexpr int HD = 32 * DPL;
    const size_t smem = ((size_t)G * HD + HD + (size_t)ATTN_WARPS * G * HD + 3 * ATTN_WARPS * G + G) * sizeof(float);
    if (!launch) return smem_opt_in((const void*)attn_chunk_kernel<DPL, G>, smem);
    AttnArgs a;
    a.qkv = e->qkv;
    a.q_norm = ly->q_norm;
    a.k_norm = ly->k_norm;
    a.kc = ly->kc;
    a.vc = ly->vc;
    a.dev_i = e->dev_i;
    a.rope = e->rope;
    a.pm = e->pm;
    a.pl = e->pl;
    a.pacc = e->pacc;
    a.out = e->attn;
    a.status = e->status;
    a.nq = e->c.nq;
    a.nkv = e->c.nkv;
    a.max_seq = e->c.max_seq;
    a.gate = ly->gate;
    a.rope_dim = e->c.rope_dim;
    a.nch = e->nchunk;
    a.eps = e->c.eps;
    cudaError_t r = pdl_launch(attn_chunk_kernel<DPL, G>, dim3(e->c.nkv, e->nchunk), dim3(ATTN_WARPS * 32), smem,
                               e->s, a);
    if (r != cudaSuccess) return r;
    const dim3 mg(e->c.nq, (HD + 31) / 32);
    const int per_warp = (e->nchunk + MERGE_WARPS - 1) / MERGE_WARPS;  // nchunk <= 148 / 1 kv head
    if (per_warp <= 4) return pdl_launch(attn_merge_kernel<4>, mg, dim3(MERGE_WARPS * 32), 0, e->s, a, HD);
    if (per_warp <= 10) return pdl_launch(attn_merge_kernel<10>, mg, dim3(MERGE_WARPS * 32), 0, e->s, a, HD);
    if (per_warp <= 19) return pdl_launch(attn_merge_kernel<19>, mg, dim3(MERGE_WARPS * 32), 0, e->s, a, HD);
    return pdl_launch(attn_merge_kernel<37>, mg, dim3(MERGE_WARPS * 32), 0, e->s, a, HD);
}

static cudaError_t attention(Engine* e, const Layer* ly, bool launch = true) {
    const int G = e->c.nq / e->c.nkv;
    const int hd = e->c.hd;
#define KQ_ATTN_CASE(D, GG) \
    if (hd == 32 * D && G == GG) return launch_attn<D, GG>(e, ly, launch);
    KQ_ATTN_CASE(8, 1) KQ_ATTN_CASE(8, 2) KQ_ATTN_CASE(8, 4) KQ_ATTN_CASE(8, 8)
    KQ_ATTN_CASE(4, 1) KQ_ATTN_CASE(4, 2) KQ_ATTN_CASE(4, 4) KQ_ATTN_CASE(4, 8)
    KQ_ATTN_CASE(2, 1) KQ_ATTN_CASE(2, 2) KQ_ATTN_CASE(2, 4) KQ_ATTN_CASE(2, 8)
#undef KQ_ATTN_CASE
    return cudaErrorInvalidValue;
}

static bool gqa_supported(const Cfg& c) {
    const int G = c.nq / c.nkv;
    return (c.hd == 64 || c.hd == 128 || c.hd == 256) && (G == 1 || G == 2 || G == 4 || G == 8);
}

template <int KPL>
static cudaError_t launch_gdn_state(Engine* e, const Layer& ly) {
    const Cfg& c = e->c;
    return pdl_launch(gdn_state_kernel<KPL>, dim3(c.lnv), dim3(256), (size_t)c.lvd * sizeof(float), e->s,
                      (const __half*)e->lconv, (const __half*)e->lproj, (const float*)ly.a_log,
                      (const float*)ly.dt_bias, (const float*)ly.gnorm, ly.state, c.lnk, c.lnv, c.lvd, c.conv_dim(),
                      c.lnv * c.lvd, c.eps, e->lnorm);
}

// GatedDeltaNet token mixer of one layer on the hidden state `x` (in place).
static int enqueue_linear(Engine* e, const Layer& ly, __half* x) {
    const Cfg& c = e->c;
    int rc = dense_gemv_res(ly.qkv, x, KQ_DT_F16, 1, ly.in_norm, c.eps, KQ_ACT_SILU, e->lproj, KQ_DT_F16, nullptr, e->s);
    if (rc) return rc;
    const int cdim = c.conv_dim();
    if (pdl_launch(gdn_conv_kernel, dim3((cdim + 255) / 256), dim3(256), 0, e->s, (const __half*)e->lproj,
                   ly.conv_state, (const float*)ly.conv_w, cdim, c.conv_k, e->lconv) != cudaSuccess)
        return KQ_ERR_CUDA;
    cudaError_t ce = c.lkd == 64 ? launch_gdn_state<2>(e, ly)
                     : c.lkd == 128 ? launch_gdn_state<4>(e, ly)
                                    : launch_gdn_state<8>(e, ly);
    if (ce != cudaSuccess) return KQ_ERR_CUDA;
    return dense_gemv_res(ly.o, e->lnorm, KQ_DT_F16, 1, nullptr, c.eps, KQ_ACT_SILU, x, KQ_DT_F16, x, e->s);
}

// Attention token mixer of one layer on the hidden state `x` (in place).
static int enqueue_attention(Engine* e, const Layer& ly, __half* x) {
    const Cfg& c = e->c;
    int rc = dense_gemv_res(ly.qkv, x, KQ_DT_F16, 1, ly.in_norm, c.eps, KQ_ACT_SILU, e->qkv, KQ_DT_F16, nullptr, e->s);
    if (rc) return rc;
    if (attention(e, &ly) != cudaSuccess) return KQ_ERR_CUDA;
    return dense_gemv_res(ly.o, e->attn, KQ_DT_F16, 1, nullptr, c.eps, KQ_ACT_SILU, x, KQ_DT_F16, x, e->s);
}

// Layers, enqueued on e->s; the hidden state ping-pongs between h and h2 across
// MoE blocks (whose output cannot alias their input).
static int enqueue_body(Engine* e) {
    const Cfg& c = e->c;
    embed_kernel<<<(c.hidden + 255) / 256, 256, 0, e->s>>>(
        e->dev_i, c.vocab, static_cast<const uint8_t*>(e->emb_w), static_cast<const uint16_t*>(e->emb_s),
        static_cast<const uint16_t*>(e->emb_b), e->emb_bits, e->emb_sb, e->emb_kind, c.hidden, c.group, e->h,
        c.rope_dim, c.theta, e->rope, e->status);
    __half* cur = e->h;
    __half* other = e->h2;
    for (int l = 0; l < c.layers; ++l) {
        const Layer& ly = e->L[l];
        int rc = ly.linear ? enqueue_linear(e, ly, cur) : enqueue_attention(e, ly, cur);
        if (rc) {
            fprintf(stderr, "[kandiga] ERROR: bakan_full: layer %d token mixer: code %d (%s)\n", l, rc,
                    cudaGetErrorString(cudaGetLastError()));
            return rc;
        }
        if (e->moe) {
            rc = moe_block_enqueue(e->moe, l, cur, other, e->s);
            if (rc != KQ_OK) {
                fprintf(stderr, "[kandiga] ERROR: bakan_full: layer %d MoE block: code %d (%s)\n", l, rc,
                        cudaGetErrorString(cudaGetLastError()));
                return KQ_ERR_CUDA;
            }
            std::swap(cur, other);
        } else {
            rc = dense_gemv_res(ly.gate_up, cur, KQ_DT_F16, 1, ly.post_norm, c.eps, c.act, e->act, KQ_DT_F16, nullptr,
                                e->s);
            if (rc) return rc;
            rc = dense_gemv_res(ly.down, e->act, KQ_DT_F16, 1, nullptr, c.eps, KQ_ACT_SILU, cur, KQ_DT_F16, cur, e->s);
            if (rc) return rc;
        }
    }
    e->hfinal = cur;
    return cudaGetLastError() == cudaSuccess ? KQ_OK : KQ_ERR_CUDA;
}

static int enqueue_head(Engine* e) {
    return dense_gemv_res(e->lm, e->hfinal, KQ_DT_F16, 1, e->final_norm, e->c.eps, KQ_ACT_SILU, e->logits, KQ_DT_F32,
                          nullptr, e->s);
}

static int capture(Engine* e, int (*fn)(Engine*), cudaGraphExec_t* out) {
    cudaGraph_t g = nullptr;
    if (cudaStreamBeginCapture(e->s, cudaStreamCaptureModeThreadLocal) != cudaSuccess) return KQ_ERR_CUDA;
    const int rc = fn(e);
    const cudaError_t ce = cudaStreamEndCapture(e->s, &g);
    if (rc || ce != cudaSuccess) {
        fprintf(stderr, "[kandiga] ERROR: bakan_full: capture: enqueue code %d, end capture: %s\n", rc,
                cudaGetErrorString(ce));
        if (g) cudaGraphDestroy(g);
        cudaGetLastError();
        return rc ? rc : KQ_ERR_CUDA;
    }
    const cudaError_t ie = cudaGraphInstantiate(out, g, 0);
    cudaGraphDestroy(g);
    return ie == cudaSuccess ? KQ_OK : KQ_ERR_CUDA;
}

static int build(Engine* e) {
    Cfg& c = e->c;
    bool ok = true;
    // embedding
    const Weight* ew = find(e, "embed_tokens.weight");
    if (!ew || ew->shape.size() != 2 || ew->shape[0] != c.vocab) {
        err("embed_tokens.weight not set or not [vocab, ...]");
        return -1;
    }
    e->emb_w = ew->p;
    if (ew->dtype == 3) {
        const Weight* es = find(e, "embed_tokens.scales");
        const Weight* eb = find(e, "embed_tokens.biases");
        if (!es || !eb || (es->dtype != 0 && es->dtype != 1)) {
            err("embed_tokens.scales / biases not set");
            return -1;
        }
        e->emb_kind = 0;
        e->emb_bits = (int)(ew->shape[1] * 32 / c.hidden);
        e->emb_s = es->p;
        e->emb_b = eb->p;
        e->emb_sb = es->dtype == 0 ? KQ_DT_F16 : KQ_DT_BF16;
        if (e->emb_bits < 2 || e->emb_bits > 8 || (size_t)ew->shape[1] * 32 != (size_t)c.hidden * e->emb_bits) {
            err("embed_tokens.weight: unsupported bit width");
            return -1;
        }
    } else if (ew->dtype == 0 || ew->dtype == 1) {
        e->emb_kind = ew->dtype == 0 ? 1 : 2;
        if (ew->shape[1] != c.hidden) {
            err("embed_tokens.weight: width != hidden_size");
            return -1;
        }
    } else {
        err("embed_tokens.weight: unsupported dtype");
        return -1;
    }
    e->final_norm = norm_f16(e, "norm.weight", c.hidden, true, &ok);
    if (find(e, "lm_head.weight"))
        e->lm = qlinear(e, {"lm_head"}, c.hidden, nullptr, &ok);
    else if (e->emb_kind == 0)  // tied embeddings
        e->lm = qlinear(e, {"embed_tokens"}, c.hidden, nullptr, &ok);
    else {
        err("lm_head.weight not set and the embedding is not quantized");
        return -1;
    }
    if (!ok) return -1;
    e->L.assign(c.layers, Layer());
    const int qrows = c.nq * c.hd, kvrows = c.nkv * c.hd;
    const int cdim = c.conv_dim(), vtot = c.lnv * c.lvd;
    for (int l = 0; l < c.layers; ++l) {
        Layer& ly = e->L[l];
        ly.linear = c.linear[l] != 0;
        ly.in_norm = norm_f16(e, lname(l, "input_layernorm.weight"), c.hidden, true, &ok);
        if (!e->moe) ly.post_norm = norm_f16(e, lname(l, "post_attention_layernorm.weight"), c.hidden, true, &ok);
        int rows = 0;
        if (ly.linear) {
            if (find(e, lname(l, "linear_attn.combined_proj.weight")))
                ly.qkv = qlinear(e, {lname(l, "linear_attn.combined_proj")}, c.hidden, &rows, &ok);
            else
                ly.qkv = qlinear(e, {lname(l, "linear_attn.in_proj_qkv"), lname(l, "linear_attn.in_proj_z"),
                                     lname(l, "linear_attn.in_proj_b"), lname(l, "linear_attn.in_proj_a")},
                                 c.hidden, &rows, &ok);
            if (!ok) return -1;
            if (rows != c.lin_proj_rows()) {
                fprintf(stderr, "[kandiga] ERROR: bakan_full: layer %d q|k|v|z|b|a has %d rows, expected %d\n", l,
                        rows, c.lin_proj_rows());
                return -1;
            }
            ly.o = qlinear(e, {lname(l, "linear_attn.out_proj")}, vtot, nullptr, &ok);
            ly.conv_w = f32_of(e, lname(l, "linear_attn.conv1d.weight"), (size_t)cdim * c.conv_k, &ok);
            ly.a_log = f32_of(e, lname(l, "linear_attn.A_log"), c.lnv, &ok);
            ly.dt_bias = f32_of(e, lname(l, "linear_attn.dt_bias"), c.lnv, &ok);
            ly.gnorm = f32_of(e, lname(l, "linear_attn.norm.weight"), c.lvd, &ok);
            if (!ok) return -1;
            ly.conv_state = dalloc<__half>(e, (size_t)cdim * c.conv_k);
            ly.state = dalloc<float>(e, (size_t)c.lnv * c.lvd * c.lkd);
            if (!ly.conv_state || !ly.state) {
                err("linear-attention state allocation failed");
                return -1;
            }
        } else {
            ly.q_norm = norm_f16(e, lname(l, "self_attn.q_norm.weight"), c.hd, false, &ok);
            ly.k_norm = norm_f16(e, lname(l, "self_attn.k_norm.weight"), c.hd, false, &ok);
            if (find(e, lname(l, "self_attn.combined_proj.weight")))
                ly.qkv = qlinear(e, {lname(l, "self_attn.combined_proj")}, c.hidden, &rows, &ok);
            else
                ly.qkv = qlinear(e, {lname(l, "self_attn.q_proj"), lname(l, "self_attn.k_proj"),
                                     lname(l, "self_attn.v_proj")},
                                 c.hidden, &rows, &ok);
            if (!ok) return -1;
            if (rows == 2 * qrows + 2 * kvrows)
                ly.gate = 1;  // q_proj carries the output gate, interleaved per head
            else if (rows != qrows + 2 * kvrows) {
                fprintf(stderr, "[kandiga] ERROR: bakan_full: layer %d q|k|v has %d rows\n", l, rows);
                return -1;
            }
            ly.o = qlinear(e, {lname(l, "self_attn.o_proj")}, qrows, nullptr, &ok);
            ly.kc = dalloc<__half>(e, (size_t)c.nkv * c.max_seq * c.hd);
            ly.vc = dalloc<__half>(e, (size_t)c.nkv * c.max_seq * c.hd);
            if (!ly.kc || !ly.vc) {
                err("KV cache allocation failed");
                return -1;
            }
        }
        if (e->moe) {
            if (moe_block_prepare(e->moe, l) != 0) return -1;
        } else {
            ly.gate_up = qlinear(e, {lname(l, "mlp.gate_proj")}, c.hidden, nullptr, &ok, lname(l, "mlp.up_proj"));
            ly.down = qlinear(e, {lname(l, "mlp.down_proj")}, c.inter, nullptr, &ok);
        }
        if (!ok) return -1;
    }
    e->nchunk = (ATTN_CTAS + c.nkv - 1) / c.nkv;  // context chunks per kv head
    e->h = dalloc<__half>(e, c.hidden);
    e->qkv = dalloc<__half>(e, (size_t)2 * qrows + 2 * kvrows);
    e->rope = dalloc<float2>(e, c.rope_dim / 2 + 1);
    e->attn = dalloc<__half>(e, qrows);
    e->act = dalloc<__half>(e, c.inter > 0 ? c.inter : 1);
    e->h2 = dalloc<__half>(e, c.hidden);
    e->lproj = dalloc<__half>(e, (size_t)c.lin_proj_rows() + 1);
    e->lconv = dalloc<__half>(e, (size_t)cdim + 1);
    e->lnorm = dalloc<__half>(e, (size_t)vtot + 1);
    e->logits = dalloc<float>(e, c.vocab);
    e->pm = dalloc<float>(e, (size_t)c.nq * e->nchunk);
    e->pl = dalloc<float>(e, (size_t)c.nq * e->nchunk);
    e->pacc = dalloc<float>(e, (size_t)c.nq * e->nchunk * c.hd);
    e->dev_i = dalloc<int>(e, 4);
    e->status = dalloc<uint32_t>(e, 1);
    if (!e->h || !e->qkv || !e->rope || !e->attn || !e->act || !e->logits || !e->pm || !e->pl || !e->pacc ||
        !e->dev_i || !e->status || !e->h2 || !e->lproj || !e->lconv || !e->lnorm) {
        err("buffer allocation failed");
        return -1;
    }
    if (cudaHostAlloc(reinterpret_cast<void**>(&e->host_i), 4 * sizeof(int), 0) != cudaSuccess ||
        cudaHostAlloc(reinterpret_cast<void**>(&e->host_logits), (size_t)c.vocab * sizeof(float), 0) != cudaSuccess ||
        cudaHostAlloc(reinterpret_cast<void**>(&e->host_status), sizeof(uint32_t), 0) != cudaSuccess ||
        cudaHostAlloc(reinterpret_cast<void**>(&e->host_moe_status), sizeof(uint32_t), 0) != cudaSuccess) {
        cudaGetLastError();
        err("pinned host buffers");
        return -1;
    }
    if (cudaStreamSynchronize(e->s) != cudaSuccess || attention(e, nullptr, false) != cudaSuccess) {
        err("weight setup failed on the device");
        return -1;
    }
    if (capture(e, enqueue_body, &e->g_body) != KQ_OK || capture(e, enqueue_head, &e->g_head) != KQ_OK) {
        err("CUDA graph capture of the decode step failed");
        return -1;
    }
    e->built = true;
    return 0;
}

// One token through the layers (and the head when logits_out != nullptr).
static int step(Engine* e, int token, int position, float* logits_out) {
    if (position < 0 || position >= e->c.max_seq) {
        fprintf(stderr, "[kandiga] ERROR: bakan_full: position %d outside [0, %d)\n", position, e->c.max_seq);
        return -1;
    }
    if (token < 0 || token >= e->c.vocab) {
        fprintf(stderr, "[kandiga] ERROR: bakan_full: token %d outside [0, %d)\n", token, e->c.vocab);
        return -1;
    }
    e->host_i[0] = token;
    e->host_i[1] = position;
    e->host_i[2] = position + 1;
    cudaError_t ce = cudaMemcpyAsync(e->dev_i, e->host_i, 3 * sizeof(int), cudaMemcpyHostToDevice, e->s);
    if (ce == cudaSuccess) ce = cudaGraphLaunch(e->g_body, e->s);
    if (ce == cudaSuccess && logits_out) {
        ce = cudaGraphLaunch(e->g_head, e->s);
        if (ce == cudaSuccess)
            ce = cudaMemcpyAsync(e->host_logits, e->logits, (size_t)e->c.vocab * sizeof(float), cudaMemcpyDeviceToHost,
                                 e->s);
    }
    if (ce == cudaSuccess)
        ce = cudaMemcpyAsync(e->host_status, e->status, sizeof(uint32_t), cudaMemcpyDeviceToHost, e->s);
    *e->host_moe_status = 0;
    if (ce == cudaSuccess && e->moe)
        ce = cudaMemcpyAsync(e->host_moe_status, moe_block_status(e->moe), sizeof(uint32_t), cudaMemcpyDeviceToHost,
                             e->s);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(e->s);
    if (ce != cudaSuccess) {
        fprintf(stderr, "[kandiga] ERROR: bakan_full: %s\n", cudaGetErrorString(ce));
        return -1;
    }
    if (*e->host_status || *e->host_moe_status) {
        fprintf(stderr, "[kandiga] ERROR: bakan_full: device status 0x%x / MoE 0x%x\n", *e->host_status,
                *e->host_moe_status);
        cudaMemsetAsync(e->status, 0, sizeof(uint32_t), e->s);
        if (e->moe) cudaMemsetAsync(moe_block_status(e->moe), 0, sizeof(uint32_t), e->s);
        cudaStreamSynchronize(e->s);
        return -1;
    }
    if (logits_out) memcpy(logits_out, e->host_logits, (size_t)e->c.vocab * sizeof(float));
    e->position = position + 1;
    return 0;
}

// the idx-th layer of one kind (GatedDeltaNet or attention), nullptr if none
static Layer* nth_layer(Engine* e, bool linear, int idx) {
    if (idx < 0) return nullptr;
    for (auto& ly : e->L)
        if (ly.linear == linear && idx-- == 0) return &ly;
    return nullptr;
}

static void destroy(Engine* e) {
    if (!e) return;
    if (e->s) cudaStreamSynchronize(e->s);
    if (e->g_body) cudaGraphExecDestroy(e->g_body);
    if (e->g_head) cudaGraphExecDestroy(e->g_head);
    for (auto* m : e->mats) kq_qmat_destroy(m);
    for (auto& kv : e->w)
        if (kv.second.p) cudaFree(kv.second.p);
    for (void* p : e->allocs) cudaFree(p);
    if (e->host_i) cudaFreeHost(e->host_i);
    if (e->host_logits) cudaFreeHost(e->host_logits);
    if (e->host_status) cudaFreeHost(e->host_status);
    if (e->host_moe_status) cudaFreeHost(e->host_moe_status);
    if (e->moe) bakan_forward_destroy(e->moe);
    if (e->s) cudaStreamDestroy(e->s);
    delete e;
}

static Engine* create(const std::string& json, const char* dir, int num_layers) {
    Engine* e = new (std::nothrow) Engine();
    if (!e) return nullptr;
    if (!parse_cfg(json, num_layers, &e->c)) {
        err("model config lacks hidden_size / intermediate_size / num_attention_heads / head_dim / vocab_size");
        delete e;
        return nullptr;
    }
    if (!gqa_supported(e->c) || e->c.hidden % 64 || e->c.inter % 64 || e->c.rope_dim > e->c.hd ||
        e->c.vocab % 16) {
        err("unsupported shape (head_dim 64/128/256, 1/2/4/8 q heads per kv head, dims multiples of 64, "
            "vocab a multiple of 16)");
        delete e;
        return nullptr;
    }
    bool any_lin = false;
    for (char x : e->c.linear) any_lin = any_lin || x;
    if (any_lin && e->c.lkd != 64 && e->c.lkd != 128 && e->c.lkd != 256) {
        err("linear_key_head_dim must be 64, 128 or 256");
        delete e;
        return nullptr;
    }
    e->dir = dir ? dir : "";
    if (cudaStreamCreateWithFlags(&e->s, cudaStreamNonBlocking) != cudaSuccess) {
        cudaGetLastError();
        delete e;
        return nullptr;
    }
    if (e->c.num_experts > 0) {  // routed experts from packed_dir/layer_XX.bin, as bakan_full_init's argument says
        e->moe = bakan_forward_init(e->dir.c_str(), e->c.layers);
        if (!e->moe || moe_block_hidden(e->moe) != e->c.hidden) {
            err("MoE layers need the BKEX expert files of every layer in packed_expert_dir, hidden_size as the model's");
            destroy(e);
            return nullptr;
        }
        const int top_k = jint(json, "num_experts_per_tok", 8);
        if (kq_forward_set_params(e->moe, top_k, e->c.eps) != KQ_OK) {
            err("num_experts_per_tok outside [1, min(16, experts)]");
            destroy(e);
            return nullptr;
        }
    }
    return e;
}

}  // namespace full
}  // namespace kq

using kq::full::Engine;

extern "C" void* kq_full_init_json(const char* config_json, const char* packed_dir, int num_layers) {
    if (!config_json) return nullptr;
    return kq::full::create(config_json, packed_dir, num_layers);
}

extern "C" void* bakan_full_init(const char* packed_expert_dir, int num_layers) {
    if (!packed_expert_dir) return nullptr;
    const std::string path = std::string(packed_expert_dir) + "/config.json";
    FILE* f = fopen(path.c_str(), "rb");
    if (!f) {
        fprintf(stderr, "[kandiga] ERROR: bakan_full: cannot open %s\n", path.c_str());
        return nullptr;
    }
    std::string js;
    char buf[4096];
    size_t n;
    while ((n = fread(buf, 1, sizeof(buf), f)) > 0) js.append(buf, n);
    fclose(f);
    return kq::full::create(js, packed_expert_dir, num_layers);
}

extern "C" int bakan_full_set_weight(void* engine, const char* name, const void* data, size_t size, int ndim,
                                     const int64_t* shape, int dtype) {
    Engine* e = static_cast<Engine*>(engine);
    if (!e || !name || (!data && size) || ndim < 0 || ndim > 8 || (ndim && !shape)) return -1;
    if (e->built) {
        kq::full::err("set_weight after build");
        return -1;
    }
    if (strstr(name, "vision") || strstr(name, "mtp.")) return 1;  // as full_forward_lg.m:784-785
    if (dtype < 0 || dtype > 3) return -1;
    std::string key(name);
    for (const char* pre : {"language_model.model.", "language_model.", "model."})
        if (key.rfind(pre, 0) == 0) {
            key = key.substr(strlen(pre));
            break;
        }
    if (e->moe) {  // the MoE block's tensors go to the MoE block engine (weight types of bakan_forward.h:35-53)
        const int layer = key.rfind("layers.", 0) == 0 ? atoi(key.c_str() + 7) : -1;
        const size_t dot = key.find('.', 7);
        const std::string rest = dot == std::string::npos ? "" : key.substr(dot + 1);
        static const struct {
            const char* name;
            int wt;
        } kMoe[] = {{"post_attention_layernorm.weight", 0},    {"mlp.gate.weight", 1},
                    {"mlp.gate.scales", 2},                    {"mlp.gate.biases", 3},
                    {"mlp.shared_expert_gate.weight", 4},      {"mlp.shared_expert_gate.scales", 5},
                    {"mlp.shared_expert_gate.biases", 6},      {"mlp.shared_expert.up_proj.weight", 7},
                    {"mlp.shared_expert.up_proj.scales", 8},   {"mlp.shared_expert.up_proj.biases", 9},
                    {"mlp.shared_expert.gate_proj.weight", 10}, {"mlp.shared_expert.gate_proj.scales", 11},
                    {"mlp.shared_expert.gate_proj.biases", 12}, {"mlp.shared_expert.down_proj.weight", 13},
                    {"mlp.shared_expert.down_proj.scales", 14}, {"mlp.shared_expert.down_proj.biases", 15}};
        if (layer >= 0 && (rest.rfind("mlp.switch_mlp.", 0) == 0 || rest.rfind("mlp.experts.", 0) == 0))
            return 1;  // routed experts come from the BKEX files
        for (const auto& m : kMoe) {
            if (layer < 0 || rest != m.name) continue;
            const int fdt = dtype == 0 ? 0 : dtype == 1 ? 2 : dtype == 3 ? 1 : -1;  // bakan_forward dtype codes
            if (fdt < 0) {
                fprintf(stderr, "[kandiga] ERROR: bakan_full: %s must be fp16, bf16 or packed\n", name);
                return -1;
            }
            const int rows = ndim == 2 ? (int)shape[0] : 1;
            const int cols = ndim == 2 ? (int)shape[1] : ndim == 1 ? (int)shape[0] : 0;
            return bakan_forward_set_weight(e->moe, layer, m.wt, data, size, rows, cols, fdt) == 0 ? 0 : -1;
        }
    }
    kq::full::Weight wt;
    wt.shape.assign(shape, shape + ndim);
    wt.dtype = dtype;
    wt.bytes = size;
    if (cudaMalloc(&wt.p, size + 16) != cudaSuccess) {
        cudaGetLastError();
        fprintf(stderr, "[kandiga] ERROR: bakan_full: allocation for '%s' failed (%zu bytes)\n", name, size);
        return -1;
    }
    if (size && cudaMemcpy(wt.p, data, size, cudaMemcpyHostToDevice) != cudaSuccess) {
        cudaFree(wt.p);
        return -1;
    }
    auto it = e->w.find(key);
    if (it != e->w.end()) cudaFree(it->second.p);
    e->w[key] = wt;
    return 0;
}

extern "C" int bakan_full_build(void* engine) {
    Engine* e = static_cast<Engine*>(engine);
    if (!e) return -1;
    if (e->built) return 0;
    return kq::full::build(e);
}

extern "C" int bakan_full_forward(void* engine, int token_id, int position, float* logits_out, int* vocab_size_out) {
    Engine* e = static_cast<Engine*>(engine);
    if (!e || !e->built) {
        kq::full::err("engine not built");
        return -1;
    }
    if (!logits_out) return -1;
    const int rc = kq::full::step(e, token_id, position, logits_out);
    if (rc == 0 && vocab_size_out) *vocab_size_out = e->c.vocab;
    return rc;
}

extern "C" int bakan_full_prefill(void* engine, const int32_t* token_ids, int num_tokens, float* logits_out,
                                  int* vocab_size_out) {
    Engine* e = static_cast<Engine*>(engine);
    if (!e || !e->built) {
        kq::full::err("engine not built");
        return -1;
    }
    if (!token_ids || !logits_out || num_tokens <= 0 || num_tokens > e->c.max_seq) {
        kq::full::err("num_tokens outside (0, max_cache_len]");
        return -1;
    }
    for (int i = 0; i < num_tokens; ++i) {
        const int rc = kq::full::step(e, token_ids[i], i, i + 1 == num_tokens ? logits_out : nullptr);
        if (rc) return rc;
    }
    if (vocab_size_out) *vocab_size_out = e->c.vocab;
    return 0;
}

extern "C" void bakan_full_reset_cache(void* engine) {
    Engine* e = static_cast<Engine*>(engine);
    if (!e || !e->built) return;
    const size_t kv = (size_t)e->c.nkv * e->c.max_seq * e->c.hd * sizeof(__half);
    const size_t conv = (size_t)e->c.conv_dim() * e->c.conv_k * sizeof(__half);
    const size_t st = (size_t)e->c.lnv * e->c.lvd * e->c.lkd * sizeof(float);
    for (auto& ly : e->L) {
        if (ly.linear) {
            cudaMemsetAsync(ly.conv_state, 0, conv, e->s);
            cudaMemsetAsync(ly.state, 0, st, e->s);
        } else {
            cudaMemsetAsync(ly.kc, 0, kv, e->s);
            cudaMemsetAsync(ly.vc, 0, kv, e->s);
        }
    }
    cudaStreamSynchronize(e->s);
    e->position = 0;
}

extern "C" void bakan_full_destroy(void* engine) { kq::full::destroy(static_cast<Engine*>(engine)); }

extern "C" int bakan_full_num_layers(void* engine) {
    Engine* e = static_cast<Engine*>(engine);
    return e ? e->c.layers : 0;
}

extern "C" int bakan_full_vocab_size(void* engine) {
    Engine* e = static_cast<Engine*>(engine);
    return e ? e->c.vocab : 0;
}

extern "C" void bakan_full_set_debug(void* engine, int enable) {
    Engine* e = static_cast<Engine*>(engine);
    if (e) e->debug = enable;
}

extern "C" int bakan_full_set_kv_cache(void* engine, int attn_layer_idx, const void* keys_data,
                                       const void* values_data, int seq_len, int num_kv_heads, int head_dim) {
    Engine* e = static_cast<Engine*>(engine);
    if (!e || !e->built) {
        kq::full::err("engine not built");
        return -1;
    }
    kq::full::Layer* lp = kq::full::nth_layer(e, false, attn_layer_idx);
    if (!lp || seq_len <= 0 || seq_len > e->c.max_seq || num_kv_heads != e->c.nkv || head_dim != e->c.hd ||
        !keys_data || !values_data) {
        kq::full::err("set_kv_cache: layer, length or shape outside the model's");
        return -1;
    }
    auto& ly = *lp;
    const size_t row = (size_t)head_dim * sizeof(__half);
    const size_t kvb = (size_t)e->c.nkv * e->c.max_seq * row;
    cudaError_t ce = cudaMemsetAsync(ly.kc, 0, kvb, e->s);
    if (ce == cudaSuccess) ce = cudaMemsetAsync(ly.vc, 0, kvb, e->s);
    // source [head][seq][dim] -> cache [head][max_seq][dim]
    if (ce == cudaSuccess)
        ce = cudaMemcpy2DAsync(ly.kc, (size_t)e->c.max_seq * row, keys_data, (size_t)seq_len * row,
                               (size_t)seq_len * row, num_kv_heads, cudaMemcpyHostToDevice, e->s);
    if (ce == cudaSuccess)
        ce = cudaMemcpy2DAsync(ly.vc, (size_t)e->c.max_seq * row, values_data, (size_t)seq_len * row,
                               (size_t)seq_len * row, num_kv_heads, cudaMemcpyHostToDevice, e->s);
    if (ce == cudaSuccess) ce = cudaStreamSynchronize(e->s);
    return ce == cudaSuccess ? 0 : -1;
}

// replaces kandiga/metal/full_forward.h:174 (state [hv][dv][dk] fp32)
extern "C" int bakan_full_set_linear_state(void* engine, int lin_layer_idx, const void* state_data, int state_bytes) {
    Engine* e = static_cast<Engine*>(engine);
    if (!e || !e->built) {
        kq::full::err("engine not built");
        return -1;
    }
    kq::full::Layer* lp = kq::full::nth_layer(e, true, lin_layer_idx);
    const size_t want = (size_t)e->c.lnv * e->c.lvd * e->c.lkd * sizeof(float);
    if (!lp) {
        fprintf(stderr, "[kandiga] ERROR: bakan_full: no linear-attention layer %d\n", lin_layer_idx);
        return -1;
    }
    if (!state_data || state_bytes < 0 || (size_t)state_bytes != want) {
        fprintf(stderr, "[kandiga] ERROR: bakan_full: linear state %d: %d bytes (expected %zu)\n", lin_layer_idx,
                state_bytes, want);
        return -1;
    }
    return cudaMemcpy(lp->state, state_data, want, cudaMemcpyHostToDevice) == cudaSuccess ? 0 : -1;
}

// replaces kandiga/metal/full_forward.h:193 (conv buffer [channel][kernel_pos] fp16)
extern "C" int bakan_full_set_conv_state(void* engine, int lin_layer_idx, const void* conv_data, int conv_bytes) {
    Engine* e = static_cast<Engine*>(engine);
    if (!e || !e->built) {
        kq::full::err("engine not built");
        return -1;
    }
    kq::full::Layer* lp = kq::full::nth_layer(e, true, lin_layer_idx);
    const size_t want = (size_t)e->c.conv_dim() * e->c.conv_k * sizeof(__half);
    if (!lp) {
        fprintf(stderr, "[kandiga] ERROR: bakan_full: no linear-attention layer %d\n", lin_layer_idx);
        return -1;
    }
    if (!conv_data || conv_bytes < 0 || (size_t)conv_bytes != want) {
        fprintf(stderr, "[kandiga] ERROR: bakan_full: conv state %d: %d bytes (expected %zu)\n", lin_layer_idx,
                conv_bytes, want);
        return -1;
    }
    return cudaMemcpy(lp->conv_state, conv_data, want, cudaMemcpyHostToDevice) == cudaSuccess ? 0 : -1;
}

extern "C" int bakan_full_set_position(void* engine, int position) {
    Engine* e = static_cast<Engine*>(engine);
    if (!e || !e->built || position < 0 || position >= e->c.max_seq) return -1;
    e->position = position;
    return 0;
}

extern "C" int kq_full_time_steps(void* engine, int token_id, int position, int steps, float* device_ms) {
    Engine* e = static_cast<Engine*>(engine);
    if (!e || !e->built || steps <= 0 || !device_ms || position < 0 || position + steps > e->c.max_seq ||
        token_id < 0 || token_id >= e->c.vocab)
        return -1;
    int* stage = nullptr;  // one slot per step, so no copy reads a slot the host rewrites
    if (cudaHostAlloc(reinterpret_cast<void**>(&stage), (size_t)steps * 4 * sizeof(int), 0) != cudaSuccess) {
        cudaGetLastError();
        return -1;
    }
    for (int i = 0; i < steps; ++i) {
        stage[4 * i] = token_id;
        stage[4 * i + 1] = position + i;
        stage[4 * i + 2] = position + i + 1;
    }
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    cudaError_t ce = cudaEventRecord(a, e->s);
    for (int i = 0; i < steps && ce == cudaSuccess; ++i) {
        ce = cudaMemcpyAsync(e->dev_i, stage + 4 * i, 3 * sizeof(int), cudaMemcpyHostToDevice, e->s);
        if (ce == cudaSuccess) ce = cudaGraphLaunch(e->g_body, e->s);
        if (ce == cudaSuccess) ce = cudaGraphLaunch(e->g_head, e->s);
    }
    if (ce == cudaSuccess) ce = cudaEventRecord(b, e->s);
    if (ce == cudaSuccess) ce = cudaEventSynchronize(b);
    float ms = 0.f;
    if (ce == cudaSuccess) ce = cudaEventElapsedTime(&ms, a, b);
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    cudaFreeHost(stage);
    if (ce != cudaSuccess) return -1;
    *device_ms = ms;
    e->position = position + steps;
    return 0;
}

extern "C" int kq_full_position(void* engine) {
    Engine* e = static_cast<Engine*>(engine);
    return e ? e->position : -1;
}
