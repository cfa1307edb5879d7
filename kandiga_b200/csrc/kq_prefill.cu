// kq_prefill.cu -- grouped routed-expert MLP for many tokens (prefill) on tcgen05.
//
// The reference groups the T*K (token, slot) assignments by expert with a
// stable sort and runs every expert once over its tokens
// (kandiga/engine.py:407-418 grouping, :260-292 gate/up+SwiGLU and down
// kernels; kandiga/metal/kandiga_cpu_expert.m:773-838 for the CPU path).  Here:
//
//   group_kernel         one CTA: tokens per expert, offsets, the position of
//                        every assignment in expert-sorted order and the list
//                        of live 128-token work chunks
//   gather_kernel        x rows gathered into expert-sorted order as fp16
//   moe_tc_kernel        grouped GEMM, once for gate/up (+SwiGLU) and once for
//                        down.  Swap-AB: the MMA's M = 128 weight rows, N = the
//                        expert's tokens (16..128 per chunk), K = input dim.
//                        Warp-specialised and persistent (one CTA per SM):
//                          warp 0     TMA: packed KQ tiles of the expert
//                                     (2D tensor map over 128-byte rows,
//                                     128-byte swizzle)
//                          warp 1     TMA: the tokens' 64-wide K chunks, several
//                                     groups per stage when the box is small
//                          warps 2-13 dequantise, three sets of four taking
//                                     alternate 64-wide groups: thread = weight
//                                     row; a group's words -> 32 exact fp16
//                                     pairs -> W = q*s + b -> one swizzled
//                                     128-byte row of an A stage
//                          next 3     one thread each issues tcgen05.mma
//                                     (M=128, N=tokens, K=16) for every 3rd
//                                     group into its own TMEM accumulator;
//                                     commits free the stages
//                          last 4     epilogue: tcgen05.ld of the
//                                     accumulators, summed; gate/up rows sit
//                                     8 lanes apart, act = silu(g)*u -> fp16
//                                     in expert-sorted order; down -> fp32
//   combine_kernel       out = [res] + sum_k w_k y_k, per-k outputs
//                        (kandiga/metal/moe_block.metal:515-584)
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstdio>
#include <cstring>

#include "kq_internal.h"
#include "kq_tc.cuh"

namespace kq {

// ---- grouping ----------------------------------------------------------------------------

constexpr int GROUP_THREADS = 1024;
constexpr int GROUP_MAX_E = 4096;  // experts per layer the one-CTA grouping supports

// Grouping in one CTA (the T*K assignments of a prefill batch are a few
// thousand ids; one CTA avoids grid-wide synchronisation):
//   1. rank[a] = atomicAdd(&cnt[idx[a]], 1) in shared memory (kept in inv_pos)
//   2. exclusive scans of the padded counts roundup(cnt, pad) (offsets) and of
//      ceil(cnt/chunk) (work chunks)
//   3. pos = offset[e] + rank[a]; s_tok[pos] = a / K; inv_pos[a] = pos
// Expert segments start on multiples of `pad` positions; the pad positions get
// s_tok = -1 and *n_pos is the padded total.  The order of an expert's
// assignments inside its segment is unspecified; each position is an
// independent MMA column, so results do not depend on it.
// Ids outside [0, E) get inv_pos = -1; all but -1 (an empty slot) latch
// KQ_DEV_BAD_EXPERT.
__global__ void __launch_bounds__(GROUP_THREADS, 1)
    group_kernel(const int32_t* __restrict__ idx, int A, int K, int E, int chunk, int pad, int* __restrict__ count,
                 int* __restrict__ offset, int32_t* __restrict__ s_tok, int32_t* __restrict__ inv_pos,
                 int4* __restrict__ chunk_list, int* __restrict__ n_chunks, int* __restrict__ n_pos,
                 uint32_t* status, uint32_t* act_flag) {
    __shared__ int cnt[GROUP_MAX_E];
    __shared__ int off_s[GROUP_MAX_E];
    __shared__ int wsum[2][32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    pdl_wait();  // the routing is complete and visible
    if (tid == 0) *act_flag = 0u;
    for (int e = tid; e < E; e += GROUP_THREADS) cnt[e] = 0;
    __syncthreads();
    // Eight ids per thread are loaded before any is counted (one CTA: a load
    // per loop trip would leave it latency-bound), and lanes of a warp with
    // the same id take their ranks with one shared-memory atomic.  The loop
    // bound is the warp's (a0 = warp's first index), so every lane reaches the
    // warp-wide match and shuffle; lanes past A carry id -1.
    constexpr int GU = 8;
    for (int a0 = tid - lane; a0 < A; a0 += GROUP_THREADS * GU) {
        int v[GU];
#pragma unroll
        for (int u = 0; u < GU; ++u) {
            const int a = a0 + lane + u * GROUP_THREADS;
            v[u] = a < A ? idx[a] : -1;
        }
#pragma unroll
        for (int u = 0; u < GU; ++u) {
            const int a = a0 + lane + u * GROUP_THREADS;
            const bool ok = (unsigned)v[u] < (unsigned)E;
            const unsigned grp = __match_any_sync(0xffffffffu, ok ? v[u] : -1);
            const int leader = __ffs(grp) - 1;
            int base = 0;
            if (ok && lane == leader) base = atomicAdd(&cnt[v[u]], __popc(grp));
            base = __shfl_sync(0xffffffffu, base, leader);
            if (a < A) {
                inv_pos[a] = ok ? base + __popc(grp & ((1u << lane) - 1u)) : -1;
                if (!ok && v[u] != -1) set_status(status, KQ_DEV_BAD_EXPERT);  // -1: an empty slot
            }
        }
    }
    __syncthreads();
    // thread t owns experts [t*per, t*per + per)
    const int per = (E + GROUP_THREADS - 1) / GROUP_THREADS;
    const int e0 = min(tid * per, E), e1 = min(e0 + per, E);
    int n_loc = 0, c_loc = 0;
    for (int e = e0; e < e1; ++e) {
        n_loc += (cnt[e] + pad - 1) / pad * pad;
        c_loc += (cnt[e] + chunk - 1) / chunk;
    }
    int n_inc = n_loc, c_inc = c_loc;  // inclusive warp scans
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int a = __shfl_up_sync(0xffffffffu, n_inc, o), b = __shfl_up_sync(0xffffffffu, c_inc, o);
        if (lane >= o) {
            n_inc += a;
            c_inc += b;
        }
    }
    if (lane == 31) {
        wsum[0][warp] = n_inc;
        wsum[1][warp] = c_inc;
    }
    __syncthreads();
    if (warp == 0) {
        int a = wsum[0][lane], b = wsum[1][lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int x = __shfl_up_sync(0xffffffffu, a, o), y = __shfl_up_sync(0xffffffffu, b, o);
            if (lane >= o) {
                a += x;
                b += y;
            }
        }
        wsum[0][lane] = a;  // inclusive over warps
        wsum[1][lane] = b;
    }
    __syncthreads();
    int n_run = n_inc - n_loc + (warp ? wsum[0][warp - 1] : 0);
    int c_run = c_inc - c_loc + (warp ? wsum[1][warp - 1] : 0);
    for (int e = e0; e < e1; ++e) {
        const int ne = cnt[e], nch = (ne + chunk - 1) / chunk, np = (ne + pad - 1) / pad * pad;
        off_s[e] = n_run;
        offset[e] = n_run;
        count[e] = ne;
        for (int c = 0; c < nch; ++c)
            chunk_list[c_run + c] = make_int4(e, min(chunk, ne - c * chunk), n_run + c * chunk, c);
        for (int i = ne; i < np; ++i) s_tok[n_run + i] = -1;
        n_run += np;
        c_run += nch;
    }
    if (tid == GROUP_THREADS - 1) {
        *n_chunks = c_run;
        *n_pos = n_run;
    }
    __syncthreads();
    for (int a0 = tid - lane; a0 < A; a0 += GROUP_THREADS * GU) {
        int r[GU], v[GU];
#pragma unroll
        for (int u = 0; u < GU; ++u) {
            const int a = a0 + lane + u * GROUP_THREADS;
            r[u] = a < A ? inv_pos[a] : -1;  // written by this thread above
            v[u] = a < A ? idx[a] : 0;
        }
#pragma unroll
        for (int u = 0; u < GU; ++u) {
            if (r[u] < 0) continue;
            const int a = a0 + lane + u * GROUP_THREADS;
            const int pos = off_s[v[u]] + r[u];
            s_tok[pos] = a / K;
            inv_pos[a] = pos;
        }
    }
}

// Xs[pos] = fp16(x[s_tok[pos]] * scale[tok]); one warp per position.  fp16
// inputs are copied unscaled (xinv == nullptr); other types get a power-of-two
// scale so every value fits fp16, and xinv[pos] = 1/scale.  Pad positions
// (s_tok < 0) are left unwritten.
__global__ void gather_kernel(const void* __restrict__ x, int x_dtype, int H, const int32_t* __restrict__ s_tok,
                              const int* __restrict__ n_pos, __half* __restrict__ Xs, float* __restrict__ xinv,
                              int8_t* __restrict__ act_exp, int n_exp) {
    const int pos = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    pdl_wait();  // the grouping is complete and visible
    if (pos >= *n_pos) return;
    for (int b = lane; b < n_exp; b += 32) act_exp[(size_t)pos * n_exp + b] = 0;  // see act_fixup_kernel
    const int tok = s_tok[pos];
    if (tok < 0) return;
    const size_t src = (size_t)tok * H;
    if (x_dtype == KQ_DT_F16) {  // a straight copy, four 16-byte loads in flight per lane
        const uint4* s4 = reinterpret_cast<const uint4*>(static_cast<const __half*>(x) + src);
        uint4* d4 = reinterpret_cast<uint4*>(Xs + (size_t)pos * H);
        const int n = H / 8;
        for (int c = lane; c < n; c += 128) {
            uint4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) v[u] = c + 32 * u < n ? __ldg(s4 + c + 32 * u) : make_uint4(0, 0, 0, 0);
#pragma unroll
            for (int u = 0; u < 4; ++u)
                if (c + 32 * u < n) d4[c + 32 * u] = v[u];
        }
        return;
    }
    float scale = 1.f;
    {
        float amax = 0.f;
        for (int c = lane; c < H / 8; c += 32) {
            float v[8];
            load8(x, x_dtype, src + (size_t)c * 8, false, v);
#pragma unroll
            for (int k = 0; k < 8; ++k) amax = fmaxf(amax, fabsf(v[k]));
        }
        scale = pow2_scale(warp_max(amax));
        if (lane == 0) xinv[pos] = 1.f / scale;
    }
    for (int c = lane; c < H / 8; c += 32) {
        float v[8];
        load8(x, x_dtype, src + (size_t)c * 8, false, v);
        uint32_t h[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const __half2 hh = __floats2half2_rn(v[2 * k] * scale, v[2 * k + 1] * scale);
            h[k] = *reinterpret_cast<const uint32_t*>(&hh);
        }
        *reinterpret_cast<uint4*>(Xs + (size_t)pos * H + (size_t)c * 8) = make_uint4(h[0], h[1], h[2], h[3]);
    }
}

// ---- grouped expert GEMM on tcgen05 ----------------------------------------------------------

struct TcParams {
    const uint8_t* base;  // layer base
    size_t expert_bytes;
    size_t mat_off;       // matrix offset inside an expert
    int nst;              // 512-wide K super-tiles
    int n_mt;             // 128-row M-tiles per expert
    int E;
    const int* count;
    const int* offset;
    const int4* chunk_list;     // live work chunks: {expert, tokens (<= 128), first position, chunk}
    const int* n_chunks;
    int mode;             // 0: gate/up + activation -> act_s; 1: down -> ys
    __half* act_s;        // [A][I]
    int I;
    float* ys;            // [A][H]
    int H;
    const float* xinv;    // [A] input scale inverse (gate/up), or null
    int act_kind;
    uint32_t* status;
    // fp16 range of the activations (see act_fixup_kernel)
    uint32_t* act_flag;   // nonzero: some activation row was stored scaled
    int8_t* act_exp;      // [P][I / 16] exponent a 16-row block of act_s was stored with
    float* act_inv;       // [P] factor the down projection of a position is multiplied by
};

constexpr int TC_NMMA = 3;            // MMA-issuing warps = dequantising warp sets (4 warps each)
constexpr int TC_SLOTS = 2;           // A stages per issuer
constexpr int TC_NSTAGE = TC_NMMA * TC_SLOTS;  // A stages (one 64-wide group of 128 weight rows each)
constexpr int TC_NKQ = 2;             // packed super-tile stages
constexpr int TC_NDQ = TC_NMMA;
// Group gi of an item (item-local index) is dequantised by set gi % TC_NMMA
// into that set's private ring of TC_SLOTS A stages and consumed by the
// issuer of the same number.  An mbarrier wait tells apart only two phases,
// so each stage must have exactly one filler and one consumer, in order.
constexpr int TC_NEPI = 8;            // epilogue warps (TC_NEPI / 4 per TMEM lane quarter)
constexpr int TC_THREADS = 32 * (2 + 4 * TC_NDQ + TC_NMMA + TC_NEPI);  // producers, dequant, MMA, epilogue
constexpr int TC_STAGE_BYTES = 16384; // 128 rows x 128 B
constexpr int TC_TMEM_COLS = 512;     // 2 buffers x 256 (TC_NMMA x 64) columns, or TC_NMMA x 128 for a 128-token box
static_assert(TC_NMMA * 64 <= 256 && TC_NMMA * 128 <= TC_TMEM_COLS, "accumulators must fit tensor memory");

// A super-tile (the 8 tiles of 128 weight rows x 512 columns) lands in shared
// memory by ONE 3D TMA load: the layer viewed as 128-byte rows (dimension 1)
// and tiles nst * tile_bytes apart (dimension 2), box = 128 bytes x one tile's
// rows x 8 tiles, 128-byte swizzle.  (Each SM's copy engine completes only a
// few copies per microsecond whatever their size: eight per-tile loads held a
// super-tile to ~17 GB/s per SM.)  The tiles sit back to back, tile j from
// 128-byte row j * rows_per_tile of the 1024-aligned slot, and byte
// (R, 16 * c + b) of the slot at R * 128 + 16 * (c ^ (R & 7)) + b, so a
// dequantising quarter-warp (rows r16 = 0..7 of one tile, one 64-wide group)
// reads eight distinct 16-byte bank groups.
template <int BITS>
__host__ __device__ constexpr int tc_super_slot() {
    return (8 * TileT<BITS>::BYTES + 1023) / 1024 * 1024;
}

// B stages (16 KB: 16384 / (box * 128) groups of tokens each): as many as shared
// memory holds beside the A stages and the packed super-tile slots.  A
// 128-token box fills a stage with one group, and a stage is refilled only
// after the MMAs that read it retire, so the ring's depth is the number of
// groups whose (strided, L2- or DRAM-latency) token loads are in flight.
template <int BITS>
__host__ __device__ constexpr int tc_nb() {
    return BITS == 3 ? 4 : 3;
}

template <int BITS>
__host__ __device__ constexpr size_t tc_smem_bytes() {
    return 1024 + (size_t)(TC_NSTAGE + tc_nb<BITS>()) * TC_STAGE_BYTES + (size_t)TC_NKQ * tc_super_slot<BITS>() + 256;
}
static_assert(tc_smem_bytes<3>() <= 232448 && tc_smem_bytes<4>() <= 232448, "shared memory per CTA");
// mbarriers (kq full/empty, A full/empty, B full/empty, D full/empty, drain) and the TMEM slot word
static_assert((2 * TC_NKQ + 2 * TC_NSTAGE + 2 * tc_nb<3>() + 4 + TC_NMMA) * 8 + 4 <= 256 &&
                  (2 * TC_NKQ + 2 * TC_NSTAGE + 2 * tc_nb<4>() + 4 + TC_NMMA) * 8 + 4 <= 256,
              "barrier area");

// 16-byte unit `lane` of 512-byte chunk `chunk` of a swizzled tile whose first
// 128-byte row is row `row0` of its 1024-aligned slot
__device__ __forceinline__ uint4 tile_u4(const uint8_t* tile, int row0, int chunk, int lane) {
    const int row = chunk * 4 + (lane >> 3);
    return *reinterpret_cast<const uint4*>(tile + row * 128 + (((lane & 7) ^ ((row0 + row) & 7)) << 4));
}

template <int SB_DT>
__device__ __forceinline__ __half to_half16(uint32_t v16) {
    if (SB_DT == KQ_DT_F16) return __ushort_as_half((unsigned short)v16);
    return __float2half_rn(__uint_as_float(v16 << 16));
}

// Dequantise row r16 (0..15) x group g (0..7) of a KQ tile into 64 fp16 weights
// W = q*s + b, written as one 128-byte row (row m) of a swizzled A stage.
// A pair extracts as two exact fp16 values 2^(10-k) + q; subtracting the
// constant 2^(10-k) leaves q exactly, and one HFMA2 forms W = q*s + b with a
// single rounding.  No intermediate exceeds |W|, so any scale and bias whose
// weights fit fp16 dequantise without overflow.
template <int BITS, int SB_DT, int J>
__device__ __forceinline__ void dq_pairs(const uint32_t* wd, const uint32_t* sh, __half2 s2, __half2 b2,
                                         uint32_t* out) {
    if constexpr (J < 32) {
        const uint32_t h = pair_of<BITS, J>(wd, sh);
        constexpr float off = pair_offset<BITS>(J);
        const __half2 q2 = __hsub2(*reinterpret_cast<const __half2*>(&h), __float2half2_rn(off));
        const __half2 w2 = __hfma2(q2, s2, b2);
        out[J] = *reinterpret_cast<const uint32_t*>(&w2);
        dq_pairs<BITS, SB_DT, J + 1>(wd, sh, s2, b2, out);
    }
}

// Returns max(|b|, |qmax*s + b|) in fp16: the largest |W| of the group (inf
// when a weight or the scale/bias itself does not fit fp16).
template <int BITS, int SB_DT>
__device__ __forceinline__ __half dequant_row(const uint8_t* tile, int row0, int r16, int g, uint32_t (&out)[32]) {
    constexpr int W = TileT<BITS>::W;  // words per (lane, set); the scale/bias chunk is chunk W
    const int l = 4 * (r16 & 7) + (g & 3);
    const int set = 2 * (r16 >> 3) + (g >> 2);
    const int q0 = set * W;  // first word of the set; q0 % 4 is 0 (4-bit) or 0/2 (3-bit)
    const uint4 u0 = tile_u4(tile, row0, q0 >> 2, l), u1 = tile_u4(tile, row0, (q0 >> 2) + 1, l);
    const uint32_t arr[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
    const bool odd = (q0 & 3) != 0;
    uint32_t wd[W], sh[W];
#pragma unroll
    for (int w = 0; w < W; ++w) wd[w] = (W == 8 || !odd) ? arr[w] : arr[(w + 2) & 7];
#pragma unroll
    for (int w = 0; w < W; ++w) sh[w] = wd[w] >> (BITS == 3 ? 9 : 8);
    const int l2 = 4 * (r16 & 7) + (g >> 1), kk = 2 * (r16 >> 3) + (g & 1);
    const int srow = W * 4 + (l2 >> 3);
    const uint32_t sbw =
        *reinterpret_cast<const uint32_t*>(tile + srow * 128 + (((l2 & 7) ^ ((row0 + srow) & 7)) << 4) + kk * 4);
    const __half s = to_half16<SB_DT>(sbw & 0xFFFFu), b = to_half16<SB_DT>(sbw >> 16);
    const __half2 s2 = __halves2half2(s, s), b2 = __halves2half2(b, b);
    dq_pairs<BITS, SB_DT, 0>(wd, sh, s2, b2, out);
    return __hmax(__habs(b), __habs(__hfma(s, __float2half_rn((float)((1 << BITS) - 1)), b)));
}

// out[32] as row m (one swizzled 128-byte row) of an A stage
__device__ __forceinline__ void a_row_store(const uint32_t (&out)[32], uint8_t* a_stage, int m) {
#pragma unroll
    for (int c = 0; c < 8; ++c)
        *reinterpret_cast<uint4*>(a_stage + tc::sw128_offset(m, c * 8)) =
            make_uint4(out[4 * c], out[4 * c + 1], out[4 * c + 2], out[4 * c + 3]);
}

struct TcItem {
    int e, mt, n, box, pos0;
};

// item = chunk * n_mt + mt over the live chunks.  The descriptor load is
// volatile so it issues where it is written: each role loads the next item's
// descriptor one item ahead.
__device__ __forceinline__ int4 tc_desc_load(const TcParams& p, int item) {
    int4 d;
    asm volatile("ld.global.nc.v4.s32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(d.x), "=r"(d.y), "=r"(d.z), "=r"(d.w)
                 : "l"(p.chunk_list + item / p.n_mt));
    return d;
}

__device__ __forceinline__ TcItem tc_item(const TcParams& p, int4 d, int item) {
    TcItem it;
    it.mt = item % p.n_mt;
    it.e = d.x;
    it.n = d.y;
    it.pos0 = d.z;
    it.box = it.n <= 16 ? 16 : (it.n <= 32 ? 32 : (it.n <= 64 ? 64 : 128));
    return it;
}

template <int BITS, int SB_DT>
__global__ void __launch_bounds__(TC_THREADS, 1)
    moe_tc_kernel(const TcParams p, const __grid_constant__ CUtensorMap tb16, const __grid_constant__ CUtensorMap tb32,
                  const __grid_constant__ CUtensorMap tb64, const __grid_constant__ CUtensorMap tb128,
                  const __grid_constant__ CUtensorMap tkq) {
    extern __shared__ uint8_t smem_raw[];
    constexpr int TB = TileT<BITS>::BYTES;
    constexpr int TR = TB / 128;             // 128-byte rows per tile
    constexpr int SS = tc_super_slot<BITS>();
    constexpr int TC_NB = tc_nb<BITS>();
    // 1024-byte aligned in the shared window; an offset from smem_raw keeps the
    // shared address space, so accesses through it compile to shared-memory ops
    uint8_t* sm = smem_raw + ((1024u - ((uint32_t)__cvta_generic_to_shared(smem_raw) & 1023u)) & 1023u);
    uint8_t* sA = sm;
    uint8_t* sB = sA + TC_NSTAGE * TC_STAGE_BYTES;
    uint8_t* sK = sB + TC_NB * TC_STAGE_BYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sK + TC_NKQ * SS);
    uint64_t* kq_full = bars;                        // [TC_NKQ]
    uint64_t* kq_empty = kq_full + TC_NKQ;           // [TC_NKQ]
    uint64_t* a_full = kq_empty + TC_NKQ;            // [TC_NSTAGE]
    uint64_t* a_empty = a_full + TC_NSTAGE;          // [TC_NSTAGE]
    uint64_t* b_full = a_empty + TC_NSTAGE;          // [TC_NB]
    uint64_t* b_empty = b_full + TC_NB;              // [TC_NB]
    uint64_t* d_full = b_empty + TC_NB;              // [2]
    uint64_t* d_empty = d_full + 2;                  // [2]
    uint64_t* drain = d_empty + 2;                   // [TC_NMMA] exit: this issuer's MMAs are done
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + TC_NMMA);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    if (tid == 0) {
        for (int i = 0; i < TC_NKQ; ++i) {
            mbar_init(&kq_full[i], 1);
            mbar_init(&kq_empty[i], 128 * TC_NDQ);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&d_full[i], TC_NMMA);
            mbar_init(&d_empty[i], 32 * TC_NEPI);
        }
        for (int i = 0; i < TC_NMMA; ++i) mbar_init(&drain[i], 1);
        for (int i = 0; i < TC_NSTAGE; ++i) {
            mbar_init(&a_full[i], 128);
            mbar_init(&a_empty[i], 1);
        }
        for (int i = 0; i < TC_NB; ++i) {
            mbar_init(&b_full[i], 1);
            mbar_init(&b_empty[i], TC_NMMA);
        }
        fence_mbar_init();
    }
    constexpr int MMA_WARP = 2 + 4 * TC_NDQ;
    if (warp == MMA_WARP) {
        tc::tmem_alloc(tmem_slot, TC_TMEM_COLS);
        tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tmem_slot;
    // The prologue above overlaps the previous kernel's tail.  Global memory
    // is touched only after the wait; the next kernel may launch at once (it
    // cannot share an SM with this one's shared memory, and waits in turn).
    pdl_wait();
    pdl_launch_dependents();
    const int n_items = *p.n_chunks * p.n_mt;
    const int groups = p.nst * 8;

    if (warp == 0) {
        // ---------------- producer: packed super-tiles ----------------
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            uint32_t kc = 0;
            int4 nd = (int)blockIdx.x < n_items ? tc_desc_load(p, blockIdx.x) : make_int4(0, 0, 0, 0);
            for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
                const TcItem it = tc_item(p, nd, item);
                if (item + (int)gridDim.x < n_items) nd = tc_desc_load(p, item + gridDim.x);
                const size_t ebase = (size_t)it.e * p.expert_bytes + p.mat_off;  // bytes into the layer
                for (int st = 0; st < p.nst; ++st, ++kc) {
                    const int s = kc % TC_NKQ;
                    mbar_wait_sleep(&kq_empty[s], ((kc / TC_NKQ) & 1) ^ 1, p.status);
                    mbar_expect_tx(&kq_full[s], 8 * TB);
                    const size_t off = ebase + ((size_t)it.mt * 8 * p.nst + st) * TB;  // multiple of 128
                    tc::tma_load_3d_hint(sK + (size_t)s * SS, &tkq, 0, (int)(off >> 7), 0, &kq_full[s], pol);
                }
            }
            for (uint32_t f = kc > TC_NKQ ? kc - TC_NKQ : 0; f < kc; ++f)  // own fills landed
                mbar_drain(&kq_full[f % TC_NKQ], (f / TC_NKQ) & 1);
        }
    } else if (warp == 1) {
        // ---------------- producer: token K-chunks (B operand) ----------------
        // A B stage holds gpb = 16384 / (box * 128) consecutive groups of the item
        // (box rows x 64 fp16 each, one swizzled block per group), fetched by one
        // 3D load through the token tensor map of the item's box size.
        if (lane == 0) {
            const uint64_t pol = tc::policy_evict_last();
            uint32_t bc = 0;
            int4 nd = (int)blockIdx.x < n_items ? tc_desc_load(p, blockIdx.x) : make_int4(0, 0, 0, 0);
            for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
                const TcItem it = tc_item(p, nd, item);
                if (item + (int)gridDim.x < n_items) nd = tc_desc_load(p, item + gridDim.x);
                const void* tm = it.box == 16 ? (const void*)&tb16
                                              : (it.box == 32 ? (const void*)&tb32
                                                              : (it.box == 64 ? (const void*)&tb64 : (const void*)&tb128));
                const int gpb = TC_STAGE_BYTES / (it.box * 128);  // divides groups (a multiple of 8)
                for (int g0 = 0; g0 < groups; g0 += gpb, ++bc) {
                    const int bs = bc % TC_NB;
                    mbar_wait_sleep(&b_empty[bs], ((bc / TC_NB) & 1) ^ 1, p.status);
                    mbar_expect_tx(&b_full[bs], (uint32_t)TC_STAGE_BYTES);
                    // one 3D load: gpb groups of box rows x 64 fp16, group j at j * box * 128 bytes
                    tc::tma_load_3d_hint(sB + (size_t)bs * TC_STAGE_BYTES, tm, 0, it.pos0, g0, &b_full[bs], pol);
                }
            }
            for (uint32_t f = bc > TC_NB ? bc - TC_NB : 0; f < bc; ++f)  // own fills landed
                mbar_drain(&b_full[f % TC_NB], (f / TC_NB) & 1);
        }
    } else if (warp >= 2 && warp < MMA_WARP) {
        // ---------------- dequantise (set `ds` takes the groups gi % TC_NMMA == ds) ----------------
        const int ds = (warp - 2) >> 2;
        const int m = (tid - 64) & 127;  // A row 0..127
        const int jt = m >> 4, r16 = m & 15;
        uint32_t kc = 0, lc = 0;
        __half wmax = __float2half_rn(0.f);  // largest |W| this thread dequantised
        for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
            for (int st = 0; st < p.nst; ++st, ++kc) {
                const int s = kc % TC_NKQ;
                mbar_wait_sleep(&kq_full[s], (kc / TC_NKQ) & 1, p.status);
                const uint8_t* tile = sK + (size_t)s * SS + (size_t)jt * TB;
                // this set's groups of the super-tile: g = first, first + TC_NMMA, ... (one copy of the body)
                const int first = (ds - (st * 8) % TC_NMMA + TC_NMMA) % TC_NMMA;
#pragma unroll 1
                for (int g = first; g < 8; g += TC_NMMA) {
                    const int gs = ds * TC_SLOTS + (int)(lc % TC_SLOTS);
                    uint32_t out[32];  // computed before the stage is awaited: a stage is held only for its stores
                    wmax = __hmax(wmax, dequant_row<BITS, SB_DT>(tile, jt * TR, r16, g, out));
                    mbar_wait_sleep(&a_empty[gs], ((lc / TC_SLOTS) & 1) ^ 1, p.status);
                    a_row_store(out, sA + (size_t)gs * TC_STAGE_BYTES, m);
                    fence_proxy_async_smem();
                    tc::mbar_arrive(&a_full[gs]);
                    ++lc;
                }
                tc::mbar_arrive(&kq_empty[s]);
            }
        }
        if (!(__half2float(wmax) < 65504.f)) set_status(p.status, KQ_DEV_RANGE);
    } else if (warp < MMA_WARP + TC_NMMA) {
        // ---------------- MMA issue ----------------
        // One thread issues an M=128, K=16 MMA about every 70 cycles at best,
        // and each group also costs it a barrier wait and a commit; the tensor
        // pipe takes one about every 40 cycles at small N.  So the groups of an
        // item are spread over the TC_NMMA issuers, issuer mi accumulating the
        // groups gi % TC_NMMA == mi into its own TMEM columns; the epilogue
        // adds the accumulators in a fixed order, so a token's result does not
        // depend on the size of the chunk it lands in.  Accumulators: boxes
        // <= 64 tokens take TC_NMMA x 64 columns of one of two 256-column
        // buffers; a 128-token box takes TC_NMMA x 128 columns from column 0,
        // across both buffers, so it (and the item after it) first waits for
        // the previous item's epilogue.  Issuers without groups in a B stage
        // still wait for and release it, so every barrier sees all issuers.
        // The issuer index and the TMEM base pass through a shuffle so the
        // compiler knows them warp-uniform: the descriptors then live in
        // uniform registers instead of being moved there for every MMA.
        const int mi = __shfl_sync(0xffffffffu, warp - MMA_WARP, 0);
        const uint32_t tmem_u = __shfl_sync(0xffffffffu, tmem, 0);
        const uint32_t leader = lane == 0;
        {
            uint32_t lc = 0, ic = 0, bc = 0;
            bool prev_full = false;
            int4 nd = (int)blockIdx.x < n_items ? tc_desc_load(p, blockIdx.x) : make_int4(0, 0, 0, 0);
            for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
                const TcItem it = tc_item(p, nd, item);
                if (item + (int)gridDim.x < n_items) nd = tc_desc_load(p, item + gridDim.x);
                const int db = ic & 1;
                const int gpb = TC_STAGE_BYTES / (it.box * 128);
                const bool full = it.box == 128;
                mbar_wait_sleep(&d_empty[db], ((ic >> 1) & 1) ^ 1, p.status);
                if ((full || prev_full) && ic > 0)  // the other buffer's item (ic - 1) must be drained too
                    mbar_wait_sleep(&d_empty[db ^ 1], ((ic - 1) >> 1) & 1, p.status);
                prev_full = full;
                __syncwarp();
                tc::fence_after_sync();
                const uint32_t d_tmem = tmem_u + (full ? (uint32_t)(mi * 128) : (uint32_t)(db * 256 + mi * 64));
                const uint32_t idesc = tc::idesc_f16(128, it.box, false);
                for (int g0 = 0; g0 < groups; g0 += gpb, ++bc) {
                    const int bs = bc % TC_NB;
                    mbar_wait_sleep(&b_full[bs], (bc / TC_NB) & 1, p.status);
                    __syncwarp();
                    tc::fence_after_sync();
                    const int g1 = min(g0 + gpb, groups);
                    {
                        for (int gi = g0 + ((mi - g0 % TC_NMMA + TC_NMMA) % TC_NMMA); gi < g1; gi += TC_NMMA, ++lc) {
                            const int gs = mi * TC_SLOTS + (int)(lc % TC_SLOTS);
                            mbar_wait_sleep(&a_full[gs], (lc / TC_SLOTS) & 1, p.status);
                            __syncwarp();
                            tc::fence_after_sync();
                            const uint64_t da = tc::smem_desc_sw128(sA + (size_t)gs * TC_STAGE_BYTES);
                            const uint64_t dbd = tc::smem_desc_sw128(sB + (size_t)bs * TC_STAGE_BYTES +
                                                                     (size_t)(gi - g0) * it.box * 128);
#pragma unroll
                            for (int k = 0; k < 4; ++k)
                                tc::mma_f16_ss_warp(d_tmem, tc::desc_advance(da, 32 * k), tc::desc_advance(dbd, 32 * k),
                                                    idesc, gi > mi || k > 0, leader);
                            tc::mma_commit_warp(&a_empty[gs], leader);
                        }
                    }
                    tc::mma_commit_warp(&b_empty[bs], leader);
                }
                tc::mma_commit_warp(&d_full[db], leader);
                ++ic;
            }
            tc::mma_commit_warp(&drain[mi], leader);  // all of this issuer's MMAs complete before exit
            mbar_drain(&drain[mi], 0);
        }
    } else {
        // ---------------- epilogue (last TC_NEPI warps) ----------------
        const int q = warp & 3;         // TMEM lane quarter this warp may access
        const int L = q * 32 + lane;    // accumulator row
        const int half = (warp - (MMA_WARP + TC_NMMA)) >> 2;  // 16-column chunks half, half + TC_NEPI / 4, ...
        const bool act_scaled = p.mode == 1 && *reinterpret_cast<volatile uint32_t*>(p.act_flag) != 0u;
        uint32_t ic = 0;
        int4 nd = (int)blockIdx.x < n_items ? tc_desc_load(p, blockIdx.x) : make_int4(0, 0, 0, 0);
        for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
            const TcItem it = tc_item(p, nd, item);
            if (item + (int)gridDim.x < n_items) nd = tc_desc_load(p, item + gridDim.x);
            const int db = ic & 1;
            mbar_wait_sleep(&d_full[db], (ic >> 1) & 1, p.status);
            tc::fence_after_sync();
            const bool full = it.box == 128;
            const uint32_t acc_cols = full ? 128u : 64u;
            const uint32_t taddr = tmem + (full ? 0u : (uint32_t)(db * 256)) + ((uint32_t)(q * 32) << 16);
            for (int c0 = half * 16; c0 < it.box; c0 += 16 * (TC_NEPI / 4)) {
                uint32_t r[16];
                tc::tmem_ld16(taddr + (uint32_t)c0, r);
#pragma unroll
                for (int a = 1; a < TC_NMMA; ++a) {  // fixed order: (acc0 + acc1) + acc2 ...
                    uint32_t r2[16];
                    tc::tmem_ld16(taddr + (uint32_t)a * acc_cols + (uint32_t)c0, r2);
                    tc::tmem_ld_wait();
#pragma unroll
                    for (int i = 0; i < 16; ++i) r[i] = __float_as_uint(__uint_as_float(r[i]) + __uint_as_float(r2[i]));
                }
                tc::tmem_ld_wait();
                if (p.mode == 0) {
                    // Rows 0..7 of a 16-row tile are gate rows, 8..15 the matching up
                    // rows.  A gate lane and its up lane (8 lanes apart) swap half of
                    // their 16 columns, so that each computes 8 activations: the gate
                    // lane those of columns c0..c0+7, the up lane c0+8..c0+15, both for
                    // intermediate row irow.
                    const int jt = L >> 4, r16 = L & 15;
                    const bool gate_lane = r16 < 8;
                    const int irow = it.mt * 64 + jt * 8 + (r16 & 7);
                    const int nb = c0 + (gate_lane ? 0 : 8);
                    float a[8];
                    float amax = 0.f;
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        const float lo = __uint_as_float(r[i]), hi = __uint_as_float(r[8 + i]);
                        const float mine_v = gate_lane ? lo : hi;
                        const float other = __shfl_xor_sync(0xffffffffu, gate_lane ? hi : lo, 8);
                        const int n = nb + i;
                        const float xi = (p.xinv && n < it.n) ? p.xinv[it.pos0 + n] : 1.f;
                        const float g = (gate_lane ? mine_v : other) * xi, u = (gate_lane ? other : mine_v) * xi;
                        a[i] = n < it.n ? (p.act_kind == KQ_ACT_GELU_TANH ? activate(g, u, p.act_kind)
                                                                          : __fdividef(g * u, 1.f + __expf(-g)))
                                        : 0.f;
                        amax = fmaxf(amax, fabsf(a[i]));
                    }
                    // The warp's 16 activation rows of position n go to fp16 unscaled
                    // unless one of them reaches 2^15; then all 16 are stored times a
                    // power of two and the exponent is recorded for act_fixup_kernel.
                    if (__any_sync(0xffffffffu, amax >= 32768.f)) {
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const float mg = warp_max(gate_lane ? fabsf(a[i]) : 0.f);
                            const float mu = warp_max(gate_lane ? 0.f : fabsf(a[i]));
                            const float cmax = gate_lane ? mg : mu;  // this column's 16 rows
                            if (cmax >= 32768.f) {
                                const float sc = pow2_scale(cmax);
                                a[i] *= sc;
                                const int n = nb + i;
                                if ((lane & 15) == (gate_lane ? 0 : 8) && lane < 16 && n < it.n && sc < 1.f) {
                                    int e = 0;
                                    frexpf(sc, &e);  // sc = 2^(e - 1)
                                    p.act_exp[(size_t)(it.pos0 + n) * (p.I / 16) + it.mt * 4 + q] = (int8_t)(1 - e);
                                    atomicOr(p.act_flag, 1u);
                                }
                            }
                        }
                    }
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        if (nb + i < it.n) p.act_s[(size_t)(it.pos0 + nb + i) * p.I + irow] = __float2half_rn(a[i]);
                } else {
                    const int hrow = it.mt * 128 + L;
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const int n = c0 + i;
                        if (n < it.n) {
                            const float f = act_scaled ? p.act_inv[it.pos0 + n] : 1.f;
                            p.ys[(size_t)(it.pos0 + n) * p.H + hrow] = __uint_as_float(r[i]) * f;
                        }
                    }
                }
            }
            tc::fence_before_sync();
            tc::mbar_arrive(&d_empty[db]);
            ++ic;
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == MMA_WARP) tc::tmem_dealloc(tmem, TC_TMEM_COLS);
}

// ---- activation range ---------------------------------------------------------------------------

// The gate/up epilogue stores activations in fp16.  A 16-row block of a
// position whose largest |act| reaches 2^15 is stored times 2^-m (m >= 1, in
// act_exp; act_flag raised).  This pass gives every position one exponent,
// the largest of its blocks: a block stored with m is multiplied by
// 2^(m - m_max) in place (exact unless a value drops below the fp16 normal
// range, i.e. under 2^-24 of the position's largest), and act_inv[pos] =
// 2^m_max, by which the down projection's epilogue multiplies the position's
// outputs.  With act_flag clear (every activation fits fp16) a CTA only reads
// the flag.  One warp per position.
__global__ void act_fixup_kernel(const uint32_t* __restrict__ act_flag, const int8_t* __restrict__ act_exp,
                                 __half* __restrict__ act_s, float* __restrict__ act_inv,
                                 const int* __restrict__ n_pos, int I) {
    pdl_wait();  // the gate/up projection is complete and visible
    pdl_launch_dependents();
    if (*reinterpret_cast<const volatile uint32_t*>(act_flag) == 0u) return;
    const int nb = I / 16, lane = threadIdx.x & 31, wpb = blockDim.x >> 5;
    const int np = *n_pos;
    for (int pos = blockIdx.x * wpb + (threadIdx.x >> 5); pos < np; pos += gridDim.x * wpb) {
        const int8_t* ex = act_exp + (size_t)pos * nb;
        int mmax = 0;
        for (int b = lane; b < nb; b += 32) mmax = max(mmax, (int)ex[b]);
        mmax = __reduce_max_sync(0xffffffffu, mmax);
        if (lane == 0) act_inv[pos] = ldexpf(1.f, mmax);
        if (mmax == 0) continue;
        uint4* row = reinterpret_cast<uint4*>(act_s + (size_t)pos * I);
        for (int c = lane; c < I / 8; c += 32) {  // 8 halves of block c / 2
            const int d = (int)ex[c >> 1] - mmax;
            if (d == 0) continue;
            const float f = ldexpf(1.f, d);
            uint4 v = row[c];
            uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                float2 a = __half22float2(*reinterpret_cast<const __half2*>(&w[k]));
                const __half2 h = __floats2half2_rn(a.x * f, a.y * f);
                w[k] = *reinterpret_cast<const uint32_t*>(&h);
            }
            row[c] = make_uint4(w[0], w[1], w[2], w[3]);
        }
    }
}

// ---- combine ----------------------------------------------------------------------------------

// out[t][h] = [res[t][h]] + sum_k w[t][k] * ys[pos(t,k)][h]; per-k outputs optional.
// One thread per 4 consecutive h (H % 4 == 0): 16-byte reads of the expert rows.
// out_rows (optional): row t goes to out_rows[t] (any device address, a
// peer's memory included; rows with a null pointer are skipped) instead of
// out + t * H; each CTA then fences once at system scope after a barrier (a
// release is cumulative over the CTA's writes ordered before it), so a flag
// released after this kernel covers the rows for a reader on another GPU.
__global__ void combine_kernel(const float* __restrict__ ys, const int32_t* __restrict__ inv_pos,
                               const float* __restrict__ w, int T, int K, int H, void* out, void* out_per_k,
                               int out_dtype, const void* residual, void* const* __restrict__ out_rows) {
    const int h = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
    pdl_wait();  // the down projection is complete and visible
    bool wrote = false;
    // rows blockIdx.y, + gridDim.y, ... (one row a CTA unless the rows go to
    // other GPUs: then a CTA takes several and fences once)
    for (int t = blockIdx.y; t < T; t += gridDim.y) {
        void* o = out;
        size_t orow = (size_t)t * H;
        if (out_rows) {  // uniform over the CTA
            o = out_rows[t];
            orow = 0;
        }
        if (h >= H || !(o || out_per_k)) continue;
        wrote |= o != nullptr;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        for (int k = 0; k < K; ++k) {
            const int pos = inv_pos[(size_t)t * K + k];
            const float4 y4 = pos >= 0 ? *reinterpret_cast<const float4*>(ys + (size_t)pos * H + h)
                                       : make_float4(0.f, 0.f, 0.f, 0.f);
            const float y[4] = {y4.x, y4.y, y4.z, y4.w};
            if (out_per_k)
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    store_from_float(out_per_k, out_dtype, ((size_t)t * K + k) * H + h + j, y[j]);
            if (o) {
                const float wk = w[(size_t)t * K + k];
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[j] += y[j] * wk;
            }
        }
        if (o) {
            float v[4];
#pragma unroll
            for (int j = 0; j < 4; ++j)
                v[j] = residual ? load_as_float(residual, out_dtype, (size_t)t * H + h + j) + acc[j] : acc[j];
            const size_t esz = out_dtype == KQ_DT_F32 ? 4 : 2;
            const uintptr_t addr = reinterpret_cast<uintptr_t>(o) + (orow + h) * esz;
            if (addr & (4 * esz - 1)) {  // a caller's buffer at an odd element offset
#pragma unroll
                for (int j = 0; j < 4; ++j) store_from_float(o, out_dtype, orow + h + j, v[j]);
            } else if (out_dtype == KQ_DT_F32) {
                *reinterpret_cast<float4*>(static_cast<float*>(o) + orow + h) = make_float4(v[0], v[1], v[2], v[3]);
            } else {
                // the four values in one 8-byte store (rows written to another GPU cross
                // NVLink as whole sectors rather than as 2-byte pieces)
                uint32_t w0, w1;
                if (out_dtype == KQ_DT_F16) {
                    const __half2 a = __floats2half2_rn(v[0], v[1]), b = __floats2half2_rn(v[2], v[3]);
                    w0 = *reinterpret_cast<const uint32_t*>(&a);
                    w1 = *reinterpret_cast<const uint32_t*>(&b);
                } else {
                    const __nv_bfloat162 a = __floats2bfloat162_rn(v[0], v[1]), b = __floats2bfloat162_rn(v[2], v[3]);
                    w0 = *reinterpret_cast<const uint32_t*>(&a);
                    w1 = *reinterpret_cast<const uint32_t*>(&b);
                }
                *reinterpret_cast<uint2*>(static_cast<uint16_t*>(o) + orow + h) = make_uint2(w0, w1);
            }
        }
    }
    if (out_rows) {  // every thread of the CTA reaches this point
        const int any = __syncthreads_or(wrote ? 1 : 0);
        if (threadIdx.x == 0 && any) __threadfence_system();
    }
}

// ---- host ---------------------------------------------------------------------------------------

// Work chunks hold at most PF_CHUNK tokens of one expert (one MMA N box);
// expert segments in the sorted order start on multiples of PF_PAD positions.
// Positions: at most A + (PF_PAD - 1) E.
constexpr int PF_CHUNK = 128;
constexpr int PF_PAD = 1;

struct PrefillWs {
    size_t status, idx, w, count, offset, chunks, n_chunks, n_pos, s_tok, inv_pos, xinv, Xs, act_s, ys;
    size_t act_flag, act_exp, act_inv, total;
    size_t pcap;  // position rows
};

static PrefillWs prefill_ws_layout(const kq_table* t, int T, int K) {
    auto al = [](size_t v) { return (v + 255) / 256 * 256; };
    const size_t A = (size_t)T * K, E = (size_t)t->d.num_experts;
    const size_t P = A + (PF_PAD - 1) * E;
    PrefillWs L{};
    L.pcap = P;
    size_t o = 0;
    L.status = o;
    o += 256;
    L.idx = o;
    o = al(o + A * 4);
    L.w = o;
    o = al(o + A * 4);
    L.count = o;
    o = al(o + E * 4);
    L.offset = o;
    o = al(o + E * 4);
    L.chunks = o;  // at most E + A / PF_CHUNK live chunks
    o = al(o + (E + A / PF_CHUNK + 1) * 16);
    L.n_chunks = o;
    o = al(o + 4);
    L.n_pos = o;
    o = al(o + 4);
    L.s_tok = o;
    o = al(o + P * 4);
    L.inv_pos = o;
    o = al(o + A * 4);
    L.xinv = o;
    o = al(o + P * 4);
    L.Xs = o;
    o = al(o + P * t->d.hidden * 2);
    L.act_s = o;
    o = al(o + P * t->d.inter * 2);
    L.ys = o;
    o = al(o + P * t->d.hidden * 4);
    L.act_flag = o;
    o = al(o + 4);
    L.act_exp = o;
    o = al(o + P * (t->d.inter / 16));
    L.act_inv = o;
    o = al(o + P * 4);
    L.total = o;
    return L;
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    if (!fn) {
        cudaDriverEntryPointQueryResult q;
        void* p = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
    return fn;
}

// fp16 row-major [rows][cols] tensor viewed as (64 columns of a group, row,
// group): boxes of 64 x box_rows x (128 / box_rows) groups (one 16 KB B stage),
// 128-byte swizzle; rows past `rows` read as zeros
static bool make_tmap(CUtensorMap* m, const void* base, int rows, int cols, int box_rows) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {64, (cuuint64_t)rows, (cuuint64_t)(cols / 64)};
    cuuint64_t strides[2] = {(cuuint64_t)cols * 2, 128};
    cuuint32_t box[3] = {64, (cuuint32_t)box_rows, (cuuint32_t)(128 / box_rows)};
    cuuint32_t es[3] = {1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// the layer's packed bytes as (128 bytes, 128-byte row, tile of a super-tile):
// rows 128 bytes apart, the 8 tiles of a super-tile nst * tile_bytes apart;
// boxes of 128 x (tile_bytes / 128) x 8 -- a whole super-tile -- 128-byte swizzle
static bool make_kq_tmap(CUtensorMap* m, const void* layer, size_t layer_bytes, int tile_bytes, int nst) {
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[3] = {128, (cuuint64_t)(layer_bytes / 128), 8};
    cuuint64_t strides[2] = {128, (cuuint64_t)nst * tile_bytes};
    cuuint32_t box[3] = {128, (cuuint32_t)(tile_bytes / 128), 8};
    cuuint32_t es[3] = {1, 1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(layer), dims, strides, box, es,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}


template <int BITS, int SB_DT>
static cudaError_t launch_tc_t(const TcParams& p, const CUtensorMap (&tm)[4], const CUtensorMap& tkq, cudaStream_t s,
                               int grid) {
    static int configured[64] = {0};
    auto kern = moe_tc_kernel<BITS, SB_DT>;
    const size_t smem = tc_smem_bytes<BITS>();
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if ((size_t)configured[dev] < smem) {
        cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (err != cudaSuccess) return err;
        configured[dev] = (int)smem;
    }
    return launch_dep(kern, dim3(grid), dim3(TC_THREADS), smem, s, p, tm[0], tm[1], tm[2], tm[3], tkq);
}

static cudaError_t launch_tc(int bits, int sb, const TcParams& p, const CUtensorMap (&tm)[4], const CUtensorMap& tkq,
                             cudaStream_t s, int grid) {
    if (bits == 3)
        return sb == KQ_DT_F16 ? launch_tc_t<3, KQ_DT_F16>(p, tm, tkq, s, grid)
                               : launch_tc_t<3, KQ_DT_BF16>(p, tm, tkq, s, grid);
    return sb == KQ_DT_F16 ? launch_tc_t<4, KQ_DT_F16>(p, tm, tkq, s, grid)
                           : launch_tc_t<4, KQ_DT_BF16>(p, tm, tkq, s, grid);
}

int launch_router_ext(const float* logits, int T, int E, int K, int32_t* idx, float* w, cudaStream_t s);

// A failed launch or tensor-map encode of the prefill path: one stderr line, KQ_ERR_CUDA.
static int pf_fail(const char* what, cudaError_t e = cudaSuccess) {
    fprintf(stderr, "[kq] prefill: %s failed%s%s\n", what, e != cudaSuccess ? ": " : "",
            e != cudaSuccess ? cudaGetErrorString(e) : "");
    return KQ_ERR_CUDA;
}

}  // namespace kq

using namespace kq;

extern "C" size_t kq_moe_prefill_workspace_size(const kq_table* t, int max_tokens, int top_k) {
    if (!t || max_tokens < 0 || top_k <= 0) return 0;
    return prefill_ws_layout(t, max_tokens, top_k).total;
}

extern "C" int kq_moe_prefill(const kq_table* t, int layer, const void* x, int x_dtype, int T, const float* logits,
                              int32_t* idx, float* weights, int K, void* out_per_k, void* out, int out_dtype,
                              const void* residual, void* workspace, size_t workspace_bytes, void* stream) {
    return kq::moe_prefill_ex(t, layer, x, x_dtype, T, logits, idx, weights, K, out_per_k, out, out_dtype, residual,
                              nullptr, workspace, workspace_bytes, stream);
}

int kq::moe_prefill_ex(const kq_table* t, int layer, const void* x, int x_dtype, int T, const float* logits,
                       int32_t* idx, float* weights, int K, void* out_per_k, void* out, int out_dtype,
                       const void* residual, void* const* out_rows, void* workspace, size_t workspace_bytes,
                       void* stream) {
    if (!t) return KQ_ERR_ARG;
    if (layer < 0 || layer >= t->d.num_layers) return KQ_ERR_ARG;
    if (T < 0 || K <= 0 || K > 32 || K > t->d.num_experts) return KQ_ERR_ARG;
    if (T == 0) return KQ_OK;
    if (!x || (x_dtype != KQ_DT_F16 && x_dtype != KQ_DT_BF16 && x_dtype != KQ_DT_F32)) return KQ_ERR_ARG;
    if (out_dtype != KQ_DT_F16 && out_dtype != KQ_DT_BF16 && out_dtype != KQ_DT_F32) return KQ_ERR_ARG;
    if (!logits && !idx) return KQ_ERR_ARG;
    if ((out || out_rows) && !weights && !logits) return KQ_ERR_ARG;
    if (!out && !out_per_k && !out_rows) return KQ_ERR_ARG;
    if (logits && t->d.num_experts > 1024) return KQ_ERR_UNSUPPORTED;
    if (t->d.num_experts > GROUP_MAX_E) return KQ_ERR_UNSUPPORTED;
    if (t->d.hidden % 512 || t->d.inter % 512) return KQ_ERR_UNSUPPORTED;  // whole 512-wide super-tiles
    if (!workspace) return KQ_ERR_WORKSPACE;
    const PrefillWs L = prefill_ws_layout(t, T, K);
    if (workspace_bytes < L.total) return KQ_ERR_WORKSPACE;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int A = T * K, E = t->d.num_experts, H = t->d.hidden, I = t->d.inter;
    int32_t* idx_use = idx ? idx : reinterpret_cast<int32_t*>(ws + L.idx);
    float* w_use = weights ? weights : reinterpret_cast<float*>(ws + L.w);
    uint32_t* status = reinterpret_cast<uint32_t*>(ws + L.status);
    int* count = reinterpret_cast<int*>(ws + L.count);
    int* offset = reinterpret_cast<int*>(ws + L.offset);
    int4* chunk_list = reinterpret_cast<int4*>(ws + L.chunks);
    int* n_chunks = reinterpret_cast<int*>(ws + L.n_chunks);
    int* n_pos = reinterpret_cast<int*>(ws + L.n_pos);
    int32_t* s_tok = reinterpret_cast<int32_t*>(ws + L.s_tok);
    int32_t* inv_pos = reinterpret_cast<int32_t*>(ws + L.inv_pos);
    float* xinv = reinterpret_cast<float*>(ws + L.xinv);
    __half* Xs = reinterpret_cast<__half*>(ws + L.Xs);
    __half* act_s = reinterpret_cast<__half*>(ws + L.act_s);
    float* ys = reinterpret_cast<float*>(ws + L.ys);
    uint32_t* act_flag = reinterpret_cast<uint32_t*>(ws + L.act_flag);
    int8_t* act_exp = reinterpret_cast<int8_t*>(ws + L.act_exp);
    float* act_inv = reinterpret_cast<float*>(ws + L.act_inv);
    const int P = (int)L.pcap;

    if (logits && launch_router_ext(logits, T, E, K, idx_use, w_use, s) != KQ_OK) return KQ_ERR_CUDA;
    {
        const int threads = 256;
        if (cudaError_t e = launch_dep(group_kernel, dim3(1), dim3(GROUP_THREADS), 0, s, (const int32_t*)idx_use, A,
                                       K, E, PF_CHUNK, PF_PAD, count, offset, s_tok, inv_pos, chunk_list, n_chunks,
                                       n_pos, status, act_flag))
            return pf_fail("grouping", e);
        if (cudaError_t e = launch_dep(gather_kernel, dim3((P * 32 + threads - 1) / threads), dim3(threads), 0, s, x,
                                       x_dtype, H, (const int32_t*)s_tok, (const int*)n_pos, Xs, xinv, act_exp, I / 16))
            return pf_fail("gather", e);
    }
    // Rows of Xs / act_s at pad positions or past the placed ones are never
    // written; the epilogues ignore the MMA columns that read them.
    int nsm = 148;
    {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev);
    }
    const uint8_t* layer_base = t->base + (size_t)layer * t->layer_bytes;
    if ((reinterpret_cast<uintptr_t>(layer_base) & 127) || (t->layer_bytes & 127) || (t->expert_bytes & 127) ||
        (t->gateup_bytes & 127) || (t->tb & 127))
        return KQ_ERR_UNSUPPORTED;  // tiles must start on 128-byte rows
    const int max_chunks = E + A / PF_CHUNK + 1;  // live chunks: sum over experts of ceil(n_e / PF_CHUNK)
    TcParams p{};
    p.base = layer_base;
    p.expert_bytes = t->expert_bytes;
    p.E = E;
    p.count = count;
    p.offset = offset;
    p.chunk_list = chunk_list;
    p.n_chunks = n_chunks;
    p.act_s = act_s;
    p.I = I;
    p.ys = ys;
    p.H = H;
    p.xinv = x_dtype == KQ_DT_F16 ? nullptr : xinv;
    p.act_kind = t->d.activation;
    p.status = status;
    p.act_flag = act_flag;
    p.act_exp = act_exp;
    p.act_inv = act_inv;
    const int boxes[4] = {16, 32, 64, 128};
    // One grouped GEMM over `src` [P][Kdim].
    auto gemm = [&](const __half* src, int Kdim) -> int {
        p.nst = Kdim / 512;
        const int items = max_chunks * p.n_mt;  // upper bound; the kernel reads the live count
        const int grid = std::min(items, nsm);
        CUtensorMap tkq;
        if (!make_kq_tmap(&tkq, layer_base, t->layer_bytes, (int)t->tb, p.nst)) return pf_fail("tile tensor map");
        CUtensorMap tm[4];
        for (int i = 0; i < 4; ++i)
            if (!make_tmap(&tm[i], src, P, Kdim, boxes[i])) return pf_fail("token tensor map");
        if (cudaError_t e = launch_tc(t->d.bits, t->d.sb_dtype, p, tm, tkq, s, grid))
            return pf_fail("grouped GEMM", e);
        return KQ_OK;
    };
    // gate/up + activation
    p.mode = 0;
    p.mat_off = 0;
    p.n_mt = I / 64;
    if (int rc = gemm(Xs, H)) return rc;
    if (cudaError_t e = launch_dep(act_fixup_kernel, dim3(nsm), dim3(256), 0, s, (const uint32_t*)act_flag,
                                   (const int8_t*)act_exp, act_s, act_inv, (const int*)n_pos, I))
        return pf_fail("activation range pass", e);
    // down
    p.mode = 1;
    p.mat_off = t->gateup_bytes;
    p.n_mt = H / 128;
    if (int rc = gemm(act_s, I)) return rc;
    // combine / per-k outputs (rows going to other GPUs: at most 128 CTA rows, so
    // a CTA fences once after several rows)
    dim3 grid((H / 4 + 255) / 256, out_rows ? std::min(T, 128) : T);
    return launch_dep(combine_kernel, grid, dim3(256), 0, s, (const float*)ys, (const int32_t*)inv_pos,
                      (const float*)w_use, T, K, H, out, out_per_k, out_dtype, residual, out_rows) == cudaSuccess
               ? KQ_OK
               : KQ_ERR_CUDA;
}
