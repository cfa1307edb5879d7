// kq_qtile.cuh -- the HBM tile layout of quantized matrices and the
// dequant-GEMV engine that consumes it.
//
// TILE LAYOUT ("KQ tile").  A quantized matrix [rows][cols] (MLX affine,
// group 64, 3 or 4 bits) is cut into tiles of 16 rows x 512 columns
// (8 groups).  A tile is 32 lanes' worth of 16-byte chunks, chunk-major:
//     byte offset of lane l's chunk c  =  c * 512 + l * 16
// so a warp reading chunk c reads 512 contiguous bytes (coalesced, and bank-
// conflict-free from shared memory).  Lane l = 4*r + t (r = l/4, t = l%4)
// owns four (row, group) "sets":
//     set 0 = (row r,   group t)     set 1 = (row r,   group t+4)
//     set 2 = (row r+8, group t)     set 3 = (row r+8, group t+4)
// W = 6 (3-bit) or 8 (4-bit) 32-bit words per set; lane word q = set*W + w
// lives in chunk q/4, position q%4.  After the 4*W/4 = W code chunks comes one
// scale/bias chunk: lane l holds (scale | bias<<16) for
//     (row r, group 2t), (row r, group 2t+1), (row r+8, group 2t), (row r+8, group 2t+1).
// Tile bytes: 3584 (3-bit) or 4608 (4-bit) -- exactly 16*512*(bits/8 + 4/64),
// the same bytes per weight as the MLX layout.
//
// Within a set, code i (0..63 of the group) is half (i%2) of pair j = i/2.
// 3-bit: pair j < 30 sits in word j/5, slot s = j%5: low code at bit 3s, high
//        code at bit 16+3s; pairs 30 and 31 are spread over bit 15 (low) and
//        bit 31 (high) of words 0-2 and 3-5 (bit b of the code in word b).
// 4-bit: pair j sits in word j/4, slot s = j%4: low at bit 4s, high at 16+4s.
// One LOP3 per pair ((word >> shift) & mask | magic) yields two fp16 values
// 2^(10-k) + q exactly (k = field offset inside the 16-bit half), i.e. an
// fp16x2 A-fragment register of the m16n8k16 MMA.  The constant 2^(10-k) per
// pair is removed once per group through C[g] = sum_pairs 2^(10-k) (x_a + x_b).
//
// MMA MAPPING.  MMA j (0..31) of a tile takes pair j of every set:
//     a0 = set 0, a1 = set 2, a2 = set 1, a3 = set 3,
// i.e. A[m][k] with k in {2t,2t+1} -> group t and k in {2t+8,2t+9} -> group t+4.
// B[k][n] = x (pair j of group n) where group(k) == n, 0 elsewhere, so column n
// of D accumulates the dot product of group n alone: after 32 MMAs
//     D[m][n] = sum_{i in group n} (2^(10-k_i) + q_{m,i}) x_i
// and the per-group affine terms are applied once:
//     y_m += s_{m,n} (D[m][n] - C[n]) + b_{m,n} X[n],   X[n] = sum_{i in n} x_i.
// Each lane ends with partial sums over its groups 2t, 2t+1 for rows r, r+8;
// two xor-shuffles finish the row dot products.
#pragma once

#include "kq_common.cuh"

namespace kq {

constexpr int TILE_ROWS = 16;
constexpr int TILE_COLS = 512;
constexpr int TILE_GROUPS = 8;
constexpr int GS = 64;

template <int BITS>
struct TileT {
    static constexpr int W = (BITS == 3) ? 6 : 8;  // words per (row, group) set
    static constexpr int CODE_CHUNKS = W;          // 4 sets * W words / 4 words per chunk
    static constexpr int CHUNKS = W + 1;
    static constexpr int BYTES = CHUNKS * 512;
};

__host__ __device__ constexpr int tile_bytes(int bits) { return bits == 3 ? 3584 : 4608; }

// offset constant 2^(10-k) of pair j (fp32)
template <int BITS>
__host__ __device__ __forceinline__ constexpr float pair_offset(int j) {
    if (BITS == 3) {
        if (j >= 30) return 1024.f;
        int s = j % 5;
        return s == 0 || s == 3 ? 1024.f : (s == 1 || s == 4 ? 128.f : 16.f);
    } else {
        return (j & 1) ? 64.f : 1024.f;
    }
}

// (a & b) | c as ONE three-input logic operation.  Written as C, the mask and
// the exponent pattern of a code pair could compile to separate AND and OR
// instructions; pinned to a single lop3 the batched decode went from 4.23 to
// 3.64 µs per token-layer (same box, bit-identical results).
__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// fp16 exponent pattern with value 2^(10-k) in both halves
__device__ __forceinline__ constexpr uint32_t magic2(int k) {
    return ((uint32_t)(25 - k) << 10) * 0x00010001u;
}

// Extract pair j of one set (words wd[0..W-1]; sh[] = words >> 9 (3-bit) or >> 8 (4-bit))
template <int BITS, int J>
__device__ __forceinline__ uint32_t pair_of(const uint32_t* wd, const uint32_t* sh) {
    if constexpr (BITS == 3) {
        if constexpr (J < 30) {
            constexpr int w = J / 5, s = J % 5;
            constexpr int k = (s < 3) ? 3 * s : 3 * (s - 3);
            constexpr uint32_t mask = (7u << k) | (7u << (16 + k));
            const uint32_t src = (s < 3) ? wd[w] : sh[w];
            return and_or(src, mask, magic2(k));
        } else {
            constexpr int b = (J - 30) * 3;
            uint32_t v = and_or(wd[b] >> 15, 0x00010001u, magic2(0));
            v = and_or(wd[b + 1] >> 14, 0x00020002u, v);
            return and_or(wd[b + 2] >> 13, 0x00040004u, v);
        }
    } else {
        constexpr int w = J / 4, s = J % 4;
        constexpr int k = (s & 1) * 4;
        constexpr uint32_t mask = (15u << k) | (15u << (16 + k));
        const uint32_t src = (s < 2) ? wd[w] : sh[w];
        return and_or(src, mask, magic2(k));
    }
}

// ---- input staging ---------------------------------------------------------------
// The engine consumes the input vector as fp16 x * 2^sigma in a per-warp shared
// buffer xs[npad] (zero-padded to a multiple of 512) plus per-group constants
// cx[g] = {C[g], X[g]}.  Loads are issued 8 elements (one 16/32-byte vector)
// per lane per chunk, BATCH chunks at a time, so a warp has all of them in
// flight instead of paying one memory latency per element.

// 8 consecutive elements starting at element i (i % 8 == 0) as floats.
__device__ __forceinline__ void load8(const void* p, int dtype, size_t i, bool cg, float (&v)[8]) {
    if (dtype == KQ_DT_F32) {
        const float4* q = reinterpret_cast<const float4*>(static_cast<const float*>(p) + i);
        const float4 a = cg ? __ldcg(q) : __ldg(q);
        const float4 b = cg ? __ldcg(q + 1) : __ldg(q + 1);
        v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
        v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
        return;
    }
    const uint4* q = reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(p) + i);
    const uint4 a = cg ? __ldcg(q) : __ldg(q);
    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        if (dtype == KQ_DT_F16) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[k]));
            v[2 * k] = f.x;
            v[2 * k + 1] = f.y;
        } else {
            v[2 * k] = __uint_as_float(w[k] << 16);
            v[2 * k + 1] = __uint_as_float(w[k] & 0xFFFF0000u);
        }
    }
}

constexpr int STAGE_BATCH = 4;

// max |x_i| and sum x_i^2 * (w_i^2 if w) over n elements (n % 8 == 0).
__device__ __forceinline__ void vec_stats(const void* x, int dtype, size_t off, int n, const void* w,
                                          bool cg, float& amax, float& sumsq) {
    const int lane = threadIdx.x & 31;
    const int nch = n / 8;
    amax = 0.f;
    sumsq = 0.f;
    for (int c0 = lane; c0 < nch; c0 += 32 * STAGE_BATCH) {
        float v[STAGE_BATCH][8];
        float wv[STAGE_BATCH][8];
#pragma unroll
        for (int b = 0; b < STAGE_BATCH; ++b) {
            const int c = c0 + 32 * b;
            if (c < nch) {
                load8(x, dtype, off + (size_t)c * 8, cg, v[b]);
                if (w) load8(w, dtype, (size_t)c * 8, false, wv[b]);
            } else {
#pragma unroll
                for (int k = 0; k < 8; ++k) v[b][k] = 0.f, wv[b][k] = 0.f;
            }
        }
#pragma unroll
        for (int b = 0; b < STAGE_BATCH; ++b)
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                sumsq += v[b][k] * v[b][k];
                amax = fmaxf(amax, fabsf(w ? v[b][k] * wv[b][k] : v[b][k]));
            }
    }
    amax = warp_max(amax);
    sumsq = warp_sum(sumsq);
}

// power-of-two scale that puts amax in [2^14, 2^15) (1 if amax is 0 or not finite)
__device__ __forceinline__ float pow2_scale(float amax) {
    if (!(amax > 0.f) || !(amax < 3.0e38f)) return 1.f;
    int e = 0;
    frexpf(amax, &e);
    return ldexpf(1.f, 15 - e);
}

// xs[i] = fp16(x[off + i] * mul * (w ? w[i] : 1)), zero beyond n; then cx.  Whole warp.
template <int BITS>
__device__ __forceinline__ void stage_vector(const void* x, int dtype, size_t off, int n, int npad,
                                             const void* w, float mul, bool cg, __half* xs, float2* cx) {
    const int lane = threadIdx.x & 31;
    const int nch = n / 8, npch = npad / 8;
    for (int c0 = lane; c0 < npch; c0 += 32 * STAGE_BATCH) {
        float v[STAGE_BATCH][8];
        float wv[STAGE_BATCH][8];
#pragma unroll
        for (int b = 0; b < STAGE_BATCH; ++b) {
            const int c = c0 + 32 * b;
            if (c < nch) {
                load8(x, dtype, off + (size_t)c * 8, cg, v[b]);
                if (w) load8(w, dtype, (size_t)c * 8, false, wv[b]);
            } else {
#pragma unroll
                for (int k = 0; k < 8; ++k) v[b][k] = 0.f, wv[b][k] = 1.f;
            }
        }
#pragma unroll
        for (int b = 0; b < STAGE_BATCH; ++b) {
            const int c = c0 + 32 * b;
            if (c < npch) {
                uint32_t h[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    float a = v[b][2 * k] * mul, bb = v[b][2 * k + 1] * mul;
                    if (w) a *= wv[b][2 * k], bb *= wv[b][2 * k + 1];
                    const __half2 hh = __floats2half2_rn(a, bb);
                    h[k] = *reinterpret_cast<const uint32_t*>(&hh);
                }
                *reinterpret_cast<uint4*>(xs + (size_t)c * 8) = make_uint4(h[0], h[1], h[2], h[3]);
            }
        }
    }
    __syncwarp();
    const int ng = npad / GS;
    for (int g = lane; g < ng; g += 32) {
        const __half2* p = reinterpret_cast<const __half2*>(xs + g * GS);
        float c = 0.f, xsum = 0.f;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
            const float2 f = __half22float2(p[j]);
            const float pr = f.x + f.y;
            c += pair_offset<BITS>(j) * pr;
            xsum += pr;
        }
        cx[g] = make_float2(c, xsum);
    }
    __syncwarp();
}

// ---- fused staging: fp16 conversion + per-group constants in one pass -------------
// A chunk is 8 consecutive inputs = 4 pairs; group g holds chunks 8g..8g+7 and
// chunk c covers pairs 4*(c%8) .. 4*(c%8)+3 of group c/8.  Threads that stage
// chunk c also produce its part of C[g] and X[g] (from the fp16 values the MMA
// will read); 8 consecutive ranks hold the 8 chunks of a group and finish the
// sums with three shuffles.  `rank` is the thread's index among `nthr`
// participating threads (nthr a multiple of 32), so c % 8 == rank % 8.

template <int BITS>
__device__ __forceinline__ float chunk_offset(int c8, int k) {
    return pair_offset<BITS>(4 * c8 + k);
}

// scaled floats -> fp16 chunk c of xs; returns (C part, X part) of the chunk
template <int BITS>
__device__ __forceinline__ float2 store_chunk(const float (&v)[8], float mul, const float (&off)[4],
                                              __half* xs, int c) {
    uint32_t h[4];
    float cc = 0.f, xx = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const __half2 hh = __floats2half2_rn(v[2 * k] * mul, v[2 * k + 1] * mul);
        h[k] = *reinterpret_cast<const uint32_t*>(&hh);
        const float2 f = __half22float2(hh);
        const float pr = f.x + f.y;
        cc += off[k] * pr;
        xx += pr;
    }
    *reinterpret_cast<uint4*>(xs + (size_t)c * 8) = make_uint4(h[0], h[1], h[2], h[3]);
    return make_float2(cc, xx);
}

// reduce a chunk's (C, X) over the 8 ranks of its group; rank%8 == 0 stores cx[g]
__device__ __forceinline__ void group_reduce_store(float2 v, int rank, int c, float2* cx, unsigned mask) {
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
        v.x += __shfl_xor_sync(mask, v.x, o);
        v.y += __shfl_xor_sync(mask, v.y, o);
    }
    if ((rank & 7) == 0) cx[c >> 3] = v;
}

// Stage n elements of `src` (dtype, starting at element `off`) times `mul` into
// xs (zero-padded to npad) and cx.  Called by `nthr` threads with ranks 0..nthr-1
// (whole warps); loads of a thread's chunks are issued before any is used.
template <int BITS, int MAXB>
__device__ __forceinline__ void stage_fused(const void* src, int dtype, size_t off, int n, int npad,
                                            float mul, bool cg, int rank, int nthr, __half* xs,
                                            float2* cx, const void* w2 = nullptr) {
    const int nch = n / 8, npch = npad / 8;
    float offv[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) offv[k] = chunk_offset<BITS>(rank & 7, k);
    for (int c0 = rank; c0 < npch; c0 += nthr * MAXB) {
        float v[MAXB][8];
#pragma unroll
        for (int b = 0; b < MAXB; ++b) {
            const int c = c0 + b * nthr;
            if (c < nch) {
                load8(src, dtype, off + (size_t)c * 8, cg, v[b]);
                if (w2) {
                    float wv[8];
                    load8(w2, dtype, (size_t)c * 8, false, wv);
#pragma unroll
                    for (int k = 0; k < 8; ++k) v[b][k] *= wv[k];
                }
            } else {
#pragma unroll
                for (int k = 0; k < 8; ++k) v[b][k] = 0.f;
            }
        }
#pragma unroll
        for (int b = 0; b < MAXB; ++b) {
            const int c = c0 + b * nthr;
            // npch is a multiple of 64 and ranks come in whole warps, so `c < npch`
            // is uniform across a warp and the full-warp shuffles are safe
            if (c < npch) {
                const float2 part = store_chunk<BITS>(v[b], mul, offv, xs, c);
                group_reduce_store(part, rank, c, cx, 0xffffffffu);
            }
        }
    }
}

// MMA steps J..31 of a tile (compile-time recursion: every pair extraction
// uses constant masks and shifts).  x pairs J..J+3 arrive in one 16-byte load.
// Two accumulator sets (pair index parity) halve the dependent MMA chain.
template <int BITS, int J>
__device__ __forceinline__ void mma_steps(float (&d)[2][4], const uint32_t (&wd)[4][TileT<BITS>::W],
                                          const uint32_t (&sh)[4][TileT<BITS>::W],
                                          const uint4* xp, bool has_x, bool use_b0, bool use_b1) {
    if constexpr (J < 32) {
        const uint4 xv = has_x ? xp[J / 4] : make_uint4(0u, 0u, 0u, 0u);
        const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            // u is a compile-time constant after unrolling; pair index J + u
            const uint32_t b0 = use_b0 ? xw[u] : 0u;
            const uint32_t b1 = use_b1 ? xw[u] : 0u;
            uint32_t a0, a1, a2, a3;
            if (u == 0) {
                a0 = pair_of<BITS, J + 0>(wd[0], sh[0]); a1 = pair_of<BITS, J + 0>(wd[2], sh[2]);
                a2 = pair_of<BITS, J + 0>(wd[1], sh[1]); a3 = pair_of<BITS, J + 0>(wd[3], sh[3]);
            } else if (u == 1) {
                a0 = pair_of<BITS, J + 1>(wd[0], sh[0]); a1 = pair_of<BITS, J + 1>(wd[2], sh[2]);
                a2 = pair_of<BITS, J + 1>(wd[1], sh[1]); a3 = pair_of<BITS, J + 1>(wd[3], sh[3]);
            } else if (u == 2) {
                a0 = pair_of<BITS, J + 2>(wd[0], sh[0]); a1 = pair_of<BITS, J + 2>(wd[2], sh[2]);
                a2 = pair_of<BITS, J + 2>(wd[1], sh[1]); a3 = pair_of<BITS, J + 2>(wd[3], sh[3]);
            } else {
                a0 = pair_of<BITS, J + 3>(wd[0], sh[0]); a1 = pair_of<BITS, J + 3>(wd[2], sh[2]);
                a2 = pair_of<BITS, J + 3>(wd[1], sh[1]); a3 = pair_of<BITS, J + 3>(wd[3], sh[3]);
            }
            mma_f16(d[u & 1], a0, a1, a2, a3, b0, b1);
        }
        mma_steps<BITS, J + 4>(d, wd, sh, xp, has_x, use_b0, use_b1);
    }
}

// Registers of one tile for this lane: its 4 sets of code words + scale/bias chunk.
template <int BITS>
struct TileRegs {
    uint32_t wd[4][TileT<BITS>::W];
    uint4 sb;
};

// Load this lane's part of a tile (16 rows x 512 cols) from shared memory.
template <int BITS>
__device__ __forceinline__ void tile_load(const uint8_t* tile, TileRegs<BITS>& R) {
    constexpr int W = TileT<BITS>::W;
    const int lane = threadIdx.x & 31;
    const uint4* ch = reinterpret_cast<const uint4*>(tile) + lane;  // chunk c at ch[c * 32]
#pragma unroll
    for (int c = 0; c < W; ++c) {
        const uint4 v = ch[c * 32];
        const int q0 = c * 4;
        R.wd[(q0 + 0) / W][(q0 + 0) % W] = v.x;
        R.wd[(q0 + 1) / W][(q0 + 1) % W] = v.y;
        R.wd[(q0 + 2) / W][(q0 + 2) % W] = v.z;
        R.wd[(q0 + 3) / W][(q0 + 3) % W] = v.w;
    }
    R.sb = ch[W * 32];
}

// 32 MMAs + per-group epilogue of one tile; st = column-tile index of the tile.
// Accumulates into y0 (row r) and y1 (row r+8) of this lane's partial sums.
template <int BITS, int SB_DT>
__device__ __forceinline__ void tile_compute(const TileRegs<BITS>& R, int st, const __half* xs,
                                             const float2* cxv, float& y0, float& y1) {
    constexpr int W = TileT<BITS>::W;
    const int lane = threadIdx.x & 31;
    const int n = lane >> 2, t = lane & 3;
    uint32_t sh[4][W];
#pragma unroll
    for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int w = 0; w < W; ++w) sh[q][w] = R.wd[q][w] >> (BITS == 3 ? 9 : 8);

    // B operand: lane (n, t) feeds b0 for group t when n == t, b1 for group t+4 when n == t+4.
    const bool use_b0 = (n == t), use_b1 = (n == t + 4);
    const int xg = use_b0 ? t : (use_b1 ? t + 4 : 0);
    const uint4* xp = reinterpret_cast<const uint4*>(xs + st * TILE_COLS + xg * GS);

    float acc[2][4] = {};
    mma_steps<BITS, 0>(acc, R.wd, sh, xp, use_b0 || use_b1, use_b0, use_b1);
    float d[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) d[i] = acc[0][i] + acc[1][i];

    // epilogue: groups G0 = 2t, G1 = 2t+1 of this column tile
    const float4 cx = *reinterpret_cast<const float4*>(cxv + st * TILE_GROUPS + 2 * t);
    const uint4 sb = R.sb;
    y0 += sb_lo<SB_DT>(sb.x) * (d[0] - cx.x) + sb_hi<SB_DT>(sb.x) * cx.y;
    y0 += sb_lo<SB_DT>(sb.y) * (d[1] - cx.z) + sb_hi<SB_DT>(sb.y) * cx.w;
    y1 += sb_lo<SB_DT>(sb.z) * (d[2] - cx.x) + sb_hi<SB_DT>(sb.z) * cx.y;
    y1 += sb_lo<SB_DT>(sb.w) * (d[3] - cx.z) + sb_hi<SB_DT>(sb.w) * cx.w;
}

// ---- padded input layout ---------------------------------------------------------
// A variant of the engine for kernels whose warps each run long sequences of
// tiles.  The staged input keeps each 64-wide group in a row of PAD_ROW bytes
// (128 of data + 16 of padding), so the eight groups a warp reads at once
// start in eight different 16-byte bank windows; and each lane reads its B
// operand halves through two pointers -- its own group's row, or a zero row
// -- instead of selecting between x and 0 at every step.
constexpr int PAD_ROW = 144;                  // bytes per staged group row
constexpr int PAD_HALFS = PAD_ROW / 2;        // 72 halves

__host__ __device__ constexpr size_t pad_bytes(int npad) { return (size_t)(npad / GS) * PAD_ROW; }

// chunk c (8 consecutive inputs) of a padded staged vector
__device__ __forceinline__ __half* pad_chunk(__half* xs, int c) { return xs + (c >> 3) * PAD_HALFS + (c & 7) * 8; }

// store_chunk into the padded layout; returns (C part, X part) as store_chunk
template <int BITS>
__device__ __forceinline__ float2 store_chunk_pad(const float (&v)[8], float mul, const float (&off)[4],
                                                  __half* xs, int c) {
    uint32_t h[4];
    float cc = 0.f, xx = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const __half2 hh = __floats2half2_rn(v[2 * k] * mul, v[2 * k + 1] * mul);
        h[k] = *reinterpret_cast<const uint32_t*>(&hh);
        const float2 f = __half22float2(hh);
        const float pr = f.x + f.y;
        cc += off[k] * pr;
        xx += pr;
    }
    *reinterpret_cast<uint4*>(pad_chunk(xs, c)) = make_uint4(h[0], h[1], h[2], h[3]);
    return make_float2(cc, xx);
}

// stage_fused into the padded layout (same arguments and rules)
template <int BITS, int MAXB>
__device__ __forceinline__ void stage_fused_pad(const void* src, int dtype, size_t off, int n, int npad, float mul,
                                                bool cg, int rank, int nthr, __half* xs, float2* cx,
                                                const void* w2 = nullptr) {
    const int nch = n / 8, npch = npad / 8;
    float offv[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) offv[k] = chunk_offset<BITS>(rank & 7, k);
    for (int c0 = rank; c0 < npch; c0 += nthr * MAXB) {
        float v[MAXB][8];
#pragma unroll
        for (int b = 0; b < MAXB; ++b) {
            const int c = c0 + b * nthr;
            if (c < nch) {
                load8(src, dtype, off + (size_t)c * 8, cg, v[b]);
                if (w2) {
                    float wv[8];
                    load8(w2, dtype, (size_t)c * 8, false, wv);
#pragma unroll
                    for (int k = 0; k < 8; ++k) v[b][k] *= wv[k];
                }
            } else {
#pragma unroll
                for (int k = 0; k < 8; ++k) v[b][k] = 0.f;
            }
        }
#pragma unroll
        for (int b = 0; b < MAXB; ++b) {
            const int c = c0 + b * nthr;
            if (c < npch) {  // warp-uniform: npch is a multiple of 64, ranks come in whole warps
                const float2 part = store_chunk_pad<BITS>(v[b], mul, offv, xs, c);
                group_reduce_store(part, rank, c, cx, 0xffffffffu);
            }
        }
    }
}

// MMA steps J..31 with B from two padded rows (x0: this lane's b0 row or the
// zero row, x1: its b1 row or the zero row) and four accumulator chains.
template <int BITS, int J>
__device__ __forceinline__ void mma_steps_pad(float (&d)[4][4], const uint32_t (&wd)[4][TileT<BITS>::W],
                                              const uint32_t (&sh)[4][TileT<BITS>::W], const uint4* x0,
                                              const uint4* x1) {
    if constexpr (J < 32) {
        const uint4 v0 = x0[J / 4], v1 = x1[J / 4];
        const uint32_t b0[4] = {v0.x, v0.y, v0.z, v0.w};
        const uint32_t b1[4] = {v1.x, v1.y, v1.z, v1.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            uint32_t a0, a1, a2, a3;
            if (u == 0) {
                a0 = pair_of<BITS, J + 0>(wd[0], sh[0]); a1 = pair_of<BITS, J + 0>(wd[2], sh[2]);
                a2 = pair_of<BITS, J + 0>(wd[1], sh[1]); a3 = pair_of<BITS, J + 0>(wd[3], sh[3]);
            } else if (u == 1) {
                a0 = pair_of<BITS, J + 1>(wd[0], sh[0]); a1 = pair_of<BITS, J + 1>(wd[2], sh[2]);
                a2 = pair_of<BITS, J + 1>(wd[1], sh[1]); a3 = pair_of<BITS, J + 1>(wd[3], sh[3]);
            } else if (u == 2) {
                a0 = pair_of<BITS, J + 2>(wd[0], sh[0]); a1 = pair_of<BITS, J + 2>(wd[2], sh[2]);
                a2 = pair_of<BITS, J + 2>(wd[1], sh[1]); a3 = pair_of<BITS, J + 2>(wd[3], sh[3]);
            } else {
                a0 = pair_of<BITS, J + 3>(wd[0], sh[0]); a1 = pair_of<BITS, J + 3>(wd[2], sh[2]);
                a2 = pair_of<BITS, J + 3>(wd[1], sh[1]); a3 = pair_of<BITS, J + 3>(wd[3], sh[3]);
            }
            mma_f16(d[u], a0, a1, a2, a3, b0[u], b1[u]);
        }
        mma_steps_pad<BITS, J + 4>(d, wd, sh, x0, x1);
    }
}

// tile_compute on a padded staged input; zrow: PAD_ROW zero bytes (16-byte aligned)
template <int BITS, int SB_DT>
__device__ __forceinline__ void tile_compute_pad(const TileRegs<BITS>& R, int st, const __half* xs,
                                                 const float2* cxv, const __half* zrow, float& y0, float& y1) {
    constexpr int W = TileT<BITS>::W;
    const int lane = threadIdx.x & 31;
    const int n = lane >> 2, t = lane & 3;
    uint32_t sh[4][W];
#pragma unroll
    for (int q = 0; q < 4; ++q)
#pragma unroll
        for (int w = 0; w < W; ++w) sh[q][w] = R.wd[q][w] >> (BITS == 3 ? 9 : 8);
    // B operand: lane (n, t) feeds b0 for group t when n == t, b1 for group t+4 when n == t+4
    const __half* row = xs + (size_t)st * TILE_GROUPS * PAD_HALFS;
    const uint4* x0 = reinterpret_cast<const uint4*>(n == t ? row + t * PAD_HALFS : zrow);
    const uint4* x1 = reinterpret_cast<const uint4*>(n == t + 4 ? row + (t + 4) * PAD_HALFS : zrow);
    float acc[4][4] = {};
    mma_steps_pad<BITS, 0>(acc, R.wd, sh, x0, x1);
    float d[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) d[i] = (acc[0][i] + acc[1][i]) + (acc[2][i] + acc[3][i]);
    const float4 cx = *reinterpret_cast<const float4*>(cxv + st * TILE_GROUPS + 2 * t);
    const uint4 sb = R.sb;
    y0 += sb_lo<SB_DT>(sb.x) * (d[0] - cx.x) + sb_hi<SB_DT>(sb.x) * cx.y;
    y0 += sb_lo<SB_DT>(sb.y) * (d[1] - cx.z) + sb_hi<SB_DT>(sb.y) * cx.w;
    y1 += sb_lo<SB_DT>(sb.z) * (d[2] - cx.x) + sb_hi<SB_DT>(sb.z) * cx.y;
    y1 += sb_lo<SB_DT>(sb.w) * (d[3] - cx.z) + sb_hi<SB_DT>(sb.w) * cx.w;
}

// finish the row dot products across the 4 lanes of a quad
__device__ __forceinline__ void quad_reduce(float& y0, float& y1) {
    y0 += __shfl_xor_sync(0xffffffffu, y0, 1);
    y1 += __shfl_xor_sync(0xffffffffu, y1, 1);
    y0 += __shfl_xor_sync(0xffffffffu, y0, 2);
    y1 += __shfl_xor_sync(0xffffffffu, y1, 2);
}

__device__ __forceinline__ float activate(float g, float u, int act) {
    if (act == KQ_ACT_GELU_TANH) {
        float tt = 0.7978845608f * (g + 0.044715f * g * g * g);
        return 0.5f * g * (1.f + tanhf(tt)) * u;
    }
    return (g / (1.f + expf(-g))) * u;
}

// ---- layout index helpers shared by the repack / unpack kernels ----------------
// Location of code (tile-local row m in 0..15, column i in 0..511) inside a tile.
struct CodeLoc {
    int lane, set, pair, hi;
};
__host__ __device__ __forceinline__ CodeLoc code_loc(int m, int i) {
    const int g8 = i / GS, ci = i % GS;
    CodeLoc L;
    L.lane = (m & 7) * 4 + (g8 & 3);
    L.set = (m >> 3) * 2 + (g8 >> 2);
    L.pair = ci >> 1;
    L.hi = ci & 1;
    return L;
}

__host__ __device__ __forceinline__ uint32_t tile_word_offset(int lane, int q) {
    return (uint32_t)((q >> 2) * 512 + lane * 16 + (q & 3) * 4);
}

}  // namespace kq
