// kq_route.cuh -- device helpers shared by the routed-expert decode kernels:
// softmax top-K on one warp (kandiga/metal/moe_block.metal:419-505), named
// barriers, and the warp-level staging of a down-projection input.
#pragma once

#include "kq_qtile.cuh"

namespace kq {

__device__ __forceinline__ void named_barrier_sync(int id, int nthr) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthr) : "memory");
}

// ---- routing ------------------------------------------------------------------------

// Order-preserving 32-bit key of a float (larger float -> larger key); +-0 share
// a key, NaN maps to 0 (never selected, as the reference's strict '>' never
// selects it).
__device__ __forceinline__ uint32_t fkey(float f) {
    uint32_t u = __float_as_uint(f);
    if ((u & 0x7fffffffu) == 0u) u = 0u;
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) return 0u;
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float kfloat(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Top-K (K <= 32) of E <= 32*VPL logits by one warp: K rounds of (warp max of
// the keys, then the lowest index holding it) -- strict '>' with the lowest index
// winning ties, as the reference's scan.  Lane k < K returns the k-th index and
// its weight exp(l_k - max) / sum_selected exp(l_j - max).
template <int VPL>
__device__ __forceinline__ void warp_topk(const float* __restrict__ l, int E, int K, int& out_idx,
                                          float& out_w) {
    const int lane = threadIdx.x & 31;
    uint32_t key[VPL];
#pragma unroll
    for (int j = 0; j < VPL; ++j) {
        const int i = lane + 32 * j;
        key[j] = i < E ? fkey(__ldcg(l + i)) : 0u;
    }
    uint32_t lm = 0u;
#pragma unroll
    for (int j = 0; j < VPL; ++j) lm = max(lm, key[j]);
    const float mx = kfloat(__reduce_max_sync(0xffffffffu, lm));
    uint32_t my_key = 0u;
    int my_i = -1;
    for (int k = 0; k < K; ++k) {
        uint32_t l2 = 0u;
#pragma unroll
        for (int j = 0; j < VPL; ++j) l2 = max(l2, key[j]);
        const uint32_t g = __reduce_max_sync(0xffffffffu, l2);
        uint32_t cand = 0xffffffffu;
#pragma unroll
        for (int j = VPL - 1; j >= 0; --j)
            if (g != 0u && key[j] == g) cand = (uint32_t)(lane + 32 * j);
        const uint32_t win = __reduce_min_sync(0xffffffffu, cand);
        if (win != 0xffffffffu && (int)(win & 31u) == lane) {
#pragma unroll
            for (int j = 0; j < VPL; ++j)
                if (j == (int)(win >> 5)) key[j] = 0u;
        }
        if (lane == k && win != 0xffffffffu) {
            my_key = g;
            my_i = (int)win;
        }
    }
    const float ev = (lane < K && my_i >= 0) ? expf(kfloat(my_key) - mx) : 0.f;
    const float esum = warp_sum(ev);
    out_idx = my_i;
    out_w = (lane < K && esum > 0.f) ? ev / esum : 0.f;
}

__device__ __forceinline__ void warp_topk_any(const float* l, int E, int K, int& i, float& w) {
    if (E <= 256)
        warp_topk<8>(l, E, K, i, w);
    else
        warp_topk<32>(l, E, K, i, w);
}

// Warp-level staging of a down-projection input: act row (fp32) scaled by the
// power of two derived from the gate/up units' max |act|.  The max and the first
// chunks are loaded together, so one round trip covers both.  Returns 1/scale.
template <int BITS>
__device__ __forceinline__ float stage_act_warp(const float* act, const float* amax, int n_part, int n,
                                                int npad, __half* xs, float2* cx) {
    const int lane = threadIdx.x & 31;
    const int nch = n / 8, npch = npad / 8;
    constexpr int MAXB = 4;
    float am = 0.f;
    for (int i = lane; i < n_part; i += 32) am = fmaxf(am, __ldcg(amax + i));
    float v[MAXB][8];
#pragma unroll
    for (int b = 0; b < MAXB; ++b) {
        const int c = lane + 32 * b;
        if (c < nch)
            load8(act, KQ_DT_F32, (size_t)c * 8, true, v[b]);
        else
#pragma unroll
            for (int k = 0; k < 8; ++k) v[b][k] = 0.f;
    }
    const float scale = pow2_scale(warp_max(am));
    float offv[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) offv[k] = chunk_offset<BITS>(lane & 7, k);
#pragma unroll
    for (int b = 0; b < MAXB; ++b) {
        const int c = lane + 32 * b;
        if (c < npch) {
            const float2 part = store_chunk<BITS>(v[b], scale, offv, xs, c);
            group_reduce_store(part, lane, c, cx, 0xffffffffu);
        }
    }
    if (npch > 32 * MAXB)  // longer rows: the rest with the generic loop
        stage_fused<BITS, MAXB>(act, KQ_DT_F32, (size_t)32 * MAXB * 8, n - 32 * MAXB * 8 > 0 ? n - 32 * MAXB * 8 : 0,
                                npad - 32 * MAXB * 8, scale, true, lane, 32, xs + 32 * MAXB * 8, cx + 4 * MAXB);
    __syncwarp();
    return 1.f / scale;
}

}  // namespace kq
