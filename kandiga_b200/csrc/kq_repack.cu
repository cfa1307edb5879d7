// kq_repack.cu -- re-quantize MLX-layout affine matrices to another bit width
// on the GPU (the 4-bit -> 3-bit expert repack of
// scripts/repack_experts_3bit.py:76-103, which dequantizes each projection and
// quantizes it again at 3 bits with group 64, bf16 scales and biases).
//
// requant_kernel: one warp per (row, 64-wide group); lane l owns elements
// 2l, 2l+1 of the group.
//   dequantize: v = fp32(q * s + b), rounded to the scale dtype (the dequantized
//               matrix is held in the scale dtype, as the reference's
//               dequantize returns it);
//   quantize:   MLX's affine quantizer per group, in IEEE fp32: mn = min v,
//               mx = max v, scale = max((mx - mn) / (2^bits - 1), 1e-7), negated
//               unless |mn| > |mx|; edge = mn if |mn| > |mx| else mx;
//               q0 = round_half_even(edge / scale); where q0 != 0, scale =
//               edge / q0 and bias = edge (else bias 0), so the edge of larger
//               magnitude and zero are exactly representable;
//               q = clip(round_half_even((v - bias) / scale), 0, 2^bits - 1)
//               from those fp32 values; scale and bias then rounded to the scale
//               dtype (the quantizer of kandiga_b200/quant.py, mode "edge");
//   pack:       MLX layout, fields LSB first: 4-bit = 8 nibbles per uint32,
//               3-bit = 8 codes per 3 bytes (kandiga/metal/kandiga_cpu_expert.m:194-201,285-291).
#include "kq_internal.h"
#include "kq_common.cuh"

namespace kq {

template <int SB>
__device__ __forceinline__ float sb_round(float v) {
    if (SB == KQ_DT_F16) return __half2float(__float2half_rn(v));
    return __bfloat162float(__float2bfloat16_rn(v));
}

template <int SB>
__device__ __forceinline__ uint16_t sb_bits(float v) {
    if (SB == KQ_DT_F16) return __half_as_ushort(__float2half_rn(v));
    return __bfloat16_as_ushort(__float2bfloat16_rn(v));
}

// code of element j (0-based column) of a packed row
__device__ __forceinline__ int code_at(const uint8_t* row, int bits, int j) {
    if (bits == 4) return (int)((reinterpret_cast<const uint32_t*>(row)[j >> 3] >> (4 * (j & 7))) & 15u);
    const uint8_t* pk = row + (j >> 3) * 3;
    const uint32_t word = (uint32_t)pk[0] | ((uint32_t)pk[1] << 8) | ((uint32_t)pk[2] << 16);
    return (int)((word >> (3 * (j & 7))) & 7u);
}

template <int SB>
__global__ void requant_kernel(const uint8_t* __restrict__ w, const uint16_t* __restrict__ s,
                               const uint16_t* __restrict__ b, long rows, int cols, int src_bits, int dst_bits,
                               uint8_t* __restrict__ w_out, uint16_t* __restrict__ s_out,
                               uint16_t* __restrict__ b_out) {
    const long gw = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int gpr = cols / 64;
    if (gw >= rows * gpr) return;
    const long r = gw / gpr;
    const int g = (int)(gw % gpr);
    const uint8_t* row = w + (size_t)r * cols * src_bits / 8;
    const float sc = sb_lo<SB>(s[(size_t)r * gpr + g]), bi = sb_lo<SB>(b[(size_t)r * gpr + g]);
    const int j0 = g * 64 + 2 * lane;
    const float v0 = sb_round<SB>(__fadd_rn(__fmul_rn((float)code_at(row, src_bits, j0), sc), bi));
    const float v1 = sb_round<SB>(__fadd_rn(__fmul_rn((float)code_at(row, src_bits, j0 + 1), sc), bi));
    float mn = fminf(v0, v1), mx = fmaxf(v0, v1);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    }
    const float nb = (float)((1 << dst_bits) - 1);
    float scale = fmaxf(__fdiv_rn(__fsub_rn(mx, mn), nb), 1e-7f);
    const bool side = fabsf(mn) > fabsf(mx);
    scale = side ? scale : -scale;
    const float edge = side ? mn : mx;
    const float qe = rintf(__fdiv_rn(edge, scale));
    float bias = 0.f;
    if (qe != 0.f) {
        scale = __fdiv_rn(edge, qe);
        bias = edge;
    }
    const uint16_t s16 = sb_bits<SB>(scale), b16 = sb_bits<SB>(bias);
    const int q0 = (int)fminf(fmaxf(rintf(__fdiv_rn(__fsub_rn(v0, bias), scale)), 0.f), nb);
    const int q1 = (int)fminf(fmaxf(rintf(__fdiv_rn(__fsub_rn(v1, bias), scale)), 0.f), nb);
    // lanes 4p..4p+3 hold the 8 codes of pack p (elements 8p..8p+7 of the group)
    uint32_t part = ((uint32_t)q0 << (dst_bits * (2 * (lane & 3)))) | ((uint32_t)q1 << (dst_bits * (2 * (lane & 3) + 1)));
    part |= __shfl_down_sync(0xffffffffu, part, 1);
    part |= __shfl_down_sync(0xffffffffu, part, 2);
    uint8_t* orow = w_out + (size_t)r * cols * dst_bits / 8;
    if ((lane & 3) == 0) {
        const int p = g * 8 + (lane >> 2);  // pack index in the row
        if (dst_bits == 4) {
            reinterpret_cast<uint32_t*>(orow)[p] = part;
        } else {
            orow[p * 3] = (uint8_t)(part & 0xFF);
            orow[p * 3 + 1] = (uint8_t)((part >> 8) & 0xFF);
            orow[p * 3 + 2] = (uint8_t)((part >> 16) & 0xFF);
        }
    }
    if (lane == 0) {
        s_out[(size_t)r * gpr + g] = s16;
        b_out[(size_t)r * gpr + g] = b16;
    }
}

}  // namespace kq

using namespace kq;

extern "C" int kq_requantize_mlx(const void* weight, const void* scales, const void* biases, long rows, int cols,
                                 int src_bits, int dst_bits, int sb_dtype, void* weight_out, void* scales_out,
                                 void* biases_out, void* stream) {
    if (rows < 0 || cols <= 0 || cols % 64) return KQ_ERR_ARG;
    if ((src_bits != 3 && src_bits != 4) || (dst_bits != 3 && dst_bits != 4)) return KQ_ERR_ARG;
    if (sb_dtype != KQ_DT_F16 && sb_dtype != KQ_DT_BF16) return KQ_ERR_ARG;
    if (rows == 0) return KQ_OK;
    if (!weight || !scales || !biases || !weight_out || !scales_out || !biases_out) return KQ_ERR_ARG;
    const long warps = rows * (cols / 64);
    const int threads = 256;
    const long blocks = (warps * 32 + threads - 1) / threads;
    if (blocks > 0x7fffffffL) return KQ_ERR_UNSUPPORTED;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    auto w = static_cast<const uint8_t*>(weight);
    auto sc = static_cast<const uint16_t*>(scales);
    auto bi = static_cast<const uint16_t*>(biases);
    auto wo = static_cast<uint8_t*>(weight_out);
    auto so = static_cast<uint16_t*>(scales_out);
    auto bo = static_cast<uint16_t*>(biases_out);
    if (sb_dtype == KQ_DT_F16)
        requant_kernel<KQ_DT_F16><<<(unsigned)blocks, threads, 0, s>>>(w, sc, bi, rows, cols, src_bits, dst_bits, wo, so,
                                                                       bo);
    else
        requant_kernel<KQ_DT_BF16><<<(unsigned)blocks, threads, 0, s>>>(w, sc, bi, rows, cols, src_bits, dst_bits, wo,
                                                                        so, bo);
    return cudaGetLastError() == cudaSuccess ? KQ_OK : KQ_ERR_CUDA;
}
