// kq_shared.cu -- shared expert gate of a MoE block (kandiga/metal/moe_block.metal:335-404).
//
// The shared expert MLP (moe_block.metal:230-324) runs as one more expert of
// the layer's table: it is stored at expert index `shared_id`, and every token
// gets it as a (K+1)-th assignment with weight sigmoid(w_gate . x), the
// reference's gate.  The routed paths then compute
// out = [res] + sum_k w_k y_k + gate * y_shared in their own combine, the
// reference's blend (moe_block.metal:515-584), with no separate shared-expert
// GEMVs or blend pass.  shared_gate_kernel: one warp per token, the gate row
// read in MLX layout (3- or 4-bit, scales/biases fp16 or bf16):
// logit = sum_i (q_i s_g + b_g) x_i, gate = 1 / (1 + exp(-logit)).
#include "kq_internal.h"
#include "kq_common.cuh"

namespace kq {

template <int BITS, int SB_DT>
__global__ void shared_gate_kernel(const void* __restrict__ x, int x_dtype, int T, int H,
                                   const uint8_t* __restrict__ gw, const uint16_t* __restrict__ gs,
                                   const uint16_t* __restrict__ gb, const int32_t* __restrict__ idx_in,
                                   const float* __restrict__ w_in, int K, int shared_id, int32_t* __restrict__ idx_out,
                                   float* __restrict__ w_out, float* __restrict__ gate_out) {
    const int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (t >= T) return;
    float acc = 0.f;
    for (int p = lane; p < H / 8; p += 32) {  // pack of 8 codes
        uint32_t codes;
        if (BITS == 4) {
            codes = reinterpret_cast<const uint32_t*>(gw)[p];
        } else {
            const uint8_t* b = gw + 3 * p;
            codes = (uint32_t)b[0] | ((uint32_t)b[1] << 8) | ((uint32_t)b[2] << 16);
        }
        const int g = (8 * p) / 64;
        const float s = SB_DT == KQ_DT_F16 ? sb_lo<KQ_DT_F16>(gs[g]) : sb_lo<KQ_DT_BF16>(gs[g]);
        const float bi = SB_DT == KQ_DT_F16 ? sb_lo<KQ_DT_F16>(gb[g]) : sb_lo<KQ_DT_BF16>(gb[g]);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float q = (float)((codes >> (BITS * j)) & ((1u << BITS) - 1u));
            acc = fmaf(fmaf(q, s, bi), load_as_float(x, x_dtype, (size_t)t * H + 8 * p + j), acc);
        }
    }
    const float logit = warp_sum(acc);
    const float gate = 1.f / (1.f + expf(-logit));
    for (int k = lane; k <= K; k += 32) {
        idx_out[(size_t)t * (K + 1) + k] = k < K ? idx_in[(size_t)t * K + k] : shared_id;
        w_out[(size_t)t * (K + 1) + k] = k < K ? w_in[(size_t)t * K + k] : gate;
    }
    if (lane == 0 && gate_out) gate_out[t] = gate;
}

}  // namespace kq

using namespace kq;

extern "C" int kq_shared_gate(const void* x, int x_dtype, int T, int H, const void* gate_weight,
                              const void* gate_scales, const void* gate_biases, int bits, int sb_dtype,
                              const int32_t* idx, const float* weights, int K, int shared_id, int32_t* idx_out,
                              float* weights_out, float* gate_out, void* stream) {
    if (T < 0 || H <= 0 || H % 64 || K < 0 || (bits != 3 && bits != 4)) return KQ_ERR_ARG;
    if (sb_dtype != KQ_DT_F16 && sb_dtype != KQ_DT_BF16) return KQ_ERR_ARG;
    if (x_dtype != KQ_DT_F16 && x_dtype != KQ_DT_BF16 && x_dtype != KQ_DT_F32) return KQ_ERR_ARG;
    if (T == 0) return KQ_OK;
    if (!x || !gate_weight || !gate_scales || !gate_biases || !idx_out || !weights_out) return KQ_ERR_ARG;
    if (K > 0 && (!idx || !weights)) return KQ_ERR_ARG;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int threads = 256, blocks = (T * 32 + threads - 1) / threads;
    const uint8_t* gw = static_cast<const uint8_t*>(gate_weight);
    const uint16_t* gs = static_cast<const uint16_t*>(gate_scales);
    const uint16_t* gb = static_cast<const uint16_t*>(gate_biases);
#define KQ_SG(B, D)                                                                                               \
    shared_gate_kernel<B, D><<<blocks, threads, 0, s>>>(x, x_dtype, T, H, gw, gs, gb, idx, weights, K, shared_id, \
                                                        idx_out, weights_out, gate_out)
    if (bits == 4) {
        if (sb_dtype == KQ_DT_F16)
            KQ_SG(4, KQ_DT_F16);
        else
            KQ_SG(4, KQ_DT_BF16);
    } else {
        if (sb_dtype == KQ_DT_F16)
            KQ_SG(3, KQ_DT_F16);
        else
            KQ_SG(3, KQ_DT_BF16);
    }
#undef KQ_SG
    return cudaGetLastError() == cudaSuccess ? KQ_OK : KQ_ERR_CUDA;
}

namespace kq {

// out[t][h] = [res[t][h]] + sum_k w[t][k] y[t][k][h] + [gate[t] shared[t][h]]
__global__ void blend_kernel(const void* __restrict__ y, int y_dtype, const float* __restrict__ w, int T, int K,
                             int H, const void* __restrict__ residual, const void* __restrict__ shared,
                             int shared_dtype, const float* __restrict__ gate, void* out, int out_dtype) {
    const int t = blockIdx.y, h = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= T || h >= H) return;
    float acc = 0.f;
    for (int k = 0; k < K; ++k) acc = fmaf(load_as_float(y, y_dtype, ((size_t)t * K + k) * H + h), w[(size_t)t * K + k], acc);
    if (shared) acc = fmaf(gate ? gate[t] : 1.f, load_as_float(shared, shared_dtype, (size_t)t * H + h), acc);
    if (residual) acc = load_as_float(residual, out_dtype, (size_t)t * H + h) + acc;
    store_from_float(out, out_dtype, (size_t)t * H + h, acc);
}

}  // namespace kq

extern "C" int kq_combine(const void* y, int y_dtype, const float* weights, int T, int K, int H, const void* residual,
                          const void* shared, int shared_dtype, const float* gate, void* out, int out_dtype,
                          void* stream) {
    if (T < 0 || K < 0 || H <= 0) return KQ_ERR_ARG;
    for (int dt : {y_dtype, out_dtype})
        if (dt != KQ_DT_F16 && dt != KQ_DT_BF16 && dt != KQ_DT_F32) return KQ_ERR_ARG;
    if (shared && shared_dtype != KQ_DT_F16 && shared_dtype != KQ_DT_BF16 && shared_dtype != KQ_DT_F32)
        return KQ_ERR_ARG;
    if (T == 0) return KQ_OK;
    if (!out || (K > 0 && (!y || !weights))) return KQ_ERR_ARG;
    dim3 grid((H + 255) / 256, T);
    blend_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(y, y_dtype, weights, T, K, H, residual, shared,
                                                                      shared_dtype, gate, out, out_dtype);
    return cudaGetLastError() == cudaSuccess ? KQ_OK : KQ_ERR_CUDA;
}
