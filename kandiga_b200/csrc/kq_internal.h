// kq_internal.h -- host-side structures shared by the libkq translation units.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <algorithm>
#include <new>

#include "kq.h"
#include "kq_qtile.cuh"

struct kq_table {
    kq_table_desc d;
    uint8_t* base = nullptr;
    size_t bytes = 0;
    int tb = 0;                 // tile bytes
    int nst_h = 0, nst_i = 0;   // column tiles along H / I
    int i8 = 0, h16 = 0;        // gate/up row-tiles (8 intermediate rows), down row-tiles
    size_t gateup_bytes = 0, down_bytes = 0, expert_bytes = 0, layer_bytes = 0;
};

struct kq_qmat {
    int rows = 0, cols = 0, bits = 0, sb_dtype = 0, pair = 0;
    int nrt = 0, nst = 0, tb = 0;
    uint8_t* base = nullptr;
    size_t bytes = 0;
};

namespace kq {

struct BkexInfo {
    int num_experts, hidden, inter, bits, sb_dtype, activation;
    uint64_t expert_size;
    uint32_t off[9], nbytes[9], d0[9], d1[9];
    uint8_t dtype[9];
};
int bkex_parse(const uint8_t* hdr, size_t n, BkexInfo* info);

// kq_moe_decode with an optional RMSNorm of x (norm_w fp16 [hidden], x fp16)
// applied in the gate/up input staging.
int moe_decode_ex(const kq_table* t, int layer, const void* x, int x_dtype, int T, const float* logits,
                  int32_t* idx, float* weights, int K, void* out_per_k, void* out, int out_dtype,
                  const void* residual, const void* norm_w, float eps, void* workspace, size_t workspace_bytes,
                  void* stream);

// kq_moe_prefill whose combined row t goes to out_rows[t] (device array of
// device addresses, a peer's memory included; null rows skipped; out unused)
// when out_rows is given.
int moe_prefill_ex(const kq_table* t, int layer, const void* x, int x_dtype, int T, const float* logits,
                   int32_t* idx, float* weights, int K, void* out_per_k, void* out, int out_dtype,
                   const void* residual, void* const* out_rows, void* workspace, size_t workspace_bytes,
                   void* stream);

// One token: idx/w [K + 1] = top-K of logits[0, E), then (shared_id, sigmoid(logits[E])).
int route_with_shared(const float* logits, int E, int K, int shared_id, int32_t* idx, float* w, cudaStream_t s);

// kq_dense_gemv with a residual added in the epilogue: y = residual + W x
// (residual in y_dtype, may alias y; not for gate/up pairs).
int dense_gemv_res(const kq_qmat* m, const void* x, int x_dtype, int T, const void* norm_w, float eps,
                   int activation, void* y, int y_dtype, const void* residual, void* stream);

// The MoE block engine (bakan_forward_*, kq_forward.cu) as one layer kind of
// the whole-model decode step.  moe_block_prepare: all weights of `layer` set,
// workspace allocated (call before capturing); moe_block_enqueue: out = in +
// MoE(rmsnorm(in)) on stream s (fp16 [hidden]; out != in); moe_block_status:
// the device status word its kernels latch into.
int moe_block_prepare(void* engine, int layer);
int moe_block_enqueue(void* engine, int layer, const __half* in, __half* out, cudaStream_t s);
int moe_block_hidden(void* engine);
uint32_t* moe_block_status(void* engine);

// Raise a kernel's dynamic shared-memory limit to at least `bytes` on the
// current device.  One record per (kernel, device) for the whole library, and
// the limit only ever rises, so launch paths that share a kernel cannot lower
// it under one another.
cudaError_t raise_smem_limit(const void* kernel, size_t bytes);

// Read packed_dir/layer_XX.bin for XX < num_layers into a new HBM table on
// stream s, with extra_experts more (empty) expert slots per layer after the
// file's.  0 on success; -1 after a "[kandiga] ERROR: ..." line on stderr,
// with nothing left allocated.
int load_bkex_dir(const char* packed_dir, int num_layers, cudaStream_t s, kq_table** out, BkexInfo* info,
                  int extra_experts = 0);

// Launch `kern` as a programmatic dependent of the kernel before it on the
// stream: it may start before that kernel ends and must call
// griddepcontrol.wait (pdl_wait) before touching what that kernel writes.
template <typename... KArgs, typename... Args>
static inline cudaError_t launch_dep(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
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
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

// Workspace carve-up for kq_moe_* (offsets in bytes, 256-aligned).
struct MoeWs {
    size_t status, idx, w, act, amax, total;
};
MoeWs moe_ws_layout(const kq_table* t, int T, int K);

}  // namespace kq

struct kq_tq_cache {
    int D = 0, H = 0, B = 0, cap = 0, len = 0;  // D: storage width (head_dim rounded up to 64 or 128)
    int Dr = 0;                                 // head_dim
    float* R = nullptr;              // [D][D] rotation: x_rot = x R
    float* RT = nullptr;             // [D][D] R transposed
    float* P = nullptr;              // [D][D] QJL projection
    uint8_t* packed[2] = {nullptr, nullptr};  // K, V: [B][H][cap][D/2], nibble = code | sign << 3
    float* scale[2] = {nullptr, nullptr};     // [B][H][cap] (+ 16 floats of tail padding)
    float* zero[2] = {nullptr, nullptr};
    uint32_t* status = nullptr;      // device word: KQ_DEV_* bits latched by the append kernels
    uint8_t* tc_ops = nullptr;       // width 128: R^T and P^T as fp16 limb pairs, swizzled (4 x 32 KB)
};

struct kq_tq3_mat {
    int rows = 0, cols = 0, block_bytes = 0;  // 20 (d0 d1 m0 m1 + codes) or 16 (d0 d1 + codes)
    size_t bytes = 0;
    uint8_t* data = nullptr;                  // the reference's block stream, row-major
};
