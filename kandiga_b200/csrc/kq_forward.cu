// kq_forward.cu -- the MoE block engine ABI that the reference declares but
// does not implement (kandiga/metal/bakan_forward.h:36-151), with the
// arithmetic of its Metal kernels (kandiga/metal/moe_block.metal:134-584).
//
// bakan_forward_init reads the routed experts' BKEX layer files into an HBM
// table (as bakan_cpu_expert_init does).  bakan_forward_set_weight uploads the
// per-layer tensors of the block in MLX layout: the post-attention norm, the
// quantized router, the shared-expert gate row and the shared expert's three
// matrices.  Once a matrix's weight, scales and biases are all present it is
// repacked: the router into a dense quantized matrix, the shared expert into
// a one-expert table.  One block call on device memory:
//   normed = fp16(h * (1 / sqrt(mean(h^2) + eps)) * w_norm)    fwd_rmsnorm_kernel
//   logits = W_router normed                                   kq_dense_gemv (fp32 out)
//   idx, w = softmax -> top-K -> renormalise;
//   routed = sum_k w_k E_idx_k(normed)                         kq_moe_decode
//   gate   = sigmoid(w_gate . normed)                          kq_shared_gate
//   shared = S(normed), fp16                                   kq_moe_decode (one-expert table)
//   out    = h + routed + gate * shared                        kq_combine
// (the _normed variant takes normed = x and adds no residual).  The host
// entry points stage h in pinned memory and replay one CUDA graph per
// (layer, variant): copy in, the kernels above, copy out, device status.
// Calls are synchronous and, like the reference's engines, not re-entrant.
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <map>
#include <vector>

#include "kq_internal.h"
#include "kq_common.cuh"

namespace kq {

// RMSNorm of one fp16 vector (kandiga/metal/moe_block.metal:134-178): 256
// threads; strided partial sums of squares, tree reduction, scale =
// 1 / sqrt(mean + eps), out = fp16(x * scale * w).
constexpr int FWD_NORM_THREADS = 256;
__global__ void __launch_bounds__(FWD_NORM_THREADS) fwd_rmsnorm_kernel(const __half* __restrict__ x,
                                                                       const void* __restrict__ w, int w_dtype,
                                                                       int H, float eps, __half* __restrict__ out) {
    __shared__ float part[FWD_NORM_THREADS];
    const int tid = threadIdx.x;
    float acc = 0.f;
    for (int i = tid; i < H; i += FWD_NORM_THREADS) {
        const float v = __half2float(x[i]);
        acc = __fadd_rn(acc, __fmul_rn(v, v));
    }
    part[tid] = acc;
    __syncthreads();
    for (int st = FWD_NORM_THREADS / 2; st > 0; st >>= 1) {
        if (tid < st) part[tid] += part[tid + st];
        __syncthreads();
    }
    const float scale = 1.f / sqrtf(part[0] / (float)H + eps);
    for (int i = tid; i < H; i += FWD_NORM_THREADS)
        out[i] = __float2half_rn(__fmul_rn(__fmul_rn(__half2float(x[i]), scale), load_as_float(w, w_dtype, i)));
}

}  // namespace kq

using namespace kq;

namespace {

// Weight types of bakan_forward_set_weight (kandiga/metal/bakan_forward.h:35-53).
enum {
    WT_POST_ATTN_NORM = 0,
    WT_ROUTER_WEIGHT = 1,
    WT_ROUTER_SCALES = 2,
    WT_ROUTER_BIASES = 3,
    WT_SHARED_GATE_W = 4,
    WT_SHARED_GATE_S = 5,
    WT_SHARED_GATE_B = 6,
    WT_SHARED_UP_W = 7,
    WT_SHARED_UP_S = 8,
    WT_SHARED_UP_B = 9,
    WT_SHARED_GATE_PROJ_W = 10,
    WT_SHARED_GATE_PROJ_S = 11,
    WT_SHARED_GATE_PROJ_B = 12,
    WT_SHARED_DOWN_W = 13,
    WT_SHARED_DOWN_S = 14,
    WT_SHARED_DOWN_B = 15,
    WT_COUNT = 16
};

// set_weight dtype codes (kandiga/metal/bakan_forward.h:78): 0 fp16, 1 uint32 (packed codes), 2 bf16
constexpr int FWD_F16 = 0, FWD_U32 = 1, FWD_BF16 = 2;

struct DevTensor {
    void* p = nullptr;
    size_t bytes = 0;
    int rows = 0, cols = 0, dtype = -1;
};

struct FwdLayer {
    DevTensor wt[WT_COUNT];
    kq_qmat* router = nullptr;
    bool shared_loaded = false;
    // fast path (finalize_layer): the shared expert as expert E of the routed
    // table, the router with the shared-gate row as row E, the norm in fp16
    bool dirty = true;
    bool merged = false;
    kq_qmat* router_ext = nullptr;  // rows: E routed, 1 gate, zero rows to a multiple of 16
    __half* norm16 = nullptr;
};

struct FwdEngine {
    kq_table* routed = nullptr;
    BkexInfo info{};
    kq_table* shared = nullptr;  // one expert per layer
    int num_layers = 0;
    int top_k = 8;               // MoeBlockParams.num_experts_per_tok (kandiga/metal/moe_block.metal:118)
    float eps = 1e-6f;           // MoeBlockParams.rms_norm_eps (kandiga/metal/moe_block.metal:120)
    cudaStream_t stream = nullptr;
    std::vector<FwdLayer> layers;
    void* ws = nullptr;
    size_t ws_bytes = 0;
    // device vectors of one call
    __half *dh = nullptr, *dnorm = nullptr, *dshared = nullptr, *dout = nullptr;
    float *dlogits = nullptr, *droute = nullptr, *dgate = nullptr, *dones = nullptr, *dw = nullptr, *dgw = nullptr;
    int32_t *didx = nullptr, *dzero = nullptr, *dgidx = nullptr;
    uint8_t* hstage = nullptr;   // pinned: [h: H fp16][out: H fp16]
    uint32_t* hstatus = nullptr; // pinned device-status word
    std::map<int, cudaGraphExec_t> graphs;  // key: layer * 2 + normed
};

void drop_graphs(FwdEngine* e) {
    for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second);
    e->graphs.clear();
}

int sb_of(int dtype) { return dtype == FWD_BF16 ? KQ_DT_BF16 : KQ_DT_F16; }

bool have(const FwdLayer& L, int a, int b) {
    for (int i = a; i <= b; ++i)
        if (!L.wt[i].p) return false;
    return true;
}

// Bits of a packed matrix of `in` columns stored as rows x words uint32.
int bits_of(const DevTensor& w, int in) {
    if (in <= 0 || (long)w.cols * 32 % in) return 0;
    const int b = (int)((long)w.cols * 32 / in);
    return b == 3 || b == 4 ? b : 0;
}

// The matrix (weight, scales, biases) at types [w, w + 2] is complete and consistent for `in` columns.
bool matrix_ok(const FwdLayer& L, int w, int in, int* rows, int* bits, int* sb) {
    const DevTensor &W = L.wt[w], &S = L.wt[w + 1], &B = L.wt[w + 2];
    *bits = bits_of(W, in);
    *rows = W.rows;
    *sb = sb_of(S.dtype);
    return W.dtype == FWD_U32 && *bits && S.dtype == B.dtype && S.dtype != FWD_U32 && S.rows == W.rows &&
           B.rows == W.rows && S.cols == in / 64 && B.cols == in / 64 && in % 64 == 0;
}

kq_mlx_matrix mlx_of(const FwdLayer& L, int w) {
    kq_mlx_matrix m{};
    m.weight = L.wt[w].p;
    m.scales = L.wt[w + 1].p;
    m.biases = L.wt[w + 2].p;
    return m;
}

int build_router(FwdEngine* e, int layer) {
    FwdLayer& L = e->layers[layer];
    if (!have(L, WT_ROUTER_WEIGHT, WT_ROUTER_BIASES)) return 0;
    int rows, bits, sb;
    if (!matrix_ok(L, WT_ROUTER_WEIGHT, e->info.hidden, &rows, &bits, &sb) || rows != e->info.num_experts) {
        fprintf(stderr, "[kandiga] ERROR: router tensors of layer %d do not form a [%d, %d] quantized matrix\n",
                layer, e->info.num_experts, e->info.hidden);
        return -1;
    }
    if (L.router) kq_qmat_destroy(L.router);
    L.router = nullptr;
    const kq_mlx_matrix a = mlx_of(L, WT_ROUTER_WEIGHT);
    if (kq_qmat_create(rows, e->info.hidden, bits, sb, 0, &L.router) != KQ_OK ||
        kq_qmat_load_mlx(L.router, &a, nullptr, e->stream) != KQ_OK || cudaStreamSynchronize(e->stream) != cudaSuccess) {
        fprintf(stderr, "[kandiga] ERROR: cannot build the router of layer %d\n", layer);
        return -1;
    }
    return 0;
}

int build_shared(FwdEngine* e, int layer) {
    FwdLayer& L = e->layers[layer];
    if (!have(L, WT_SHARED_UP_W, WT_SHARED_DOWN_B)) return 0;
    const int H = e->info.hidden;
    int Iu, bu, su, Ig, bg, sg, Hd, bd, sd;
    const int I = L.wt[WT_SHARED_UP_W].rows;
    if (!matrix_ok(L, WT_SHARED_UP_W, H, &Iu, &bu, &su) || !matrix_ok(L, WT_SHARED_GATE_PROJ_W, H, &Ig, &bg, &sg) ||
        !matrix_ok(L, WT_SHARED_DOWN_W, I, &Hd, &bd, &sd) || Ig != I || Hd != H || bg != bu || bd != bu ||
        sg != su || sd != su) {
        fprintf(stderr, "[kandiga] ERROR: shared-expert tensors of layer %d are inconsistent\n", layer);
        return -1;
    }
    if (!e->shared) {
        kq_table_desc d{};
        d.num_layers = e->num_layers;
        d.num_experts = 1;
        d.hidden = H;
        d.inter = I;
        d.bits = bu;
        d.group_size = 64;
        d.sb_dtype = su;
        d.activation = KQ_ACT_SILU;  // shared_expert_up_gate_kernel: silu(gate) * up (moe_block.metal:286-287)
        if (kq_table_create(&d, &e->shared) != KQ_OK) {
            fprintf(stderr, "[kandiga] ERROR: cannot create the shared-expert table\n");
            return -1;
        }
    } else {
        kq_table_desc d{};
        kq_table_desc_get(e->shared, &d);
        if (d.inter != I || d.bits != bu || d.sb_dtype != su) {
            fprintf(stderr, "[kandiga] ERROR: shared expert of layer %d differs in shape from earlier layers\n", layer);
            return -1;
        }
    }
    const kq_mlx_matrix g = mlx_of(L, WT_SHARED_GATE_PROJ_W), u = mlx_of(L, WT_SHARED_UP_W),
                        dn = mlx_of(L, WT_SHARED_DOWN_W);
    if (kq_table_load_mlx(e->shared, layer, 0, 1, &g, &u, &dn, e->stream) != KQ_OK ||
        cudaStreamSynchronize(e->stream) != cudaSuccess) {
        fprintf(stderr, "[kandiga] ERROR: cannot load the shared expert of layer %d\n", layer);
        return -1;
    }
    L.shared_loaded = true;
    return 0;
}

bool alloc_all(FwdEngine* e) {
    const int H = e->info.hidden, E = e->info.num_experts;
    auto dev = [](void** p, size_t n) { return cudaMalloc(p, n) == cudaSuccess; };
    bool ok = dev((void**)&e->dh, H * 2) && dev((void**)&e->dnorm, H * 2) && dev((void**)&e->dshared, H * 2) &&
              dev((void**)&e->dout, H * 2) && dev((void**)&e->dlogits, (size_t)(E + 16) * 4) && dev((void**)&e->droute, H * 4) &&
              dev((void**)&e->dgate, 4) && dev((void**)&e->dones, 4) && dev((void**)&e->dw, 32 * 4) &&
              dev((void**)&e->dgw, 4) && dev((void**)&e->didx, 32 * 4) && dev((void**)&e->dzero, 4) &&
              dev((void**)&e->dgidx, 4);
    ok = ok && cudaHostAlloc((void**)&e->hstage, (size_t)H * 4, cudaHostAllocDefault) == cudaSuccess &&
         cudaHostAlloc((void**)&e->hstatus, 4, cudaHostAllocDefault) == cudaSuccess;
    if (!ok) {
        cudaGetLastError();
        return false;
    }
    const float one = 1.f;
    const int32_t zero = 0;
    return cudaMemcpy(e->dones, &one, 4, cudaMemcpyHostToDevice) == cudaSuccess &&
           cudaMemcpy(e->dzero, &zero, 4, cudaMemcpyHostToDevice) == cudaSuccess;
}

bool ensure_ws(FwdEngine* e) {
    size_t need = kq_moe_workspace_size(e->routed, 1, e->top_k + 1);
    if (e->shared) need = std::max(need, kq_moe_workspace_size(e->shared, 1, 1));
    if (need <= e->ws_bytes) return true;
    drop_graphs(e);
    if (e->ws) cudaFree(e->ws);
    e->ws = nullptr;
    e->ws_bytes = 0;
    if (cudaMalloc(&e->ws, need) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    e->ws_bytes = need;
    return kq_workspace_init(e->ws, need, e->stream) == KQ_OK;
}

__global__ void fwd_to_f16_kernel(const void* __restrict__ src, int dtype, int n, __half* __restrict__ dst) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) dst[i] = __float2half(load_as_float(src, dtype, i));
}

// Build the fast path of a layer once its tensors are all set: the shared
// expert into slot E of the routed table (same inter, bits and scale dtype as
// the routed experts), the router with the gate row appended (same bits and
// scale dtype), the norm weight in fp16.  Layers that do not match keep the
// separate path.  Called before a graph of the layer is captured.
int finalize_layer(FwdEngine* e, int layer) {
    FwdLayer& L = e->layers[layer];
    if (!L.dirty) return 0;
    const int H = e->info.hidden, E = e->info.num_experts;
    cudaStream_t s = e->stream;
    L.merged = false;
    if (L.router_ext) kq_qmat_destroy(L.router_ext);
    L.router_ext = nullptr;
    if (L.shared_loaded) {
        int I, b, sb;
        if (matrix_ok(L, WT_SHARED_UP_W, H, &I, &b, &sb) && I == e->info.inter && b == e->info.bits &&
            sb == e->info.sb_dtype) {
            const kq_mlx_matrix g = mlx_of(L, WT_SHARED_GATE_PROJ_W), u = mlx_of(L, WT_SHARED_UP_W),
                                dn = mlx_of(L, WT_SHARED_DOWN_W);
            if (kq_table_load_mlx(e->routed, layer, E, 1, &g, &u, &dn, s) != KQ_OK) return -1;
            L.merged = true;
        }
    }
    int rr, rb, rs, gr, gb, gs;
    if (L.router && have(L, WT_SHARED_GATE_W, WT_SHARED_GATE_B) && matrix_ok(L, WT_ROUTER_WEIGHT, H, &rr, &rb, &rs) &&
        matrix_ok(L, WT_SHARED_GATE_W, H, &gr, &gb, &gs) && gr >= 1 && gb == rb && gs == rs) {
        const int rows = (E + 1 + 15) / 16 * 16;
        const size_t wrow = (size_t)H * rb / 8, srow = (size_t)H / 64 * 2;
        uint8_t* buf = nullptr;
        const size_t wbytes = rows * wrow, sbytes = rows * srow;
        if (cudaMalloc(&buf, wbytes + 2 * sbytes) != cudaSuccess) {
            cudaGetLastError();
            return -1;
        }
        bool ok = cudaMemsetAsync(buf, 0, wbytes + 2 * sbytes, s) == cudaSuccess;
        uint8_t* parts[3] = {buf, buf + wbytes, buf + wbytes + sbytes};
        const size_t per[3] = {wrow, srow, srow};
        for (int k = 0; k < 3 && ok; ++k) {
            ok = cudaMemcpyAsync(parts[k], L.wt[WT_ROUTER_WEIGHT + k].p, (size_t)E * per[k], cudaMemcpyDeviceToDevice,
                                 s) == cudaSuccess &&
                 cudaMemcpyAsync(parts[k] + (size_t)E * per[k], L.wt[WT_SHARED_GATE_W + k].p, per[k],
                                 cudaMemcpyDeviceToDevice, s) == cudaSuccess;
        }
        kq_mlx_matrix m{};
        m.weight = parts[0];
        m.scales = parts[1];
        m.biases = parts[2];
        ok = ok && kq_qmat_create(rows, H, rb, rs, 0, &L.router_ext) == KQ_OK &&
             kq_qmat_load_mlx(L.router_ext, &m, nullptr, s) == KQ_OK && cudaStreamSynchronize(s) == cudaSuccess;
        cudaFree(buf);
        if (!ok) {
            if (L.router_ext) kq_qmat_destroy(L.router_ext);
            L.router_ext = nullptr;
            return -1;
        }
    }
    const DevTensor& nt = L.wt[WT_POST_ATTN_NORM];
    if (nt.p) {
        if (!L.norm16 && cudaMalloc(&L.norm16, (size_t)H * 2) != cudaSuccess) {
            cudaGetLastError();
            return -1;
        }
        fwd_to_f16_kernel<<<(H + 255) / 256, 256, 0, s>>>(nt.p, nt.dtype == FWD_BF16 ? KQ_DT_BF16 : KQ_DT_F16, H,
                                                          L.norm16);
        if (cudaStreamSynchronize(s) != cudaSuccess) return -1;
    }
    L.dirty = false;
    return 0;
}

// Enqueue one block on stream s: out = [in] + MoE(x), x = in or rmsnorm(in).
int enqueue_block_io(FwdEngine* e, int layer, bool normed, const __half* in, __half* out, cudaStream_t s) {
    const FwdLayer& L = e->layers[layer];
    const int H = e->info.hidden;
    if (L.merged && L.router_ext && (normed || L.norm16)) {
        // router + shared gate in one GEMV (RMSNorm prologue), top-K + (shared, sigmoid(gate)),
        // then K + 1 experts whose down pass blends them into the residual
        const int E = e->info.num_experts;
        const __half* nw = normed ? nullptr : L.norm16;
        int rc = dense_gemv_res(L.router_ext, in, KQ_DT_F16, 1, nw, e->eps, KQ_ACT_SILU, e->dlogits, KQ_DT_F32,
                                nullptr, s);
        if (rc == KQ_OK) rc = route_with_shared(e->dlogits, E, e->top_k, E, e->didx, e->dw, s);
        if (rc == KQ_OK)
            rc = moe_decode_ex(e->routed, layer, in, KQ_DT_F16, 1, nullptr, e->didx, e->dw, e->top_k + 1, nullptr, out,
                               KQ_DT_F16, normed ? nullptr : in, nw, e->eps, e->ws, e->ws_bytes, s);
        return rc;
    }
    const __half* x = in;
    if (!normed) {
        fwd_rmsnorm_kernel<<<1, FWD_NORM_THREADS, 0, s>>>(in, L.wt[WT_POST_ATTN_NORM].p,
                                                          L.wt[WT_POST_ATTN_NORM].dtype == FWD_BF16 ? KQ_DT_BF16
                                                                                                     : KQ_DT_F16,
                                                          H, e->eps, e->dnorm);
        if (cudaGetLastError() != cudaSuccess) return KQ_ERR_CUDA;
        x = e->dnorm;
    }
    // the routed table has one slot past the E routed experts: route over E explicitly
    int rc = kq_dense_gemv(L.router, x, KQ_DT_F16, 1, nullptr, 0.f, KQ_ACT_SILU, e->dlogits, KQ_DT_F32, s);
    if (rc == KQ_OK) rc = kq_router_topk(e->dlogits, 1, e->info.num_experts, e->top_k, e->didx, e->dw, s);
    if (rc == KQ_OK)
        rc = kq_moe_decode(e->routed, layer, x, KQ_DT_F16, 1, nullptr, e->didx, e->dw, e->top_k, nullptr, e->droute,
                           KQ_DT_F32, nullptr, e->ws, e->ws_bytes, s);
    const DevTensor& gw = L.wt[WT_SHARED_GATE_W];
    if (rc == KQ_OK)
        rc = kq_shared_gate(x, KQ_DT_F16, 1, H, gw.p, L.wt[WT_SHARED_GATE_S].p, L.wt[WT_SHARED_GATE_B].p,
                            bits_of(gw, H), sb_of(L.wt[WT_SHARED_GATE_S].dtype), nullptr, nullptr, 0, 0, e->dgidx,
                            e->dgw, e->dgate, s);
    if (rc == KQ_OK)
        rc = kq_moe_decode(e->shared, layer, x, KQ_DT_F16, 1, nullptr, e->dzero, e->dones, 1, nullptr, e->dshared,
                           KQ_DT_F16, nullptr, e->ws, e->ws_bytes, s);
    if (rc == KQ_OK)
        rc = kq_combine(e->droute, KQ_DT_F32, e->dones, 1, 1, H, normed ? nullptr : in, e->dshared, KQ_DT_F16,
                        e->dgate, out, KQ_DT_F16, s);
    return rc;
}

// Enqueue one block on e->stream (input in e->dh, output in e->dout).
int enqueue_block(FwdEngine* e, int layer, bool normed) {
    return enqueue_block_io(e, layer, normed, e->dh, e->dout, e->stream);
}

const char* block_missing(const FwdEngine* e, int layer, bool normed) {
    const FwdLayer& L = e->layers[layer];
    if (!normed && !L.wt[WT_POST_ATTN_NORM].p) return "post-attention norm";
    if (!L.router) return "router";
    if (!have(L, WT_SHARED_GATE_W, WT_SHARED_GATE_B) || !bits_of(L.wt[WT_SHARED_GATE_W], e->info.hidden))
        return "shared-expert gate";
    if (!L.shared_loaded) return "shared expert";
    return nullptr;
}

int run_block(FwdEngine* e, int layer, const void* in, void* out, bool normed) {
    if (!e || layer < 0 || layer >= e->num_layers || !in || !out) {
        fprintf(stderr, "[kandiga] ERROR: bad arguments to the MoE block (layer %d)\n", layer);
        return -1;
    }
    if (const char* miss = block_missing(e, layer, normed)) {
        fprintf(stderr, "[kandiga] ERROR: layer %d has no %s weights\n", layer, miss);
        return -1;
    }
    if (!ensure_ws(e) || finalize_layer(e, layer) != 0) {
        fprintf(stderr, "[kandiga] ERROR: device allocation or setup failed (layer %d)\n", layer);
        return -1;
    }
    const int H = e->info.hidden;
    cudaStream_t s = e->stream;
    const int key = layer * 2 + (normed ? 1 : 0);
    auto it = e->graphs.find(key);
    if (it == e->graphs.end()) {
        cudaGraph_t graph = nullptr;
        if (cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
            fprintf(stderr, "[kandiga] ERROR: graph capture failed for layer %d\n", layer);
            return -1;
        }
        bool ok = cudaMemcpyAsync(e->dh, e->hstage, (size_t)H * 2, cudaMemcpyHostToDevice, s) == cudaSuccess;
        ok = ok && enqueue_block(e, layer, normed) == KQ_OK;
        ok = ok && cudaMemcpyAsync(e->hstage + (size_t)H * 2, e->dout, (size_t)H * 2, cudaMemcpyDeviceToHost, s) ==
                       cudaSuccess;
        ok = ok && cudaMemcpyAsync(e->hstatus, e->ws, 4, cudaMemcpyDeviceToHost, s) == cudaSuccess &&
             cudaMemsetAsync(e->ws, 0, 4, s) == cudaSuccess;
        const bool ended = cudaStreamEndCapture(s, &graph) == cudaSuccess;
        cudaGraphExec_t exec = nullptr;
        ok = ok && ended && graph && cudaGraphInstantiate(&exec, graph, 0) == cudaSuccess;
        if (graph) cudaGraphDestroy(graph);
        if (!ok) {
            cudaGetLastError();
            fprintf(stderr, "[kandiga] ERROR: graph capture failed for layer %d\n", layer);
            return -1;
        }
        it = e->graphs.emplace(key, exec).first;
    }
    memcpy(e->hstage, in, (size_t)H * 2);
    *e->hstatus = 0;
    if (cudaGraphLaunch(it->second, s) != cudaSuccess || cudaStreamSynchronize(s) != cudaSuccess) {
        fprintf(stderr, "[kandiga] ERROR: MoE block failed for layer %d\n", layer);
        return -1;
    }
    if (*e->hstatus != 0) {
        fprintf(stderr, "[kandiga] ERROR: device status 0x%x for layer %d\n", *e->hstatus, layer);
        return -1;
    }
    memcpy(out, e->hstage + (size_t)H * 2, (size_t)H * 2);
    return 0;
}

}  // namespace

extern "C" void bakan_forward_destroy(void* engine);

extern "C" void* bakan_forward_init(const char* packed_expert_dir, int num_layers) {
    if (!packed_expert_dir || num_layers <= 0) {
        fprintf(stderr, "[kandiga] ERROR: bad arguments to init\n");
        return nullptr;
    }
    FwdEngine* e = new (std::nothrow) FwdEngine();
    if (!e) return nullptr;
    e->num_layers = num_layers;
    e->layers.resize(num_layers);
    if (cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking) != cudaSuccess) {
        fprintf(stderr, "[kandiga] ERROR: no CUDA device\n");
        delete e;
        return nullptr;
    }
    // one slot per layer past the routed experts: the shared expert, when its shape matches theirs
    if (load_bkex_dir(packed_expert_dir, num_layers, e->stream, &e->routed, &e->info, 1) || !alloc_all(e)) {
        if (e->routed) fprintf(stderr, "[kandiga] ERROR: device allocation failed\n");
        bakan_forward_destroy(e);
        return nullptr;
    }
    e->top_k = std::min(e->top_k, e->info.num_experts);
    fprintf(stderr, "[kandiga] MoE block engine: %d layers, %d experts, %d-bit, HBM-resident\n", num_layers,
            e->info.num_experts, e->info.bits);
    return e;
}

extern "C" int bakan_forward_set_weight(void* engine, int layer_idx, int weight_type, const void* data, size_t size,
                                        int rows, int cols, int dtype) {
    FwdEngine* e = static_cast<FwdEngine*>(engine);
    if (!e || layer_idx < 0 || layer_idx >= e->num_layers || weight_type < 0 || weight_type >= WT_COUNT || !data ||
        rows <= 0 || cols <= 0 || (dtype != FWD_F16 && dtype != FWD_U32 && dtype != FWD_BF16)) {
        fprintf(stderr, "[kandiga] ERROR: bad arguments to set_weight (layer %d, type %d)\n", layer_idx, weight_type);
        return -1;
    }
    const size_t want = (size_t)rows * cols * (dtype == FWD_U32 ? 4 : 2);
    if (size != want) {
        fprintf(stderr, "[kandiga] ERROR: weight type %d of layer %d: %zu bytes for [%d, %d] (expected %zu)\n",
                weight_type, layer_idx, size, rows, cols, want);
        return -1;
    }
    if (weight_type == WT_POST_ATTN_NORM && (dtype == FWD_U32 || (long)rows * cols != e->info.hidden)) {
        fprintf(stderr, "[kandiga] ERROR: the post-attention norm of layer %d must hold %d fp16/bf16 values\n",
                layer_idx, e->info.hidden);
        return -1;
    }
    drop_graphs(e);
    DevTensor& t = e->layers[layer_idx].wt[weight_type];
    if (t.bytes < size) {
        if (t.p) cudaFree(t.p);
        t.p = nullptr;
        t.bytes = 0;
        if (cudaMalloc(&t.p, size) != cudaSuccess) {
            cudaGetLastError();
            fprintf(stderr, "[kandiga] ERROR: device allocation failed\n");
            return -1;
        }
        t.bytes = size;
    }
    if (cudaMemcpy(t.p, data, size, cudaMemcpyHostToDevice) != cudaSuccess) {
        fprintf(stderr, "[kandiga] ERROR: copy of weight type %d of layer %d failed\n", weight_type, layer_idx);
        return -1;
    }
    t.rows = rows;
    t.cols = cols;
    t.dtype = dtype;
    e->layers[layer_idx].dirty = true;
    if (weight_type >= WT_ROUTER_WEIGHT && weight_type <= WT_ROUTER_BIASES) return build_router(e, layer_idx);
    if (weight_type >= WT_SHARED_UP_W) return build_shared(e, layer_idx);
    return 0;
}

extern "C" int bakan_forward_moe_block(void* engine, int layer_idx, const void* h_f16, void* output_f16) {
    return run_block(static_cast<FwdEngine*>(engine), layer_idx, h_f16, output_f16, false);
}

extern "C" int bakan_forward_moe_block_normed(void* engine, int layer_idx, const void* x_f16, void* output_f16) {
    return run_block(static_cast<FwdEngine*>(engine), layer_idx, x_f16, output_f16, true);
}

extern "C" int bakan_forward_num_layers(void* engine) {
    FwdEngine* e = static_cast<FwdEngine*>(engine);
    return e ? e->num_layers : 0;
}

extern "C" int kq_forward_set_params(void* engine, int top_k, float rms_norm_eps) {
    FwdEngine* e = static_cast<FwdEngine*>(engine);
    if (!e || top_k <= 0 || top_k > e->info.num_experts || top_k > 16 || !(rms_norm_eps >= 0.f)) return KQ_ERR_ARG;
    drop_graphs(e);
    e->top_k = top_k;
    e->eps = rms_norm_eps;
    return KQ_OK;
}

// ---- the MoE layers of the whole-model decode step (kq_full.cu) ----------------
namespace kq {

int moe_block_prepare(void* engine, int layer) {
    FwdEngine* e = static_cast<FwdEngine*>(engine);
    if (!e || layer < 0 || layer >= e->num_layers) return -1;
    if (const char* miss = block_missing(e, layer, false)) {
        fprintf(stderr, "[kandiga] ERROR: layer %d has no %s weights\n", layer, miss);
        return -1;
    }
    return ensure_ws(e) && finalize_layer(e, layer) == 0 ? 0 : -1;
}

int moe_block_enqueue(void* engine, int layer, const __half* in, __half* out, cudaStream_t s) {
    return enqueue_block_io(static_cast<FwdEngine*>(engine), layer, false, in, out, s);
}

int moe_block_hidden(void* engine) { return engine ? static_cast<FwdEngine*>(engine)->info.hidden : 0; }

uint32_t* moe_block_status(void* engine) {
    return engine ? static_cast<uint32_t*>(static_cast<FwdEngine*>(engine)->ws) : nullptr;
}

}  // namespace kq

extern "C" void bakan_forward_destroy(void* engine) {
    FwdEngine* e = static_cast<FwdEngine*>(engine);
    if (!e) return;
    if (e->stream) cudaStreamSynchronize(e->stream);
    drop_graphs(e);
    for (FwdLayer& L : e->layers) {
        for (DevTensor& t : L.wt)
            if (t.p) cudaFree(t.p);
        if (L.router) kq_qmat_destroy(L.router);
        if (L.router_ext) kq_qmat_destroy(L.router_ext);
        if (L.norm16) cudaFree(L.norm16);
    }
    kq_table_destroy(e->routed);
    kq_table_destroy(e->shared);
    for (void* p : {(void*)e->dh, (void*)e->dnorm, (void*)e->dshared, (void*)e->dout, (void*)e->dlogits,
                    (void*)e->droute, (void*)e->dgate, (void*)e->dones, (void*)e->dw, (void*)e->dgw, (void*)e->didx,
                    (void*)e->dzero, (void*)e->dgidx, e->ws})
        if (p) cudaFree(p);
    if (e->hstage) cudaFreeHost(e->hstage);
    if (e->hstatus) cudaFreeHost(e->hstatus);
    if (e->stream) cudaStreamDestroy(e->stream);
    delete e;
    fprintf(stderr, "[kandiga] MoE block engine destroyed\n");
}
