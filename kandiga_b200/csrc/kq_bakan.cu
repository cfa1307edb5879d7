// kq_bakan.cu -- reference-compatible host ABI (bakan_cpu_expert_*).
//
// The reference's native library (kandiga/metal/kandiga_cpu_expert.m) preads K
// experts from the BKEX layer files on every call and computes them on CPU
// cores.  Here init reads every layer file once into the HBM table, and each
// call is: host -> device copy of x and the expert ids, the sm_100a decode
// (one token) or grouped prefill kernels, device -> host copy of the
// per-expert outputs; a single-token call replays one CUDA graph.  Calls are
// synchronous and, like the reference, not re-entrant per engine.
// Errors: -1 with a "[kandiga] ERROR: ..." line on stderr, as the reference.
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <vector>

#include "kq_internal.h"

namespace kq {

int load_bkex_dir(const char* packed_dir, int num_layers, cudaStream_t s, kq_table** out, BkexInfo* info,
                  int extra_experts) {
    *out = nullptr;
    kq_table* table = nullptr;
    auto fail = [&]() {
        if (table) kq_table_destroy(table);
        return -1;
    };
    std::vector<uint8_t> file;
    for (int l = 0; l < num_layers; ++l) {
        char path[1024];
        snprintf(path, sizeof(path), "%s/layer_%02d.bin", packed_dir, l);
        FILE* f = fopen(path, "rb");
        if (!f) {
            fprintf(stderr, "[kandiga] ERROR: Cannot open %s\n", path);
            return fail();
        }
        fseek(f, 0, SEEK_END);
        const long n = ftell(f);
        fseek(f, 0, SEEK_SET);
        file.resize(n > 0 ? (size_t)n : 0);
        const size_t got = n > 0 ? fread(file.data(), 1, (size_t)n, f) : 0;
        fclose(f);
        if (n <= 0 || got != (size_t)n) {
            fprintf(stderr, "[kandiga] ERROR: read failed for %s\n", path);
            return fail();
        }
        if (l == 0) {
            if (bkex_parse(file.data(), file.size(), info) != KQ_OK) {
                fprintf(stderr, "[kandiga] ERROR: %s is not a BKEX layer file\n", path);
                return fail();
            }
            kq_table_desc d{};
            d.num_layers = num_layers;
            d.num_experts = info->num_experts + extra_experts;
            d.hidden = info->hidden;
            d.inter = info->inter;
            d.bits = info->bits;
            d.group_size = 64;
            d.sb_dtype = info->sb_dtype;
            d.activation = info->activation;
            if (kq_table_create(&d, &table) != KQ_OK) {
                fprintf(stderr, "[kandiga] ERROR: cannot create the HBM expert table\n");
                return fail();
            }
        }
        if (kq_table_load_bkex(table, l, file.data(), file.size(), s) != KQ_OK) {
            fprintf(stderr, "[kandiga] ERROR: cannot load %s\n", path);
            return fail();
        }
    }
    *out = table;
    return 0;
}

}  // namespace kq

using namespace kq;

namespace {

constexpr int kMaxExperts = 16;  // MAX_EXPERTS, kandiga/metal/kandiga_cpu_expert.m:37

struct Engine {
    kq_table* table = nullptr;
    BkexInfo info{};
    int num_layers = 0;
    cudaStream_t stream = nullptr;
    // device scratch, grown on demand (never on the single-token path after init)
    void* ws = nullptr;
    size_t ws_bytes = 0;
    int ws_tokens = 0;
    void* dx = nullptr;
    size_t dx_bytes = 0;
    void* dout = nullptr;
    size_t dout_bytes = 0;
    int32_t* didx = nullptr;
    size_t didx_bytes = 0;
    uint32_t* hstatus = nullptr;  // pinned, mapped host word the device status is copied into
    uint32_t* hstatus_d = nullptr;  // its device address
    // Single-token calls: pinned, mapped staging [x: H*4 | ids: kMaxExperts*4 |
    // out: kMaxExperts*H*4] and one instantiated CUDA graph per (layer, K, x
    // dtype, out dtype): a stage-in kernel (x and ids from the mapped stage to
    // the device), the decode kernels, a stage-out kernel (outputs and the
    // status word straight into the mapped stage, status cleared).  Kernels
    // instead of copy-engine nodes: each copy node costs microseconds of
    // copy-engine latency, which dominated the call.  The graphs hold the
    // device buffers' addresses, so any reallocation drops them.
    uint8_t* hstage = nullptr;
    uint8_t* hstage_d = nullptr;  // its device address
    std::map<uint64_t, cudaGraphExec_t> graphs;
};

// x (n16 16-byte units) and K ids from the mapped host stage to the device.
__global__ void stage_in_kernel(const uint4* __restrict__ hx, uint4* __restrict__ dx, int n16,
                                const int32_t* __restrict__ hidx, int32_t* __restrict__ didx, int K) {
    for (int i = threadIdx.x; i < n16; i += blockDim.x) dx[i] = hx[i];
    if (threadIdx.x < K) didx[threadIdx.x] = hidx[threadIdx.x];
}

// outputs (n16 16-byte units) into the mapped host stage; the device status
// word into its mapped host word, then cleared for the next call.
__global__ void stage_out_kernel(const uint4* __restrict__ dout, uint4* __restrict__ hout, int n16,
                                 uint32_t* ws_status, uint32_t* hstatus) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += gridDim.x * blockDim.x) hout[i] = dout[i];
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        *hstatus = *ws_status;
        *ws_status = 0u;
    }
}

void drop_graphs(Engine* e) {
    for (auto& kv : e->graphs) cudaGraphExecDestroy(kv.second);
    e->graphs.clear();
}

bool grow(void** p, size_t* have, size_t need) {
    if (*have >= need) return true;
    if (*p) cudaFree(*p);
    *p = nullptr;
    *have = 0;
    if (cudaMalloc(p, need) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    *have = need;
    return true;
}

// Many tokens go through the grouped tensor-core path (every expert once over
// its tokens); one or a few tokens through the decode kernels.
bool use_prefill(const Engine* e, int T) {
    return T >= 16 && e->info.hidden % 512 == 0 && e->info.inter % 512 == 0;
}

size_t ws_need(const Engine* e, int T, int K) {
    return use_prefill(e, T) ? kq_moe_prefill_workspace_size(e->table, T, K)
                             : kq_moe_workspace_size(e->table, T, K);
}

bool ensure(Engine* e, int T, int K) {
    const int H = e->info.hidden;
    if (!e->hstatus) {
        if (cudaHostAlloc(reinterpret_cast<void**>(&e->hstatus), 4, cudaHostAllocMapped) != cudaSuccess ||
            cudaHostGetDevicePointer(reinterpret_cast<void**>(&e->hstatus_d), e->hstatus, 0) != cudaSuccess) {
            cudaGetLastError();
            if (e->hstatus) cudaFreeHost(e->hstatus);
            e->hstatus = nullptr;
            return false;
        }
    }
    if (!e->hstage) {
        if (cudaHostAlloc(reinterpret_cast<void**>(&e->hstage),
                          (size_t)H * 4 + kMaxExperts * 4 + (size_t)kMaxExperts * H * 4,
                          cudaHostAllocMapped) != cudaSuccess ||
            cudaHostGetDevicePointer(reinterpret_cast<void**>(&e->hstage_d), e->hstage, 0) != cudaSuccess) {
            cudaGetLastError();
            if (e->hstage) cudaFreeHost(e->hstage);
            e->hstage = nullptr;
            return false;
        }
    }
    if (e->dx_bytes < (size_t)T * H * 4 || e->dout_bytes < (size_t)T * K * H * 4 ||
        e->didx_bytes < (size_t)T * K * 4 || T > e->ws_tokens || e->ws_bytes < ws_need(e, T, K))
        drop_graphs(e);
    if (!grow(&e->dx, &e->dx_bytes, (size_t)T * H * 4)) return false;
    if (!grow(&e->dout, &e->dout_bytes, (size_t)T * K * H * 4)) return false;
    if (!grow(reinterpret_cast<void**>(&e->didx), &e->didx_bytes, (size_t)T * K * 4)) return false;
    if (T > e->ws_tokens || e->ws_bytes < ws_need(e, T, K)) {
        size_t need = std::max(ws_need(e, std::max(T, e->ws_tokens), kMaxExperts),
                               kq_moe_workspace_size(e->table, std::max(T, e->ws_tokens), kMaxExperts));
        if (e->ws) cudaFree(e->ws);
        e->ws = nullptr;
        e->ws_bytes = 0;
        if (cudaMalloc(&e->ws, need) != cudaSuccess) {
            cudaGetLastError();
            return false;
        }
        e->ws_bytes = need;
        e->ws_tokens = std::max(T, e->ws_tokens);
        if (kq_workspace_init(e->ws, need, e->stream) != KQ_OK) return false;
    }
    return true;
}

int check_call(Engine* e, int layer, const int32_t* idx, int n, int K) {
    if (!e) return -1;
    if (layer < 0 || layer >= e->num_layers) {
        fprintf(stderr, "[kandiga] ERROR: layer_idx %d out of range [0, %d)\n", layer, e->num_layers);
        return -1;
    }
    if (K <= 0 || K > kMaxExperts) {
        fprintf(stderr, "[kandiga] ERROR: num_experts %d out of range [1, %d]\n", K, kMaxExperts);
        return -1;
    }
    for (int i = 0; i < n; ++i)
        if (idx[i] < 0 || idx[i] >= e->info.num_experts) {
            fprintf(stderr, "[kandiga] ERROR: expert index %d out of range [0, %d)\n", idx[i],
                    e->info.num_experts);
            return -1;
        }
    return 0;
}

// Enqueue on e->stream: host -> device copy of x [T][H] and idx [T][K], the
// expert kernels into e->dout [T][K][H] (out_dtype).  Nothing is copied back.
int launch(Engine* e, int layer, const void* x, int x_dtype, const int32_t* idx, int T, int K, int out_dtype) {
    if (!ensure(e, T, K)) {
        fprintf(stderr, "[kandiga] ERROR: device allocation failed\n");
        return -1;
    }
    const size_t xb = (size_t)T * e->info.hidden * (x_dtype == KQ_DT_F32 ? 4 : 2);
    cudaStream_t s = e->stream;
    if (cudaMemcpyAsync(e->dx, x, xb, cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaMemcpyAsync(e->didx, idx, (size_t)T * K * 4, cudaMemcpyHostToDevice, s) != cudaSuccess) {
        fprintf(stderr, "[kandiga] ERROR: host->device copy failed for layer %d\n", layer);
        return -1;
    }
    int rc = (use_prefill(e, T) ? kq_moe_prefill : kq_moe_decode)(e->table, layer, e->dx, x_dtype, T, nullptr,
                                                                 e->didx, nullptr, K, e->dout, nullptr, out_dtype,
                                                                 nullptr, e->ws, e->ws_bytes, s);
    if (rc != KQ_OK) {
        fprintf(stderr, "[kandiga] ERROR: expert kernels failed for layer %d (code %d)\n", layer, rc);
        return -1;
    }
    return 0;
}

// Copy rows [r0, r1) of e->dout (row = one (token, k) output of `row` bytes) to host `out`.
int copy_rows(Engine* e, int layer, void* out, size_t row, size_t r0, size_t r1) {
    if (cudaMemcpyAsync(static_cast<uint8_t*>(out) + r0 * row, static_cast<const uint8_t*>(e->dout) + r0 * row,
                        (r1 - r0) * row, cudaMemcpyDeviceToHost, e->stream) != cudaSuccess) {
        fprintf(stderr, "[kandiga] ERROR: Expert computation failed for layer %d\n", layer);
        return -1;
    }
    return 0;
}

// Copy and clear the kernels' device status word behind the output copies,
// wait for the stream once, then check the word.
int finish(Engine* e, int layer) {
    *e->hstatus = 0;
    if (cudaMemcpyAsync(e->hstatus, e->ws, 4, cudaMemcpyDeviceToHost, e->stream) != cudaSuccess ||
        cudaMemsetAsync(e->ws, 0, 4, e->stream) != cudaSuccess || cudaStreamSynchronize(e->stream) != cudaSuccess) {
        fprintf(stderr, "[kandiga] ERROR: Expert computation failed for layer %d\n", layer);
        return -1;
    }
    if (*e->hstatus != 0) {
        fprintf(stderr, "[kandiga] ERROR: device status 0x%x for layer %d\n", *e->hstatus, layer);
        return -1;
    }
    return 0;
}

// Run T tokens x K experts: x host [T][H] in x_dtype -> out host [T][K][H] in out_dtype.
int run(Engine* e, int layer, const void* x, int x_dtype, const int32_t* idx, int T, int K,
        void* out, int out_dtype) {
    if (launch(e, layer, x, x_dtype, idx, T, K, out_dtype)) return -1;
    const size_t row = (size_t)e->info.hidden * (out_dtype == KQ_DT_F32 ? 4 : 2);
    if (copy_rows(e, layer, out, row, 0, (size_t)T * K)) return -1;
    return finish(e, layer);
}

// One token x K experts through the engine's CUDA graph for (layer, K, dtypes):
// the caller's x and ids are staged in pinned memory, one graph launch, one
// synchronize, the outputs copied out of the pinned stage.
int run_one(Engine* e, int layer, const void* x, int x_dtype, const int32_t* idx, int K, void* out,
            int out_dtype) {
    if (!ensure(e, 1, K)) {
        fprintf(stderr, "[kandiga] ERROR: device allocation failed\n");
        return -1;
    }
    const int H = e->info.hidden;
    const size_t xb = (size_t)H * (x_dtype == KQ_DT_F32 ? 4 : 2);
    const size_t ob = (size_t)K * H * (out_dtype == KQ_DT_F32 ? 4 : 2);
    uint8_t* hx = e->hstage;
    int32_t* hidx = reinterpret_cast<int32_t*>(e->hstage + (size_t)H * 4);
    uint8_t* hout = e->hstage + (size_t)H * 4 + kMaxExperts * 4;
    const uint64_t key = ((uint64_t)layer << 24) | ((uint64_t)K << 16) | ((uint64_t)x_dtype << 8) | (uint64_t)out_dtype;
    auto it = e->graphs.find(key);
    if (it == e->graphs.end()) {
        cudaStream_t s = e->stream;
        cudaGraph_t graph = nullptr;
        if (cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal) != cudaSuccess) {
            fprintf(stderr, "[kandiga] ERROR: graph capture failed for layer %d\n", layer);
            return -1;
        }
        const uint8_t* hx_d = e->hstage_d;
        const int32_t* hidx_d = reinterpret_cast<const int32_t*>(e->hstage_d + (size_t)H * 4);
        uint8_t* hout_d = e->hstage_d + (size_t)H * 4 + kMaxExperts * 4;
        stage_in_kernel<<<1, 256, 0, s>>>(reinterpret_cast<const uint4*>(hx_d), static_cast<uint4*>(e->dx),
                                          (int)(xb / 16), hidx_d, e->didx, K);
        bool ok = cudaGetLastError() == cudaSuccess;
        ok = ok && kq_moe_decode(e->table, layer, e->dx, x_dtype, 1, nullptr, e->didx, nullptr, K, e->dout, nullptr,
                                 out_dtype, nullptr, e->ws, e->ws_bytes, s) == KQ_OK;
        if (ok) {
            stage_out_kernel<<<16, 256, 0, s>>>(static_cast<const uint4*>(e->dout), reinterpret_cast<uint4*>(hout_d),
                                                (int)(ob / 16), static_cast<uint32_t*>(e->ws), e->hstatus_d);
            ok = cudaGetLastError() == cudaSuccess;
        }
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
    memcpy(hx, x, xb);
    memcpy(hidx, idx, (size_t)K * 4);
    *e->hstatus = 0;
    if (cudaGraphLaunch(it->second, e->stream) != cudaSuccess || cudaStreamSynchronize(e->stream) != cudaSuccess) {
        fprintf(stderr, "[kandiga] ERROR: Expert computation failed for layer %d\n", layer);
        return -1;
    }
    if (*e->hstatus != 0) {
        fprintf(stderr, "[kandiga] ERROR: device status 0x%x for layer %d\n", *e->hstatus, layer);
        return -1;
    }
    memcpy(out, hout, ob);
    return 0;
}

}  // namespace

extern "C" void bakan_cpu_expert_destroy(void* engine_ptr);

extern "C" void* bakan_cpu_expert_init(const char* packed_dir, int num_layers) {
    if (!packed_dir || num_layers <= 0) {
        fprintf(stderr, "[kandiga] ERROR: bad arguments to init\n");
        return nullptr;
    }
    Engine* e = new (std::nothrow) Engine();
    if (!e) {
        fprintf(stderr, "[kandiga] ERROR: Failed to allocate engine\n");
        return nullptr;
    }
    e->num_layers = num_layers;
    if (cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking) != cudaSuccess) {
        fprintf(stderr, "[kandiga] ERROR: no CUDA device\n");
        delete e;
        return nullptr;
    }
    if (load_bkex_dir(packed_dir, num_layers, e->stream, &e->table, &e->info)) {
        bakan_cpu_expert_destroy(e);
        return nullptr;
    }
    if (!ensure(e, 1, kMaxExperts)) {
        fprintf(stderr, "[kandiga] ERROR: device allocation failed\n");
        bakan_cpu_expert_destroy(e);
        return nullptr;
    }
    fprintf(stderr, "[kandiga] Initialized: %d layers, %d experts (%zu KB each), %d-bit, HBM-resident\n",
            num_layers, e->info.num_experts, (size_t)e->info.expert_size / 1024, e->info.bits);
    return e;
}

extern "C" int bakan_cpu_expert_mlp(void* engine, int layer_idx, const float* x_f32,
                                    const int32_t* expert_indices, int num_experts, float* output_f32) {
    Engine* e = static_cast<Engine*>(engine);
    if (check_call(e, layer_idx, expert_indices, num_experts, num_experts)) return -1;
    return run_one(e, layer_idx, x_f32, KQ_DT_F32, expert_indices, num_experts, output_f32, KQ_DT_F32);
}

extern "C" int bakan_cpu_expert_mlp_f16(void* engine, int layer_idx, const void* x_f16,
                                        const int32_t* expert_indices, int num_experts,
                                        void* output_f16) {
    Engine* e = static_cast<Engine*>(engine);
    if (check_call(e, layer_idx, expert_indices, num_experts, num_experts)) return -1;
    return run_one(e, layer_idx, x_f16, KQ_DT_F16, expert_indices, num_experts, output_f16, KQ_DT_F16);
}

extern "C" int bakan_cpu_expert_mlp_bf16(void* engine, int layer_idx, const void* x_bf16,
                                         const int32_t* expert_indices, int num_experts,
                                         void* output_f16) {
    Engine* e = static_cast<Engine*>(engine);
    if (check_call(e, layer_idx, expert_indices, num_experts, num_experts)) return -1;
    return run_one(e, layer_idx, x_bf16, KQ_DT_BF16, expert_indices, num_experts, output_f16, KQ_DT_F16);
}

extern "C" int bakan_cpu_expert_mlp_batch_f16(void* engine, int layer_idx, const void* x_f16_batch,
                                              const int32_t* indices_batch, int num_tokens, int K,
                                              void* output_f16_batch) {
    Engine* e = static_cast<Engine*>(engine);
    if (!e || num_tokens <= 0) return -1;
    if (check_call(e, layer_idx, indices_batch, num_tokens * K, K)) return -1;
    return run(e, layer_idx, x_f16_batch, KQ_DT_F16, indices_batch, num_tokens, K, output_f16_batch,
               KQ_DT_F16);
}

extern "C" int bakan_cpu_expert_mlp_prefill_f16(void* engine, int layer_idx, const void* x_f16,
                                                int num_tokens, int K, int hidden_size,
                                                const int32_t* sorted_token_indices,
                                                const int32_t* sorted_expert_indices,
                                                const int32_t* sorted_k_positions,
                                                const int32_t* group_starts,
                                                const int32_t* unique_experts,
                                                int num_unique_experts, void* output_f16) {
    Engine* e = static_cast<Engine*>(engine);
    if (!e || layer_idx < 0 || layer_idx >= e->num_layers) return -1;
    if (num_tokens <= 0 || K <= 0 || K > kMaxExperts || hidden_size != e->info.hidden) return -1;
    if (num_unique_experts < 0) return -1;
    if (num_unique_experts == 0) return 0;
    const int total = group_starts[num_unique_experts];
    if (group_starts[0] < 0 || total < group_starts[0]) return -1;
    // Rebuild the [T][K] id table from the CSR groups; pairs no group covers
    // keep their output untouched, as in the reference.
    std::vector<int32_t> idx((size_t)num_tokens * K, 0);
    std::vector<uint8_t> covered((size_t)num_tokens * K, 0);
    for (int g = 0; g < num_unique_experts; ++g) {
        const int eid = unique_experts[g];
        if (eid < 0 || eid >= e->info.num_experts) {
            fprintf(stderr, "[kandiga] ERROR: expert index %d out of range\n", eid);
            return -1;
        }
        for (int i = group_starts[g]; i < group_starts[g + 1]; ++i) {
            const int t = sorted_token_indices[i], k = sorted_k_positions[i];
            if (t < 0 || t >= num_tokens || k < 0 || k >= K) return -1;
            idx[(size_t)t * K + k] = eid;
            covered[(size_t)t * K + k] = 1;
        }
    }
    (void)sorted_expert_indices;
    // Covered (token, k) rows are copied straight from HBM into the caller's
    // buffer, one copy per run of consecutive covered rows (one copy in total
    // when the groups cover every pair).
    if (launch(e, layer_idx, x_f16, KQ_DT_F16, idx.data(), num_tokens, K, KQ_DT_F16)) return -1;
    const size_t row = (size_t)hidden_size * 2, n = covered.size();
    for (size_t i = 0; i < n;) {
        if (!covered[i]) {
            ++i;
            continue;
        }
        size_t j = i;
        while (j < n && covered[j]) ++j;
        if (copy_rows(e, layer_idx, output_f16, row, i, j)) return -1;
        i = j;
    }
    return finish(e, layer_idx);
}

extern "C" int bakan_cpu_expert_pread_batch(void* engine, int layer_idx, const int32_t* expert_ids,
                                            int num_experts_to_read, void* output_buffer) {
    Engine* e = static_cast<Engine*>(engine);
    if (!e || layer_idx < 0 || layer_idx >= e->num_layers || num_experts_to_read < 0) return -1;
    if (num_experts_to_read == 0) return 0;
    if (!expert_ids || !output_buffer) return -1;
    const BkexInfo& I = e->info;
    const size_t esz = I.expert_size;
    void* dbuf = nullptr;
    if (cudaMalloc(&dbuf, esz) != cudaSuccess) {
        cudaGetLastError();
        return -1;
    }
    uint8_t* d = static_cast<uint8_t*>(dbuf);
    int rc = 0;
    for (int i = 0; i < num_experts_to_read && rc == 0; ++i) {
        const int eid = expert_ids[i];
        if (eid < 0 || eid >= I.num_experts) {
            rc = -1;
            break;
        }
        for (int m = 0; m < 3 && rc == 0; ++m)
            if (kq_table_unpack_mlx(e->table, layer_idx, eid, m, d + I.off[3 * m], d + I.off[3 * m + 1],
                                    d + I.off[3 * m + 2], e->stream) != KQ_OK)
                rc = -1;
        if (rc == 0 &&
            (cudaMemcpyAsync(static_cast<uint8_t*>(output_buffer) + (size_t)i * esz, d, esz,
                             cudaMemcpyDeviceToHost, e->stream) != cudaSuccess ||
             cudaStreamSynchronize(e->stream) != cudaSuccess))
            rc = -1;
    }
    cudaFree(dbuf);
    return rc;
}

extern "C" void bakan_cpu_expert_destroy(void* engine_ptr) {
    Engine* e = static_cast<Engine*>(engine_ptr);
    if (!e) return;
    if (e->stream) cudaStreamSynchronize(e->stream);
    kq_table_destroy(e->table);
    if (e->ws) cudaFree(e->ws);
    if (e->dx) cudaFree(e->dx);
    if (e->dout) cudaFree(e->dout);
    if (e->didx) cudaFree(e->didx);
    if (e->hstatus) cudaFreeHost(e->hstatus);
    drop_graphs(e);
    if (e->hstage) cudaFreeHost(e->hstage);
    if (e->stream) cudaStreamDestroy(e->stream);
    delete e;
    fprintf(stderr, "[kandiga] Engine destroyed\n");
}

extern "C" int bakan_cpu_expert_num_layers(void* engine_ptr) {
    Engine* e = static_cast<Engine*>(engine_ptr);
    return e ? e->num_layers : 0;
}
