// kq_spill.cu -- routed-expert tables larger than HBM: the whole table in
// pinned, device-mapped host memory, a per-layer pool of expert slots in HBM.
//
// The reference serves such models from the SSD: each call preads the routed
// experts (kandiga/metal/kandiga_cpu_expert.m:495-515) and a background thread
// warms the page cache for the experts a cross-layer predictor expects next
// (kandiga/engine.py:577-668).  Here the slow tier is host memory over the
// host link and the fast tier is an HBM slot pool, and the residency decisions
// are made on the GPU, in stream order, so a decode step needs no host round
// trip and can be captured in a CUDA graph:
//
//   spill_assign_kernel (one CTA)  ids -> requested-expert bitmap; resident
//       experts get this call's stamp; missing experts, in expert-id order,
//       take the slots with the oldest stamps among those this call does not
//       name (ties: lowest slot); writes the (expert, slot) copy list, the
//       slot ids and the counters.
//   spill_copy_kernel (a few CTAs)  copies the listed experts from host
//       memory into their slots with 16-byte loads, eight in flight per thread,
//       so a handful of CTAs keep the host link busy and the rest of the GPU
//       stays free for the layer that is computing.
//
// Device state, one block: slot_of [L][E] (slot or -1), owner [L][S] (expert
// or -1), stamp [L][S], clock [L], copy list [L][1 + 2S], counters [4].
#include "kq_internal.h"
#include "kq_common.cuh"

#include <new>

#ifndef KQ_SPILL_COPY_CTAS
#define KQ_SPILL_COPY_CTAS 16  // 16, 64 and 148 CTAs all copy at ~49.6 GB/s; fewest SMs taken
#endif

struct kq_spill {
    kq_table* pool = nullptr;
    uint8_t* host = nullptr;  // pinned, mapped; [L][E][expert_bytes]
    uint8_t* host_dev = nullptr;
    int L = 0, E = 0, S = 0;
    size_t eb = 0;
    void* state = nullptr;
    int32_t* slot_of = nullptr;
    int32_t* owner = nullptr;
    uint32_t* stamp = nullptr;
    uint32_t* clock = nullptr;
    int32_t* copy = nullptr;
    unsigned long long* counters = nullptr;
};

namespace kq {

constexpr int SP_THREADS = 1024;
constexpr int SP_MAX_EXPERTS = 16384;
constexpr int SP_MAX_SLOTS = 1024;
constexpr int SP_COPY_THREADS = 256;
constexpr int SP_COPY_UNROLL = 8;

struct SpillArgs {
    int32_t* slot_of;
    int32_t* owner;
    uint32_t* stamp;
    uint32_t* clock;
    int32_t* copy;
    unsigned long long* counters;  // hits, misses, bytes, status
    const int32_t* ids;
    int32_t* slot_ids;
    int n, layer, E, S;
    int fetch;  // 1: kq_spill_fetch (slot ids, capacity status); 0: prefetch
    unsigned long long eb;
};

__global__ void __launch_bounds__(SP_THREADS) spill_assign_kernel(SpillArgs a) {
    __shared__ uint32_t req[SP_MAX_EXPERTS / 32];
    __shared__ int32_t miss[SP_MAX_SLOTS];
    __shared__ uint32_t sst[SP_MAX_SLOTS];
    __shared__ int wcount[SP_THREADS / 32];
    __shared__ int chunk_total, hsum;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    pdl_wait();  // ids and the state come from earlier work on the stream
    pdl_launch_dependents();
    int32_t* slot_of = a.slot_of + (size_t)a.layer * a.E;
    int32_t* owner = a.owner + (size_t)a.layer * a.S;
    uint32_t* stamp = a.stamp + (size_t)a.layer * a.S;
    int32_t* copy = a.copy + (size_t)a.layer * (1 + 2 * a.S);
    const uint32_t t = a.clock[a.layer] + 1u;

    const int words = (a.E + 31) >> 5;
    for (int w = tid; w < words; w += SP_THREADS) req[w] = 0u;
    if (tid == 0) hsum = 0;
    __syncthreads();
    int bad = 0;
    for (int i = tid; i < a.n; i += SP_THREADS) {
        const int e = a.ids[i];
        if (e < 0 || e >= a.E) bad = 1;
        else atomicOr(&req[e >> 5], 1u << (e & 31));
    }
    bad = __syncthreads_or(bad);

    // resident experts keep their slot (stamp refreshed); missing ones are
    // listed in expert-id order by a block-wide compaction
    int hits = 0, m_total = 0;
    for (int e0 = 0; e0 < a.E; e0 += SP_THREADS) {
        const int e = e0 + tid;
        const bool want = e < a.E && ((req[e >> 5] >> (e & 31)) & 1u);
        const int s = want ? slot_of[e] : -1;
        if (want && s >= 0) {
            stamp[s] = t;
            ++hits;
        }
        const bool m = want && s < 0;
        const uint32_t bal = __ballot_sync(0xffffffffu, m);
        if (lane == 0) wcount[warp] = __popc(bal);
        __syncthreads();
        if (warp == 0) {
            const int v = wcount[lane];
            int incl = v;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int u = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += u;
            }
            wcount[lane] = incl - v;
            if (lane == 31) chunk_total = incl;
        }
        __syncthreads();
        if (m) {
            const int pos = m_total + wcount[warp] + __popc(bal & ((1u << lane) - 1u));
            if (pos < a.S) miss[pos] = e;
        }
        m_total += chunk_total;
        __syncthreads();
    }

    // victims: slots this call does not name, oldest stamp first (ties: lowest slot)
    int served = 0;
    if (m_total > 0) {
        for (int s = tid; s < a.S; s += SP_THREADS) sst[s] = stamp[s];
        __syncthreads();
        const bool cand = tid < a.S && sst[tid] != t;
        const int n_cand = __syncthreads_count(cand);
        served = min(m_total, n_cand);
        if (cand) {
            const uint32_t my = sst[tid];
            int rank = 0;
            for (int j = 0; j < a.S; ++j) {
                const uint32_t o = sst[j];
                rank += (o != t) && (o < my || (o == my && j < tid));
            }
            if (rank < served) {
                const int e = miss[rank];
                const int old = owner[tid];
                if (old >= 0) slot_of[old] = -1;
                owner[tid] = e;
                slot_of[e] = tid;
                stamp[tid] = t;
                copy[1 + 2 * rank] = e;
                copy[2 + 2 * rank] = tid;
            }
        }
        __syncthreads();
    }

    if (a.fetch && a.slot_ids) {
        for (int i = tid; i < a.n; i += SP_THREADS) {
            const int e = a.ids[i];
            a.slot_ids[i] = (e >= 0 && e < a.E) ? slot_of[e] : -1;
        }
    }
    if (hits) atomicAdd(&hsum, hits);
    __syncthreads();
    if (tid == 0) {
        copy[0] = served;
        a.clock[a.layer] = t;
        atomicAdd(&a.counters[0], (unsigned long long)hsum);
        atomicAdd(&a.counters[1], (unsigned long long)served);
        atomicAdd(&a.counters[2], (unsigned long long)served * a.eb);
        unsigned long long st = 0;
        if (bad) st |= KQ_DEV_BAD_EXPERT;
        if (a.fetch && served < m_total) st |= KQ_DEV_CAPACITY;
        if (st) atomicOr(&a.counters[3], st);
    }
}

// Copies the listed experts host -> HBM.  The m listed experts are one flat
// run of m * (expert_bytes / 16) 16-byte vectors, strided over every thread of
// the grid with eight loads in flight per thread, so the last pass is not
// partly idle for each expert.  The host pointer is not __restrict__, so its
// loads stay on the coherent global path.
__global__ void __launch_bounds__(SP_COPY_THREADS) spill_copy_kernel(const uint8_t* host,
                                                                      uint8_t* __restrict__ pool,
                                                                      const int32_t* __restrict__ copy, int layer,
                                                                      int E, int S, unsigned long long eb) {
    pdl_wait();  // the assign kernel has completed: the copy list is final
    pdl_launch_dependents();
    const int m = copy[(size_t)layer * (1 + 2 * S)];
    const int32_t* list = copy + (size_t)layer * (1 + 2 * S) + 1;
    const unsigned long long nvec = eb / 16;
    const unsigned long long total = (unsigned long long)m * nvec;
    const unsigned long long stride = (unsigned long long)gridDim.x * SP_COPY_THREADS;
    const uint4* hsrc = reinterpret_cast<const uint4*>(host + (size_t)layer * E * eb);
    uint4* pdst = reinterpret_cast<uint4*>(pool + (size_t)layer * S * eb);
    for (unsigned long long i0 = (unsigned long long)blockIdx.x * SP_COPY_THREADS + threadIdx.x; i0 < total;
         i0 += stride * SP_COPY_UNROLL) {
        uint4 r[SP_COPY_UNROLL];
        unsigned long long d[SP_COPY_UNROLL];
#pragma unroll
        for (int u = 0; u < SP_COPY_UNROLL; ++u) {
            const unsigned long long i = i0 + (unsigned long long)u * stride;
            if (i < total) {
                const unsigned long long j = i / nvec, k = i - j * nvec;
                r[u] = hsrc[(unsigned long long)list[2 * j] * nvec + k];
                d[u] = (unsigned long long)list[2 * j + 1] * nvec + k;
            }
        }
#pragma unroll
        for (int u = 0; u < SP_COPY_UNROLL; ++u) {
            const unsigned long long i = i0 + (unsigned long long)u * stride;
            if (i < total) pdst[d[u]] = r[u];
        }
    }
}

}  // namespace kq

using namespace kq;

extern "C" int kq_spill_create(const kq_table_desc* desc, int slots, kq_spill** out) {
    if (!out || !desc) return KQ_ERR_ARG;
    *out = nullptr;
    if (desc->num_experts <= 0 || desc->num_experts > SP_MAX_EXPERTS) return KQ_ERR_ARG;
    if (slots <= 0 || slots > SP_MAX_SLOTS || slots > desc->num_experts) return KQ_ERR_ARG;
    kq_table_desc pd = *desc;
    pd.num_experts = slots;
    kq_spill* s = new (std::nothrow) kq_spill();
    if (!s) return KQ_ERR_ALLOC;
    int rc = kq_table_create(&pd, &s->pool);
    if (rc) {
        delete s;
        return rc;
    }
    s->L = desc->num_layers;
    s->E = desc->num_experts;
    s->S = slots;
    s->eb = s->pool->expert_bytes;
    const size_t host_bytes = (size_t)s->L * s->E * s->eb;
    if (cudaHostAlloc(reinterpret_cast<void**>(&s->host), host_bytes, cudaHostAllocMapped | cudaHostAllocPortable) !=
        cudaSuccess) {
        cudaGetLastError();
        kq_table_destroy(s->pool);
        delete s;
        return KQ_ERR_ALLOC;
    }
    if (cudaHostGetDevicePointer(reinterpret_cast<void**>(&s->host_dev), s->host, 0) != cudaSuccess) {
        cudaGetLastError();
        cudaFreeHost(s->host);
        kq_table_destroy(s->pool);
        delete s;
        return KQ_ERR_CUDA;
    }
    const size_t n_slot_of = (size_t)s->L * s->E, n_slot = (size_t)s->L * s->S;
    const size_t n_copy = (size_t)s->L * (1 + 2 * s->S);
    const size_t bytes = 4 * n_slot_of + 4 * n_slot * 2 + 4 * (size_t)s->L + 4 * n_copy + 4 * 8;
    const size_t bytes_aligned = (bytes + 255) & ~(size_t)255;
    if (cudaMalloc(&s->state, bytes_aligned + 64) != cudaSuccess) {
        cudaGetLastError();
        cudaFreeHost(s->host);
        kq_table_destroy(s->pool);
        delete s;
        return KQ_ERR_ALLOC;
    }
    uint8_t* p = static_cast<uint8_t*>(s->state);
    s->counters = reinterpret_cast<unsigned long long*>(p);  // 64 B at the front keeps it 8-aligned
    p += 64;
    s->slot_of = reinterpret_cast<int32_t*>(p);
    p += 4 * n_slot_of;
    s->owner = reinterpret_cast<int32_t*>(p);
    p += 4 * n_slot;
    s->stamp = reinterpret_cast<uint32_t*>(p);
    p += 4 * n_slot;
    s->clock = reinterpret_cast<uint32_t*>(p);
    p += 4 * (size_t)s->L;
    s->copy = reinterpret_cast<int32_t*>(p);
    // empty residency: slot_of / owner -1, stamps / clocks / copy counts / counters 0
    cudaError_t e = cudaMemset(s->state, 0, bytes_aligned + 64);
    if (e == cudaSuccess) e = cudaMemset(s->slot_of, 0xFF, 4 * (n_slot_of + n_slot));
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        kq_spill_destroy(s);
        return KQ_ERR_CUDA;
    }
    *out = s;
    return KQ_OK;
}

extern "C" int kq_spill_destroy(kq_spill* s) {
    if (!s) return KQ_OK;
    if (s->state) cudaFree(s->state);
    if (s->host) cudaFreeHost(s->host);
    if (s->pool) kq_table_destroy(s->pool);
    delete s;
    return KQ_OK;
}

extern "C" const kq_table* kq_spill_pool(const kq_spill* s) { return s ? s->pool : nullptr; }

extern "C" size_t kq_spill_host_bytes(const kq_spill* s) { return s ? (size_t)s->L * s->E * s->eb : 0; }

extern "C" int kq_spill_store_layer(kq_spill* s, int layer, const kq_table* src, int src_layer, void* stream) {
    if (!s || !src) return KQ_ERR_ARG;
    if (layer < 0 || layer >= s->L || src_layer < 0 || src_layer >= src->d.num_layers) return KQ_ERR_ARG;
    const kq_table_desc& a = src->d;
    const kq_table_desc& b = s->pool->d;
    if (a.num_experts != s->E || a.hidden != b.hidden || a.inter != b.inter || a.bits != b.bits ||
        a.group_size != b.group_size || a.sb_dtype != b.sb_dtype || a.activation != b.activation)
        return KQ_ERR_ARG;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const size_t lb = (size_t)s->E * s->eb;
    cudaError_t e = cudaMemcpyAsync(s->host + (size_t)layer * lb, src->base + (size_t)src_layer * src->layer_bytes, lb,
                                    cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(s->slot_of + (size_t)layer * s->E, 0xFF, 4 * (size_t)s->E, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(s->owner + (size_t)layer * s->S, 0xFF, 4 * (size_t)s->S, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(s->stamp + (size_t)layer * s->S, 0, 4 * (size_t)s->S, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(s->clock + layer, 0, 4, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);  // the host store is complete on return
    return e == cudaSuccess ? KQ_OK : KQ_ERR_CUDA;
}

static int spill_run(kq_spill* s, int layer, const int32_t* ids, int n, int32_t* slot_ids, int fetch,
                     void* stream) {
    if (!s || layer < 0 || layer >= s->L || n < 0 || (n > 0 && !ids)) return KQ_ERR_ARG;
    if (n == 0) return KQ_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    SpillArgs a;
    a.slot_of = s->slot_of;
    a.owner = s->owner;
    a.stamp = s->stamp;
    a.clock = s->clock;
    a.copy = s->copy;
    a.counters = s->counters;
    a.ids = ids;
    a.slot_ids = slot_ids;
    a.n = n;
    a.layer = layer;
    a.E = s->E;
    a.S = s->S;
    a.fetch = fetch;
    a.eb = s->eb;
    // Both kernels are launched as programmatic dependents of their
    // predecessor: each starts with griddepcontrol.wait (its predecessor has
    // completed and its writes are visible) and then releases its own
    // dependents, so launch latency overlaps the previous kernel.
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.stream = st;
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(SP_THREADS);
    cudaError_t e = cudaLaunchKernelEx(&cfg, spill_assign_kernel, a);
    if (e == cudaSuccess) {
        cfg.gridDim = dim3(KQ_SPILL_COPY_CTAS);
        cfg.blockDim = dim3(SP_COPY_THREADS);
        e = cudaLaunchKernelEx(&cfg, spill_copy_kernel, (const uint8_t*)s->host_dev, s->pool->base,
                               (const int32_t*)s->copy, layer, s->E, s->S, (unsigned long long)s->eb);
    }
    return e == cudaSuccess ? KQ_OK : KQ_ERR_CUDA;
}

extern "C" int kq_spill_fetch(kq_spill* s, int layer, const int32_t* ids, int n, int32_t* slot_ids, void* stream) {
    return spill_run(s, layer, ids, n, slot_ids, 1, stream);
}

extern "C" int kq_spill_prefetch(kq_spill* s, int layer, const int32_t* ids, int n, void* stream) {
    return spill_run(s, layer, ids, n, nullptr, 0, stream);
}

extern "C" int kq_spill_stats(kq_spill* s, uint64_t out[4], int reset, void* stream) {
    if (!s || !out) return KQ_ERR_ARG;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemcpyAsync(out, s->counters, 4 * sizeof(uint64_t), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess && reset) e = cudaMemsetAsync(s->counters, 0, 4 * sizeof(uint64_t), st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    return e == cudaSuccess ? KQ_OK : KQ_ERR_CUDA;
}

extern "C" int kq_spill_residency(const kq_spill* s, int layer, int32_t* slot_of, int32_t* owner, void* stream) {
    if (!s || layer < 0 || layer >= s->L) return KQ_ERR_ARG;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaSuccess;
    if (slot_of)
        e = cudaMemcpyAsync(slot_of, s->slot_of + (size_t)layer * s->E, 4 * (size_t)s->E, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess && owner)
        e = cudaMemcpyAsync(owner, s->owner + (size_t)layer * s->S, 4 * (size_t)s->S, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    return e == cudaSuccess ? KQ_OK : KQ_ERR_CUDA;
}
