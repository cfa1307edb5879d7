// kq_ep.cu -- expert-parallel MoE layer over peer memory (one rank per GPU of
// a node).
//
// The reference runs every expert of a token on one machine, in parallel over
// the K experts (kandiga/metal/kandiga_cpu_expert.m:522-543, a GCD loop).  At
// node scale the routed experts of a layer are partitioned over the ranks and
// tokens are data-parallel: each rank routes its own tokens, every token row
// travels once to every rank that owns one of its experts, that rank applies
// the weighted sum of its experts, and the partial sum travels back.
//
// Every rank holds one exchange buffer of the same layout (cudaMalloc; peers
// map it with CUDA IPC, or share it by plain pointer when several contexts
// live in one process on one device).  All transfers are plain 16-byte stores
// into the destination's buffer over NVLink; nothing is loaded from a peer.
// Per layer, on the stream of the call:
//
//   plan      1 CTA: calls += 1; for each (token t, rank d) whether t has an
//             expert on d (with a shared expert, every token also goes to its
//             own rank), and its slot pos[t][d] in d's receive segment of
//             this rank (tokens in order); n_out[d]
//   dispatch  one warp per (t, d) pair: the row x[t] and, per k, the expert's
//             id local to d (or -1) and its weight, into d's segment; the
//             last CTA to finish publishes n_out[d] and releases
//             data_flag[rank] = calls on every d
//   receive   one CTA per source s: wait until data_flag[s] >= calls, then
//             mark the unused rows of segment s empty (ids -1, weights 0)
//   compute   the grouped expert MLP of the local table on all segments
//             (kq_moe_prefill), whose weighted combine over the K slots
//             writes each received row's partial sum straight into its
//             owner's ret[t][rank] (row destinations built by receive; empty
//             rows skipped); below 16 rows kq_moe_decode into part[s][row]
//   return    grouped path: one thread releases ret_flag[rank] = calls on
//             every s; decode path: one warp per received row copies
//             part[s][row] into s's ret[t][rank], the last CTA releases
//   combine   every CTA waits until ret_flag[d] >= calls for all d, then
//             out[t] = residual[t] + sum_{d: pos[t][d] >= 0} ret[t][d] + shared[t]
//
// Flags only grow: a sender writes its own call count, a receiver waits for
// its own call count, and every rank makes the same calls in the same order,
// so no flag is ever reset and the sequence can be captured in a CUDA graph.
// A single buffer set is reused by every layer: a rank dispatches layer l+1
// only after its combine of layer l saw every peer's return of layer l, and a
// peer returns only after its compute has read the rows of layer l.
//
// Waits are bounded by wall time (wait_ns, %globaltimer); a wait that gives up
// latches KQ_DEV_WAIT_TIMEOUT and records (site, source, value seen, CTA) in
// the control words, and the kernel carries on with that source's rows
// treated as empty, so no launch outlives the bound.
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

#include <cstdio>
#include <cstring>
#include <type_traits>

#include "kq_common.cuh"
#include "kq_internal.h"

namespace kq {

constexpr int EP_MAXR = KQ_EP_MAX_RANKS;
constexpr int EP_THREADS = 256;
constexpr int EP_PLAN_THREADS = 1024;

// control words (u32 offsets inside the first 4 KB of the buffer)
enum : int {
    EPC_CALLS = 0,
    EPC_STATUS = 1,
    EPC_SITE = 4,        // site, source, value seen, CTA
    EPC_DONE_DISP = 16,  // CTA arrivals of the dispatch launch
    EPC_DONE_RET = 17,   // CTA arrivals of the return launch
    EPC_DATA_FLAG = 32,  // [EP_MAXR] written by source s
    EPC_RET_FLAG = 48,   // [EP_MAXR] written by destination d
    EPC_N_IN = 64,       // [EP_MAXR] rows from source s (written by s)
    EPC_N_OUT = 80,      // [EP_MAXR] rows to destination d (local)
    EPC_N_USE = 96,      // [EP_MAXR] rows of segment s taken as valid (local)
};
enum : int { EP_SITE_RECEIVE = 1, EP_SITE_COMBINE = 2 };

struct EpLayout {
    size_t ctl, pos, recv_tok, recv_idx, recv_w, recv_x, part, ret, rowptr, total;
};

static EpLayout ep_layout(int world, int T, int H, int K) {
    auto al = [](size_t v) { return (v + 255) / 256 * 256; };
    EpLayout L{};
    size_t o = 0;
    L.ctl = o;
    o += 4096;
    L.pos = o;
    o = al(o + (size_t)T * EP_MAXR * 4);
    L.recv_tok = o;
    o = al(o + (size_t)world * T * 4);
    L.recv_idx = o;
    o = al(o + (size_t)world * T * K * 4);
    L.recv_w = o;
    o = al(o + (size_t)world * T * K * 4);
    L.recv_x = o;
    o = al(o + (size_t)world * T * H * 2);
    L.part = o;
    o = al(o + (size_t)world * T * H * 2);
    L.ret = o;
    o = al(o + (size_t)T * world * H * 2);
    L.rowptr = o;  // local: destination of each received row's partial sum
    o = al(o + (size_t)world * T * 8);
    L.total = o;
    return L;
}

// Everything a kernel needs, passed by value (peer bases included).
struct EpParams {
    uint8_t* peer[EP_MAXR];  // every rank's buffer in this address space (peer[rank] = own)
    uint8_t* self;
    EpLayout L;
    int rank, world, T_max, H, K;
    uint64_t wait_ns;
};

__device__ __forceinline__ uint32_t* ctl(uint8_t* base) { return reinterpret_cast<uint32_t*>(base); }

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint32_t ld_relaxed_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Wait until *flag >= target, bounded by wait_ns of wall time.  Relaxed polls
// with a growing pause; one acquire load on success.
__device__ bool ep_wait_flag(const uint32_t* flag, uint32_t target, uint64_t wait_ns, uint32_t* c, int site,
                             int src) {
    if (ld_acquire_sys(flag) >= target) return true;
    // after a wait has given up the ranks are out of step until the status is
    // cleared: later waits give up at once instead of each taking wait_ns
    if (*reinterpret_cast<volatile uint32_t*>(c + EPC_STATUS) & KQ_DEV_WAIT_TIMEOUT) return false;
    const uint64_t t0 = global_ns();
    unsigned pause = 32;
    for (;;) {
        __nanosleep(pause);
        if (ld_relaxed_sys(flag) >= target) {
            (void)ld_acquire_sys(flag);
            return true;
        }
        if (pause < 2048) pause *= 2;
        if (global_ns() - t0 > wait_ns) {
            atomicOr(c + EPC_STATUS, KQ_DEV_WAIT_TIMEOUT);
            if (atomicCAS(c + EPC_SITE, 0u, (uint32_t)site) == 0u) {
                c[EPC_SITE + 1] = (uint32_t)src;
                c[EPC_SITE + 2] = ld_relaxed_sys(flag);
                c[EPC_SITE + 3] = blockIdx.x;
            }
            return false;
        }
    }
}

// Copy one row of H 16-bit values (H % 8 == 0), one warp, 16-byte accesses,
// eight loads in flight per lane (a 6 KB row in two rounds).
__device__ __forceinline__ void warp_copy_row(const uint4* __restrict__ src, uint4* dst, int n16, int lane) {
    constexpr int U = 8;
    for (int c = lane; c < n16; c += 32 * U) {
        uint4 v[U];
#pragma unroll
        for (int u = 0; u < U; ++u) v[u] = c + 32 * u < n16 ? src[c + 32 * u] : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int u = 0; u < U; ++u)
            if (c + 32 * u < n16) dst[c + 32 * u] = v[u];
    }
}

// ---- plan ----------------------------------------------------------------------
// Token t goes to rank d iff some valid slot k has owner[idx[t][k]] == d; its
// slot in d's segment is the number of earlier tokens that go to d.  Ids
// outside [0, E) other than -1 latch KQ_DEV_BAD_EXPERT and are dropped; -1 is
// an empty slot.
__global__ void __launch_bounds__(EP_PLAN_THREADS, 1)
    ep_plan_kernel(EpParams p, const int32_t* __restrict__ idx, int T, int k_route, bool self_slot,
                   const int32_t* __restrict__ owner, int E) {
    __shared__ int wsum[EP_MAXR][32];
    __shared__ int run[EP_MAXR];
    uint32_t* c = ctl(p.self);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) c[EPC_CALLS] += 1u;  // read by the later launches of this call only
    if (tid < EP_MAXR) run[tid] = 0;
    __syncthreads();
    int32_t* pos = reinterpret_cast<int32_t*>(p.self + p.L.pos);
    // tokens in rounds of EP_PLAN_THREADS, one token per thread, order kept by scans
    for (int t0 = 0; t0 < T; t0 += EP_PLAN_THREADS) {
        const int t = t0 + tid;
        uint32_t mask = 0;
        if (t < T) {
            if (self_slot) mask = 1u << p.rank;
            // ids of up to 8 slots at a time, then their owners: two memory
            // round trips per 8 slots instead of two per slot
            for (int k0 = 0; k0 < k_route; k0 += 8) {
                int e[8], d[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) e[u] = k0 + u < k_route ? idx[(size_t)t * k_route + k0 + u] : -1;
#pragma unroll
                for (int u = 0; u < 8; ++u) d[u] = (unsigned)e[u] < (unsigned)E ? owner[e[u]] : -1;
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    if ((unsigned)e[u] < (unsigned)E) {
                        if ((unsigned)d[u] < (unsigned)p.world) mask |= 1u << d[u];
                        else atomicOr(c + EPC_STATUS, KQ_DEV_BAD_INDEX);
                    } else if (e[u] != -1) {
                        atomicOr(c + EPC_STATUS, KQ_DEV_BAD_EXPERT);
                    }
                }
            }
        }
        int incl[EP_MAXR];
#pragma unroll
        for (int d = 0; d < EP_MAXR; ++d) {
            int v = (mask >> d) & 1u;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int n = __shfl_up_sync(0xffffffffu, v, o);
                if (lane >= o) v += n;
            }
            incl[d] = v;
            if (lane == 31) wsum[d][warp] = v;
        }
        __syncthreads();
        if (warp < p.world) {  // warp d scans the warp totals of rank d
            int v = wsum[warp][lane];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int n = __shfl_up_sync(0xffffffffu, v, o);
                if (lane >= o) v += n;
            }
            wsum[warp][lane] = v;
        }
        __syncthreads();
        if (t < T) {
#pragma unroll
            for (int d = 0; d < EP_MAXR; ++d) {
                int slot = -1;
                if (d < p.world && ((mask >> d) & 1u))
                    slot = run[d] + (warp ? wsum[d][warp - 1] : 0) + incl[d] - 1;
                pos[(size_t)t * EP_MAXR + d] = slot;
            }
        }
        __syncthreads();
        if (tid < p.world) run[tid] += wsum[tid][31];
        __syncthreads();
    }
    if (tid < p.world) c[EPC_N_OUT + tid] = (uint32_t)run[tid];
}

// ---- dispatch ------------------------------------------------------------------
__global__ void __launch_bounds__(EP_THREADS)
    ep_dispatch_kernel(EpParams p, const void* __restrict__ x, const int32_t* __restrict__ idx,
                       const float* __restrict__ w, int T, int k_route, const int32_t* __restrict__ owner,
                       const int32_t* __restrict__ local, int E, int shared_id, const float* __restrict__ shared_w) {
    uint32_t* c = ctl(p.self);
    const int lane = threadIdx.x & 31;
    const int gw = (blockIdx.x * EP_THREADS + threadIdx.x) >> 5, nw = gridDim.x * (EP_THREADS / 32);
    const int32_t* pos = reinterpret_cast<const int32_t*>(p.self + p.L.pos);
    const int n16 = p.H / 8;
    for (int pr = gw; pr < T * p.world; pr += nw) {
        const int t = pr / p.world, d = pr - t * p.world;
        const int slot = pos[(size_t)t * EP_MAXR + d];
        if (slot < 0) continue;
        uint8_t* dst = p.peer[d];
        const size_t row = (size_t)p.rank * p.T_max + slot;  // this rank's segment on d
        if (lane < k_route) {
            const int e = idx[(size_t)t * k_route + lane];
            const bool mine = (unsigned)e < (unsigned)E && owner[e] == d;
            reinterpret_cast<int32_t*>(dst + p.L.recv_idx)[row * p.K + lane] = mine ? local[e] : -1;
            reinterpret_cast<float*>(dst + p.L.recv_w)[row * p.K + lane] = mine ? w[(size_t)t * k_route + lane] : 0.f;
        } else if (lane < p.K) {  // the shared expert's slot: only in the owner's own segment
            const bool mine = shared_id >= 0 && d == p.rank;
            reinterpret_cast<int32_t*>(dst + p.L.recv_idx)[row * p.K + lane] = mine ? shared_id : -1;
            reinterpret_cast<float*>(dst + p.L.recv_w)[row * p.K + lane] = mine ? shared_w[t] : 0.f;
        }
        if (lane == 0) reinterpret_cast<int32_t*>(dst + p.L.recv_tok)[row] = t;
        warp_copy_row(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(x) + (size_t)t * p.H),
                      reinterpret_cast<uint4*>(dst + p.L.recv_x + row * p.H * 2), n16, lane);
    }
    __syncthreads();  // the CTA's rows are written; one fence covers them (release is cumulative)
    if (threadIdx.x == 0) {
        __threadfence_system();
        const uint32_t prev = atomicAdd(c + EPC_DONE_DISP, 1u);
        if (prev == gridDim.x - 1) {  // the last CTA: every row of this call has been written
            __threadfence_system();
            c[EPC_DONE_DISP] = 0u;
            const uint32_t calls = c[EPC_CALLS];
            for (int d = 0; d < p.world; ++d) ctl(p.peer[d])[EPC_N_IN + p.rank] = c[EPC_N_OUT + d];
            __threadfence_system();
            for (int d = 0; d < p.world; ++d) st_release_sys(ctl(p.peer[d]) + EPC_DATA_FLAG + p.rank, calls);
        }
    }
}

// ---- receive -------------------------------------------------------------------
__global__ void __launch_bounds__(EP_THREADS) ep_receive_kernel(EpParams p) {
    uint32_t* c = ctl(p.self);
    const int s = blockIdx.x;
    __shared__ int n_s;
    if (threadIdx.x == 0) {
        const uint32_t calls = c[EPC_CALLS];
        int n = 0;
        if (ep_wait_flag(c + EPC_DATA_FLAG + s, calls, p.wait_ns, c, EP_SITE_RECEIVE, s)) {
            n = (int)ld_acquire_sys(c + EPC_N_IN + s);
            if (n < 0 || n > p.T_max) {
                atomicOr(c + EPC_STATUS, KQ_DEV_BAD_INDEX);
                n = 0;
            }
        }
        c[EPC_N_USE + s] = (uint32_t)n;
        n_s = n;
    }
    __syncthreads();
    const int n = n_s;
    int32_t* ids = reinterpret_cast<int32_t*>(p.self + p.L.recv_idx) + (size_t)s * p.T_max * p.K;
    float* ws = reinterpret_cast<float*>(p.self + p.L.recv_w) + (size_t)s * p.T_max * p.K;
    for (int i = n * p.K + threadIdx.x; i < p.T_max * p.K; i += EP_THREADS) {
        ids[i] = -1;
        ws[i] = 0.f;
    }
    // where each row's partial sum goes: the owner's ret[token][rank] (null: skip)
    const int32_t* tok = reinterpret_cast<const int32_t*>(p.self + p.L.recv_tok) + (size_t)s * p.T_max;
    uint8_t** rp = reinterpret_cast<uint8_t**>(p.self + p.L.rowptr) + (size_t)s * p.T_max;
    for (int j = threadIdx.x; j < p.T_max; j += EP_THREADS) {
        uint8_t* d = nullptr;
        if (j < n) {
            const int t = tok[j];
            if ((unsigned)t < (unsigned)p.T_max)
                d = p.peer[s] + p.L.ret + ((size_t)t * p.world + p.rank) * p.H * 2;
            else
                atomicOr(c + EPC_STATUS, KQ_DEV_BAD_INDEX);
        }
        rp[j] = d;
    }
}

// The grouped compute wrote every partial row into its owner's buffer (and
// fenced): release the return flags.
__global__ void ep_signal_kernel(EpParams p) {
    uint32_t* c = ctl(p.self);
    if (threadIdx.x == 0) {
        __threadfence_system();
        const uint32_t calls = c[EPC_CALLS];
        for (int s = 0; s < p.world; ++s) st_release_sys(ctl(p.peer[s]) + EPC_RET_FLAG + p.rank, calls);
    }
}

// ---- return --------------------------------------------------------------------
__global__ void __launch_bounds__(EP_THREADS) ep_return_kernel(EpParams p) {
    uint32_t* c = ctl(p.self);
    const int lane = threadIdx.x & 31;
    const int gw = (blockIdx.x * EP_THREADS + threadIdx.x) >> 5, nw = gridDim.x * (EP_THREADS / 32);
    const int n16 = p.H / 8;
    const int32_t* tok = reinterpret_cast<const int32_t*>(p.self + p.L.recv_tok);
    for (int r = gw; r < p.world * p.T_max; r += nw) {
        const int s = r / p.T_max, j = r - s * p.T_max;
        if (j >= (int)c[EPC_N_USE + s]) continue;
        const int t = tok[r];
        if ((unsigned)t >= (unsigned)p.T_max) {
            if (lane == 0) atomicOr(c + EPC_STATUS, KQ_DEV_BAD_INDEX);
            continue;
        }
        uint8_t* dst = p.peer[s] + p.L.ret + ((size_t)t * p.world + p.rank) * p.H * 2;
        warp_copy_row(reinterpret_cast<const uint4*>(p.self + p.L.part + (size_t)r * p.H * 2),
                      reinterpret_cast<uint4*>(dst), n16, lane);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        const uint32_t prev = atomicAdd(c + EPC_DONE_RET, 1u);
        if (prev == gridDim.x - 1) {
            __threadfence_system();
            c[EPC_DONE_RET] = 0u;
            const uint32_t calls = c[EPC_CALLS];
            for (int s = 0; s < p.world; ++s) st_release_sys(ctl(p.peer[s]) + EPC_RET_FLAG + p.rank, calls);
        }
    }
}

// ---- combine -------------------------------------------------------------------
template <typename TX>
__device__ __forceinline__ void add8(float (&acc)[8], const TX* src) {
    const uint4 v = __ldcg(reinterpret_cast<const uint4*>(src));  // written by a peer: bypass L1
    const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float2 f;
        if constexpr (std::is_same<TX, __half>::value)
            f = __half22float2(*reinterpret_cast<const __half2*>(&u[i]));
        else
            f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u[i]));
        acc[2 * i] += f.x;
        acc[2 * i + 1] += f.y;
    }
}

// out[t] = residual[t] + sum_d ret[t][d] + gate[t] * shared[t]; one thread per 8
// columns, grid (ceil(H/8/EP_THREADS), T).
template <typename TX>
__global__ void __launch_bounds__(EP_THREADS)
    ep_combine_kernel(EpParams p, int T, const void* __restrict__ residual, int res_dtype,
                      const void* __restrict__ shared, int shared_dtype, const float* __restrict__ gate, void* out,
                      int out_dtype) {
    uint32_t* c = ctl(p.self);
    __shared__ uint32_t ok_mask;
    if (threadIdx.x == 0) {
        const uint32_t calls = c[EPC_CALLS];
        uint32_t ok = 0;
        for (int d = 0; d < p.world; ++d)
            if (ep_wait_flag(c + EPC_RET_FLAG + d, calls, p.wait_ns, c, EP_SITE_COMBINE, d)) ok |= 1u << d;
        ok_mask = ok;
    }
    __syncthreads();
    const int t = blockIdx.y, h = (blockIdx.x * EP_THREADS + threadIdx.x) * 8;
    if (t >= T || h >= p.H) return;
    const uint32_t ok = ok_mask;
    const int32_t* pos = reinterpret_cast<const int32_t*>(p.self + p.L.pos) + (size_t)t * EP_MAXR;
    const TX* ret = reinterpret_cast<const TX*>(p.self + p.L.ret) + (size_t)t * p.world * p.H + h;
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = residual ? load_as_float(residual, res_dtype, (size_t)t * p.H + h + j) : 0.f;
    for (int d = 0; d < p.world; ++d)
        if (pos[d] >= 0 && ((ok >> d) & 1u)) add8<TX>(acc, ret + (size_t)d * p.H);
    if (shared) {
        const float g = gate ? gate[t] : 1.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] += g * load_as_float(shared, shared_dtype, (size_t)t * p.H + h + j);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) store_from_float(out, out_dtype, (size_t)t * p.H + h + j, acc[j]);
}

}  // namespace kq

using namespace kq;

struct kq_ep {
    int rank = 0, world = 1, T_max = 0, H = 0, K = 0, x_dtype = KQ_DT_F16, dev = 0;
    EpLayout L{};
    uint8_t* base = nullptr;
    uint8_t* peer[EP_MAXR] = {};
    bool opened[EP_MAXR] = {};
    uint64_t wait_ns = 2000000000ull;
    int nsm = 148;
    bool fused_return = false;  // the last compute wrote the partial rows to their owners
};

static EpParams ep_params(const kq_ep* ep) {
    EpParams p{};
    for (int i = 0; i < EP_MAXR; ++i) p.peer[i] = ep->peer[i];
    p.self = ep->base;
    p.L = ep->L;
    p.rank = ep->rank;
    p.world = ep->world;
    p.T_max = ep->T_max;
    p.H = ep->H;
    p.K = ep->K;
    p.wait_ns = ep->wait_ns;
    return p;
}

static bool ep_connected(const kq_ep* ep) {
    for (int i = 0; i < ep->world; ++i)
        if (!ep->peer[i]) return false;
    return true;
}

static int ep_fail(const char* what, cudaError_t e) {
    fprintf(stderr, "[kandiga] ERROR: kq_ep %s: %s\n", what, cudaGetErrorString(e));
    return KQ_ERR_CUDA;
}

extern "C" size_t kq_ep_buffer_bytes(int world, int max_tokens, int hidden, int top_k) {
    if (world < 1 || world > EP_MAXR || max_tokens < 1 || hidden < 8 || top_k < 1) return 0;
    return ep_layout(world, max_tokens, hidden, top_k).total;
}

extern "C" int kq_ep_create(int rank, int world, int max_tokens, int hidden, int top_k, int x_dtype, kq_ep** out) {
    if (!out) return KQ_ERR_ARG;
    *out = nullptr;
    if (world < 1 || world > EP_MAXR || rank < 0 || rank >= world) return KQ_ERR_ARG;
    if (max_tokens < 1 || hidden < 8 || hidden % 8 || top_k < 1 || top_k > 32) return KQ_ERR_ARG;
    if (x_dtype != KQ_DT_F16 && x_dtype != KQ_DT_BF16) return KQ_ERR_ARG;
    kq_ep* ep = new (std::nothrow) kq_ep();
    if (!ep) return KQ_ERR_ALLOC;
    ep->rank = rank;
    ep->world = world;
    ep->T_max = max_tokens;
    ep->H = hidden;
    ep->K = top_k;
    ep->x_dtype = x_dtype;
    ep->L = ep_layout(world, max_tokens, hidden, top_k);
    cudaGetDevice(&ep->dev);
    cudaDeviceGetAttribute(&ep->nsm, cudaDevAttrMultiProcessorCount, ep->dev);
    if (cudaMalloc(&ep->base, ep->L.total) != cudaSuccess) {
        delete ep;
        return KQ_ERR_ALLOC;
    }
    // zero control words, slots and return rows (unused rows are never read, but
    // a fresh buffer should not hold another allocation's bytes)
    if (cudaMemset(ep->base, 0, ep->L.total) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
        cudaFree(ep->base);
        delete ep;
        return KQ_ERR_CUDA;
    }
    ep->peer[rank] = ep->base;
    *out = ep;
    return KQ_OK;
}

extern "C" int kq_ep_ipc_handle(const kq_ep* ep, void* handle_out) {
    if (!ep || !handle_out) return KQ_ERR_ARG;
    static_assert(sizeof(cudaIpcMemHandle_t) == KQ_EP_HANDLE_BYTES, "IPC handle size");
    cudaIpcMemHandle_t h;
    if (cudaError_t e = cudaIpcGetMemHandle(&h, ep->base)) return ep_fail("cudaIpcGetMemHandle", e);
    memcpy(handle_out, &h, sizeof(h));
    return KQ_OK;
}

extern "C" int kq_ep_connect(kq_ep* ep, const void* handles) {
    if (!ep || !handles) return KQ_ERR_ARG;
    for (int r = 0; r < ep->world; ++r) {
        if (r == ep->rank || ep->peer[r]) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const uint8_t*>(handles) + (size_t)r * KQ_EP_HANDLE_BYTES, sizeof(h));
        void* p = nullptr;
        if (cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess))
            return ep_fail("cudaIpcOpenMemHandle", e);
        ep->peer[r] = static_cast<uint8_t*>(p);
        ep->opened[r] = true;
    }
    return KQ_OK;
}

extern "C" int kq_ep_connect_local(kq_ep* const* eps, int n) {
    if (!eps || n < 1) return KQ_ERR_ARG;
    for (int i = 0; i < n; ++i) {
        if (!eps[i] || eps[i]->world != n || eps[i]->rank != i || eps[i]->dev != eps[0]->dev ||
            eps[i]->T_max != eps[0]->T_max || eps[i]->H != eps[0]->H || eps[i]->K != eps[0]->K)
            return KQ_ERR_ARG;
    }
    for (int i = 0; i < n; ++i)
        for (int r = 0; r < n; ++r) eps[i]->peer[r] = eps[r]->base;
    return KQ_OK;
}

extern "C" void kq_ep_destroy(kq_ep* ep) {
    if (!ep) return;
    cudaDeviceSynchronize();
    for (int r = 0; r < EP_MAXR; ++r)
        if (ep->opened[r]) cudaIpcCloseMemHandle(ep->peer[r]);
    cudaFree(ep->base);
    delete ep;
}

extern "C" int kq_ep_set_wait_ns(kq_ep* ep, uint64_t ns) {
    if (!ep || ns == 0) return KQ_ERR_ARG;
    ep->wait_ns = ns;
    return KQ_OK;
}

extern "C" int kq_ep_dispatch(kq_ep* ep, const void* x, const int32_t* idx, const float* weights, int T,
                              int k_route, const int32_t* owner, const int32_t* local, int num_experts,
                              int shared_id, const float* shared_w, void* stream) {
    if (!ep || !ep_connected(ep)) return KQ_ERR_ARG;
    if (T < 0 || T > ep->T_max || num_experts < 1 || !owner || !local) return KQ_ERR_ARG;
    const bool has_shared = shared_id >= 0;  // the shared expert's slot (its gate per token in shared_w)
    if (k_route < 1 || k_route + (has_shared ? 1 : 0) != ep->K) return KQ_ERR_ARG;
    if (has_shared && T > 0 && !shared_w) return KQ_ERR_ARG;
    if (T > 0 && (!x || !idx || !weights)) return KQ_ERR_ARG;
    if (reinterpret_cast<uintptr_t>(x) & 15) return KQ_ERR_ARG;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const EpParams p = ep_params(ep);
    ep_plan_kernel<<<1, EP_PLAN_THREADS, 0, s>>>(p, idx, T, k_route, has_shared, owner, num_experts);
    if (cudaError_t e = cudaGetLastError()) return ep_fail("plan", e);
    const int pairs = T * ep->world, wpb = EP_THREADS / 32;
    const int grid = std::max(1, std::min((pairs + wpb - 1) / wpb, ep->nsm * 8));
    ep_dispatch_kernel<<<grid, EP_THREADS, 0, s>>>(p, x, idx, weights, T, k_route, owner, local, num_experts,
                                                   shared_id, shared_w);
    if (cudaError_t e = cudaGetLastError()) return ep_fail("dispatch", e);
    return KQ_OK;
}

extern "C" int kq_ep_receive(kq_ep* ep, void** recv_x, int32_t** recv_idx, float** recv_w, int* rows, void* stream) {
    if (!ep || !ep_connected(ep)) return KQ_ERR_ARG;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    ep_receive_kernel<<<ep->world, EP_THREADS, 0, s>>>(ep_params(ep));
    if (cudaError_t e = cudaGetLastError()) return ep_fail("receive", e);
    if (recv_x) *recv_x = ep->base + ep->L.recv_x;
    if (recv_idx) *recv_idx = reinterpret_cast<int32_t*>(ep->base + ep->L.recv_idx);
    if (recv_w) *recv_w = reinterpret_cast<float*>(ep->base + ep->L.recv_w);
    if (rows) *rows = ep->world * ep->T_max;
    return KQ_OK;
}

extern "C" void* kq_ep_partials(kq_ep* ep) { return ep ? ep->base + ep->L.part : nullptr; }

extern "C" int kq_ep_return(kq_ep* ep, void* stream) {
    if (!ep || !ep_connected(ep)) return KQ_ERR_ARG;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (ep->fused_return) {
        ep_signal_kernel<<<1, 32, 0, s>>>(ep_params(ep));
        if (cudaError_t e = cudaGetLastError()) return ep_fail("signal", e);
        return KQ_OK;
    }
    const int rows = ep->world * ep->T_max, wpb = EP_THREADS / 32;
    const int grid = std::max(1, std::min((rows + wpb - 1) / wpb, ep->nsm * 8));
    ep_return_kernel<<<grid, EP_THREADS, 0, s>>>(ep_params(ep));
    if (cudaError_t e = cudaGetLastError()) return ep_fail("return", e);
    return KQ_OK;
}

extern "C" int kq_ep_combine(kq_ep* ep, int T, const void* residual, int res_dtype, const void* shared,
                             int shared_dtype, const float* gate, void* out, int out_dtype, void* stream) {
    if (!ep || !ep_connected(ep)) return KQ_ERR_ARG;
    if (T < 0 || T > ep->T_max || (T > 0 && !out)) return KQ_ERR_ARG;
    auto okdt = [](int d) { return d == KQ_DT_F16 || d == KQ_DT_BF16 || d == KQ_DT_F32; };
    if (!okdt(out_dtype) || (residual && !okdt(res_dtype)) || (shared && !okdt(shared_dtype))) return KQ_ERR_ARG;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    // every CTA waits for the returns, so launch at least one even for T == 0
    const dim3 grid((ep->H / 8 + EP_THREADS - 1) / EP_THREADS, std::max(T, 1));
    if (ep->x_dtype == KQ_DT_F16)
        ep_combine_kernel<__half><<<grid, EP_THREADS, 0, s>>>(ep_params(ep), T, residual, res_dtype, shared,
                                                              shared_dtype, gate, out, out_dtype);
    else
        ep_combine_kernel<__nv_bfloat16><<<grid, EP_THREADS, 0, s>>>(ep_params(ep), T, residual, res_dtype, shared,
                                                                     shared_dtype, gate, out, out_dtype);
    if (cudaError_t e = cudaGetLastError()) return ep_fail("combine", e);
    return KQ_OK;
}

static bool ep_grouped(const kq_ep* ep, const kq_table* t) {
    return ep->world * ep->T_max >= 16 && t->d.hidden % 512 == 0 && t->d.inter % 512 == 0;
}

extern "C" size_t kq_ep_moe_workspace_size(const kq_ep* ep, const kq_table* t) {
    if (!ep || !t) return 0;
    const int rows = ep->world * ep->T_max;
    return ep_grouped(ep, t) ? kq_moe_prefill_workspace_size(t, rows, ep->K) : kq_moe_workspace_size(t, rows, ep->K);
}

extern "C" int kq_ep_compute(kq_ep* ep, const kq_table* t, int layer, void* workspace, size_t workspace_bytes,
                             void* stream) {
    if (!ep || !t || t->d.hidden != ep->H) return KQ_ERR_ARG;
    const int rows = ep->world * ep->T_max;
    void* x = ep->base + ep->L.recv_x;
    int32_t* idx = reinterpret_cast<int32_t*>(ep->base + ep->L.recv_idx);
    float* w = reinterpret_cast<float*>(ep->base + ep->L.recv_w);
    void* part = ep->base + ep->L.part;
    ep->fused_return = ep_grouped(ep, t);
    if (ep->fused_return)
        return moe_prefill_ex(t, layer, x, ep->x_dtype, rows, nullptr, idx, w, ep->K, nullptr, nullptr, ep->x_dtype,
                              nullptr, reinterpret_cast<void* const*>(ep->base + ep->L.rowptr), workspace,
                              workspace_bytes, stream);
    return kq_moe_decode(t, layer, x, ep->x_dtype, rows, nullptr, idx, w, ep->K, nullptr, part, ep->x_dtype, nullptr,
                         workspace, workspace_bytes, stream);
}

extern "C" int kq_ep_moe(kq_ep* ep, const kq_table* t, int layer, const void* x, int T, const int32_t* idx,
                         const float* weights, int k_route, int num_experts, const int32_t* owner,
                         const int32_t* local, int shared_id, const float* shared_w, const void* residual,
                         int res_dtype, const void* shared, int shared_dtype, const float* gate, void* out,
                         int out_dtype, void* workspace, size_t workspace_bytes, void* stream) {
    if (!ep || !t) return KQ_ERR_ARG;
    if (int rc = kq_ep_dispatch(ep, x, idx, weights, T, k_route, owner, local, num_experts, shared_id, shared_w,
                                stream))
        return rc;
    if (int rc = kq_ep_receive(ep, nullptr, nullptr, nullptr, nullptr, stream)) return rc;
    if (int rc = kq_ep_compute(ep, t, layer, workspace, workspace_bytes, stream)) return rc;
    if (int rc = kq_ep_return(ep, stream)) return rc;
    return kq_ep_combine(ep, T, residual, res_dtype, shared, shared_dtype, gate, out, out_dtype, stream);
}

extern "C" int kq_ep_status(kq_ep* ep, uint32_t* status_out, uint32_t* site_out, void* stream) {
    if (!ep || !status_out) return KQ_ERR_ARG;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    uint32_t w[8];
    if (cudaError_t e = cudaMemcpyAsync(w, ep->base, sizeof(w), cudaMemcpyDeviceToHost, s)) return ep_fail("status", e);
    if (cudaError_t e = cudaStreamSynchronize(s)) return ep_fail("status", e);
    *status_out = w[EPC_STATUS];
    if (site_out) memcpy(site_out, w + EPC_SITE, 4 * sizeof(uint32_t));
    return KQ_OK;
}

extern "C" int kq_ep_clear_status(kq_ep* ep, void* stream) {
    if (!ep) return KQ_ERR_ARG;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (cudaError_t e = cudaMemsetAsync(ep->base + EPC_STATUS * 4, 0, 7 * 4, s)) return ep_fail("clear", e);
    return KQ_OK;
}

extern "C" int kq_ep_calls(kq_ep* ep, uint32_t* calls_out) {
    if (!ep || !calls_out) return KQ_ERR_ARG;
    uint32_t v = 0;
    if (cudaError_t e = cudaMemcpy(&v, ep->base, sizeof(v), cudaMemcpyDeviceToHost)) return ep_fail("calls", e);
    *calls_out = v;
    return KQ_OK;
}
