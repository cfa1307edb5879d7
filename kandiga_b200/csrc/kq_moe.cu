// kq_moe.cu -- routed-expert decode path and dense quantized GEMV on sm_100a.
//
// Kernels
//   router_topk_kernel  softmax/top-K/renormalise, one warp per token
//                       (kandiga/metal/moe_block.metal:419-505).
//   qgemv_kernel        the tile engine of kq_qtile.cuh driven by a per-warp
//                       TMA bulk-copy ring.  Four epilogues:
//     MODE_GATEUP   gate+up rows of the routed experts -> act = silu(g)*u (fp32
//                   scratch)  (kandiga/metal/kandiga_cpu_expert.m:372-394)
//     MODE_DOWN     down rows -> unweighted per-expert outputs and/or the
//                   weighted combine (+ residual) done by the last of the K
//                   experts to finish a 16-row tile (no spin: an arrival
//                   counter, self-resetting)
//                   (kandiga/metal/kandiga_cpu_expert.m:396-398,
//                    kandiga/metal/moe_block.metal:556-584)
//     MODE_DENSE    y = W x with optional RMSNorm prologue
//     MODE_DENSE_PAIR  y = act(Wg x) * (Wu x)
//
// Each warp owns a ring of NBUF tile slots in shared memory.  Lane 0 issues a
// cp.async.bulk per 16x512 tile (3.5 KB at 3-bit) as soon as a slot frees up,
// so every warp keeps NBUF tiles of HBM traffic in flight; the whole warp
// waits on the slot's mbarrier (bounded), pulls its lane's words into
// registers and runs the 32-MMA tile.  The decode chain router -> gate/up ->
// down uses programmatic dependent launch: the down kernel issues its weight
// copies before waiting for the gate/up kernel's activations.
#include <cstdio>

#include "kq_internal.h"

namespace kq {

enum { MODE_GATEUP = 0, MODE_DOWN = 1, MODE_DENSE = 2, MODE_DENSE_PAIR = 3 };

struct GemvParams {
    const uint8_t* base;  // layer base (MoE) or matrix base (dense)
    size_t expert_bytes;  // MoE: bytes per expert (0 dense)
    size_t mat_off;       // matrix offset inside an expert
    int nrt, nst;         // row-tiles per vector, column tiles
    int E;                // experts (1 for dense)
    int ncols;            // real input length
    int T, K;             // tokens, experts per token (dense: 1)
    const void* x;
    int x_dtype;
    const void* norm_w;
    float eps;
    const int32_t* idx;   // [T*K]
    const float* w;       // [T*K]
    float* act;           // [T*K][I]
    float* amax;          // [T*K][I/8] per gate/up tile max |act| (scales the down input)
    int nrt_up;           // gate/up row-tiles per vector (I/8)
    int I;
    float* y;             // [T*K][H] fp32 (combine input) or null
    uint32_t* cnt;        // [T][nrt of the down matrix]
    int cnt_per_token;    // counters per token (down row-tiles)
    void* out_per_k;      // [T*K][H] (out_dtype) or null
    void* out;            // [T][rows]
    int out_dtype;
    const void* residual;
    int act_kind;
    int H;                // output rows (down: hidden; dense: rows or rows/2 for pair)
    uint32_t* status;
    int prefetch_before_wait;
    int mode;
};

__host__ __device__ constexpr size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

template <int BITS, int NBUF>
__host__ __device__ constexpr size_t warp_smem(int nst) {
    return align_up((size_t)NBUF * TileT<BITS>::BYTES + (size_t)nst * TILE_COLS * 2 +
                        (size_t)nst * TILE_GROUPS * 8 + NBUF * 8,
                    128);
}

template <int BITS, int SB_DT, int NBUF, int WARPS>
__global__ void __launch_bounds__(WARPS * 32) qgemv_kernel(const GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int TB = TileT<BITS>::BYTES;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int npad = p.nst * TILE_COLS, ng = npad / GS;
    uint8_t* wb = smem + (size_t)warp * warp_smem<BITS, NBUF>(p.nst);
    uint8_t* tiles = wb;
    __half* xs = reinterpret_cast<__half*>(wb + NBUF * TB);
    float2* cx = reinterpret_cast<float2*>(wb + NBUF * TB + (size_t)npad * 2);
    uint64_t* bars = reinterpret_cast<uint64_t*>(wb + NBUF * TB + (size_t)npad * 2 + (size_t)ng * 8);
    const int mode = p.mode;
    const bool is_moe = (mode == MODE_GATEUP || mode == MODE_DOWN);

    if (lane == 0) {
#pragma unroll
        for (int b = 0; b < NBUF; ++b) mbar_init(&bars[b], 1);
        fence_mbar_init();
    }
    __syncwarp();
    if (!p.prefetch_before_wait) pdl_wait();

    const int units = p.T * p.K * p.nrt;
    const int wg = blockIdx.x * WARPS + warp, stride = gridDim.x * WARPS;
    const int nun = wg < units ? (units - 1 - wg) / stride + 1 : 0;
    const int ntiles = nun * p.nst;
    const uint64_t pol = policy_evict_first();

    auto issue = [&](int f) {
        const int u = wg + (f / p.nst) * stride, st = f % p.nst;
        const int tk = u / p.nrt, rt = u % p.nrt;
        int e = 0;
        if (is_moe) {
            e = __ldcg(p.idx + tk);
            if ((unsigned)e >= (unsigned)p.E) e = 0;  // flagged and zeroed in the epilogue
        }
        const uint8_t* src =
            p.base + (size_t)e * p.expert_bytes + p.mat_off + ((size_t)rt * p.nst + st) * TB;
        const int slot = f % NBUF;
        mbar_expect_tx(&bars[slot], TB);
        bulk_g2s(tiles + (size_t)slot * TB, src, TB, &bars[slot], pol);
    };
    if (lane == 0)
        for (int f = 0; f < NBUF && f < ntiles; ++f) issue(f);
    if (p.prefetch_before_wait) pdl_wait();
    if (mode == MODE_GATEUP && blockIdx.x == 0 && p.cnt) {
        // The down kernel's arrival counters for this call: zeroed here, before
        // the down kernel (which waits for this grid) can reach its combine.
        // Their offset in the workspace depends on T and K, so a previous call
        // with other shapes may have left other data there.
        const int ncnt = p.T * p.cnt_per_token;
        for (int i = threadIdx.x; i < ncnt; i += blockDim.x) p.cnt[i] = 0u;
    }
    pdl_launch_dependents();

    int staged = -1;
    float inv = 1.f, y0 = 0.f, y1 = 0.f;
    for (int f = 0; f < ntiles; ++f) {
        const int u = wg + (f / p.nst) * stride, st = f % p.nst;
        const int tk = u / p.nrt, rt = u % p.nrt;
        if (st == 0) {
            const int vec = (mode == MODE_DOWN) ? tk : tk / p.K;
            if (vec != staged) {
                float scale = 1.f;
                if (mode == MODE_DOWN) {
                    // max |act| of this (token, k) from the gate/up epilogue's per-tile maxima
                    const float* pm = p.amax + (size_t)vec * p.nrt_up;
                    float a = 0.f;
                    for (int i = lane; i < p.nrt_up; i += 32) a = fmaxf(a, __ldcg(pm + i));
                    scale = pow2_scale(warp_max(a));
                    stage_vector<BITS>(p.act, KQ_DT_F32, (size_t)vec * p.I, p.ncols, npad, nullptr, scale,
                                       true, xs, cx);
                } else {
                    const size_t off = (size_t)vec * p.ncols;
                    if (p.norm_w) {
                        float amax, ss;
                        vec_stats(p.x, p.x_dtype, off, p.ncols, p.norm_w, false, amax, ss);
                        const float rinv = rsqrtf(ss / (float)p.ncols + p.eps);
                        scale = pow2_scale(amax * rinv);
                        stage_vector<BITS>(p.x, p.x_dtype, off, p.ncols, npad, p.norm_w, rinv * scale, false,
                                           xs, cx);
                    } else {
                        if (p.x_dtype != KQ_DT_F16) {  // fp16 inputs are staged exactly, unscaled
                            float amax, ss;
                            vec_stats(p.x, p.x_dtype, off, p.ncols, nullptr, false, amax, ss);
                            scale = pow2_scale(amax);
                        }
                        stage_vector<BITS>(p.x, p.x_dtype, off, p.ncols, npad, nullptr, scale, false, xs, cx);
                    }
                }
                inv = 1.f / scale;
                staged = vec;
            }
            y0 = y1 = 0.f;
        }
        const int slot = f % NBUF;
        mbar_wait(&bars[slot], (uint32_t)((f / NBUF) & 1), p.status);
        TileRegs<BITS> R;
        tile_load<BITS>(tiles + (size_t)slot * TB, R);
        __syncwarp();
        if (lane == 0 && f + NBUF < ntiles) {
            fence_proxy_async_smem();
            issue(f + NBUF);
        }
        tile_compute<BITS, SB_DT>(R, st, xs, cx, y0, y1);
        if (st != p.nst - 1) continue;

        // ---- unit epilogue --------------------------------------------------------
        quad_reduce(y0, y1);
        const int r = lane >> 2;
        bool valid = true;
        if (is_moe) {
            const int e = __ldcg(p.idx + tk);
            valid = (unsigned)e < (unsigned)p.E;
            if (!valid && lane == 0) set_status(p.status, KQ_DEV_BAD_EXPERT);
        }
        const float g = valid ? y0 * inv : 0.f, h = valid ? y1 * inv : 0.f;
        if (mode == MODE_GATEUP || mode == MODE_DENSE_PAIR) {
            const float a = valid ? activate(g, h, p.act_kind) : 0.f;
            if ((lane & 3) == 0) {
                const int row = rt * 8 + r;
                if (mode == MODE_GATEUP)
                    p.act[(size_t)tk * p.I + row] = a;
                else
                    store_from_float(p.out, p.out_dtype, (size_t)tk * p.H + row, a);
            }
            if (mode == MODE_GATEUP) {
                const float m = warp_max(fabsf(a));
                if (lane == 0) p.amax[(size_t)tk * p.nrt + rt] = m;
            }
            continue;
        }
        if (mode == MODE_DENSE) {
            if ((lane & 3) == 0) {
                store_from_float(p.out, p.out_dtype, (size_t)tk * p.H + rt * 16 + r, g);
                store_from_float(p.out, p.out_dtype, (size_t)tk * p.H + rt * 16 + r + 8, h);
            }
            continue;
        }
        // MODE_DOWN
        if ((lane & 3) == 0) {
            const size_t o = (size_t)tk * p.H + rt * 16 + r;
            if (p.out_per_k) {
                store_from_float(p.out_per_k, p.out_dtype, o, g);
                store_from_float(p.out_per_k, p.out_dtype, o + 8, h);
            }
            if (p.out) {
                p.y[o] = g;
                p.y[o + 8] = h;
            }
        }
        if (!p.out) continue;
        __threadfence();
        __syncwarp();
        const int t = tk / p.K;
        uint32_t old = 0;
        if (lane == 0) old = atomicAdd(p.cnt + (size_t)t * p.nrt + rt, 1u);
        old = __shfl_sync(0xffffffffu, old, 0);
        if (old == (uint32_t)(p.K - 1)) {
            __threadfence();
            if (lane < 16) {
                const int row = rt * 16 + lane;
                float acc = 0.f;
                for (int k = 0; k < p.K; ++k)
                    acc += __ldcg(p.y + ((size_t)t * p.K + k) * p.H + row) * __ldcg(p.w + (size_t)t * p.K + k);
                if (p.residual) acc = load_as_float(p.residual, p.out_dtype, (size_t)t * p.H + row) + acc;
                store_from_float(p.out, p.out_dtype, (size_t)t * p.H + row, acc);
            }
            if (lane == 0) atomicExch(p.cnt + (size_t)t * p.nrt + rt, 0u);
        }
    }
}

// ---- router ------------------------------------------------------------------------
// One warp per token.  Selection compares logits (softmax is monotone) with
// strict '>' and lowest index on ties; weights = exp(l_k - max) / sum_sel.
__global__ void router_topk_kernel(const float* __restrict__ logits, int T, int E, int K,
                                   int32_t* __restrict__ idx, float* __restrict__ wout) {
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    pdl_wait();
    pdl_launch_dependents();
    if (t >= T) return;
    constexpr int MAXV = 32;  // E <= 1024
    float v[MAXV];
    const float* l = logits + (size_t)t * E;
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < MAXV; ++j) {
        const int i = lane + 32 * j;
        v[j] = i < E ? l[i] : -INFINITY;
        mx = fmaxf(mx, v[j]);
    }
    mx = warp_max(mx);
    uint32_t taken = 0;
    float esel = 0.f, esum = 0.f;
    for (int k = 0; k < K; ++k) {
        float bv = 0.f;
        int bi = -1;
#pragma unroll
        for (int j = 0; j < MAXV; ++j) {
            const int i = lane + 32 * j;
            if (i < E && !((taken >> j) & 1u) && (bi < 0 || v[j] > bv)) {
                bv = v[j];
                bi = i;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            const bool take = oi >= 0 && (bi < 0 || ov > bv || (ov == bv && oi < bi));
            if (take) {
                bv = ov;
                bi = oi;
            }
        }
        if (bi >= 0 && (bi & 31) == lane) taken |= 1u << (bi >> 5);
        const float ev = expf(bv - mx);
        esum += ev;
        if (lane == k) esel = ev;
        if (lane == 0) idx[(size_t)t * K + k] = bi;
    }
    if (lane < K) wout[(size_t)t * K + lane] = esel / esum;
}

// ---- launch helpers -----------------------------------------------------------------

template <int BITS, int SB_DT, int NBUF>
static cudaError_t launch_gemv(const GemvParams& p, cudaStream_t s, bool pdl, int max_blocks) {
    constexpr int WARPS = 4;
    const size_t smem = warp_smem<BITS, NBUF>(p.nst) * WARPS;
    auto kern = qgemv_kernel<BITS, SB_DT, NBUF, WARPS>;
    // raise the dynamic shared-memory limit once per instantiation (and per device)
    static int configured_bytes[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if ((size_t)configured_bytes[dev] < smem) {
        cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (err != cudaSuccess) return err;
        configured_bytes[dev] = (int)smem;
    }
    const int units = p.T * p.K * p.nrt;
    int blocks = (units + WARPS - 1) / WARPS;
    if (max_blocks > 0 && blocks > max_blocks) blocks = max_blocks;
    if (blocks < 1) blocks = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(blocks);
    cfg.blockDim = dim3(WARPS * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

static cudaError_t dispatch_gemv(int bits, int sb_dt, bool down, const GemvParams& p, cudaStream_t s,
                                 bool pdl) {
    const int maxb = 148 * 8;
    if (bits == 3) {
        if (down) return sb_dt == KQ_DT_F16 ? launch_gemv<3, KQ_DT_F16, 2>(p, s, pdl, maxb)
                                            : launch_gemv<3, KQ_DT_BF16, 2>(p, s, pdl, maxb);
        return sb_dt == KQ_DT_F16 ? launch_gemv<3, KQ_DT_F16, 4>(p, s, pdl, maxb)
                                  : launch_gemv<3, KQ_DT_BF16, 4>(p, s, pdl, maxb);
    }
    if (down) return sb_dt == KQ_DT_F16 ? launch_gemv<4, KQ_DT_F16, 2>(p, s, pdl, maxb)
                                        : launch_gemv<4, KQ_DT_BF16, 2>(p, s, pdl, maxb);
    return sb_dt == KQ_DT_F16 ? launch_gemv<4, KQ_DT_F16, 4>(p, s, pdl, maxb)
                              : launch_gemv<4, KQ_DT_BF16, 4>(p, s, pdl, maxb);
}

static cudaError_t launch_router(const float* logits, int T, int E, int K, int32_t* idx, float* w,
                                 cudaStream_t s, bool pdl) {
    const int warps = 4;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((T + warps - 1) / warps);
    cfg.blockDim = dim3(warps * 32);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, router_topk_kernel, logits, T, E, K, idx, w);
}

MoeWs moe_ws_layout(const kq_table* t, int T, int K) {
    MoeWs L{};
    size_t o = 0;
    L.status = o;
    o += 256;
    L.idx = o;
    o = align_up(o + (size_t)T * K * 4, 256);
    L.w = o;
    o = align_up(o + (size_t)T * K * 4, 256);
    L.act = o;
    o = align_up(o + (size_t)T * K * t->d.inter * 4, 256);
    L.y = o;
    o = align_up(o + (size_t)T * K * t->d.hidden * 4, 256);
    L.amax = o;
    o = align_up(o + (size_t)T * K * t->i8 * 4, 256);
    L.cnt = o;
    o = align_up(o + (size_t)T * t->h16 * 4, 256);
    L.total = o;
    return L;
}

static bool valid_dtype(int d) { return d == KQ_DT_F16 || d == KQ_DT_BF16 || d == KQ_DT_F32; }

}  // namespace kq

using namespace kq;

extern "C" size_t kq_moe_workspace_size(const kq_table* t, int max_tokens, int top_k) {
    if (!t || max_tokens < 0 || top_k <= 0) return 0;
    return moe_ws_layout(t, max_tokens, top_k).total;
}

extern "C" int kq_workspace_init(void* workspace, size_t bytes, void* stream) {
    if (!workspace) return KQ_ERR_ARG;
    return cudaMemsetAsync(workspace, 0, bytes, static_cast<cudaStream_t>(stream)) == cudaSuccess
               ? KQ_OK
               : KQ_ERR_CUDA;
}

extern "C" int kq_status_read(void* workspace, uint32_t* status, void* stream) {
    if (!workspace || !status) return KQ_ERR_ARG;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    if (cudaMemcpyAsync(status, workspace, 4, cudaMemcpyDeviceToHost, s) != cudaSuccess) return KQ_ERR_CUDA;
    if (cudaMemsetAsync(workspace, 0, 4, s) != cudaSuccess) return KQ_ERR_CUDA;
    return cudaStreamSynchronize(s) == cudaSuccess ? KQ_OK : KQ_ERR_CUDA;
}

extern "C" int kq_router_topk(const float* logits, int T, int E, int K, int32_t* idx, float* weights,
                              void* stream) {
    if (T < 0 || E <= 0 || E > 1024 || K <= 0 || K > E || K > 32) return KQ_ERR_ARG;
    if (T == 0) return KQ_OK;
    if (!logits || !idx || !weights) return KQ_ERR_ARG;
    return launch_router(logits, T, E, K, idx, weights, static_cast<cudaStream_t>(stream), false) ==
                   cudaSuccess
               ? KQ_OK
               : KQ_ERR_CUDA;
}

extern "C" int kq_moe_decode(const kq_table* t, int layer, const void* x, int x_dtype, int T,
                             const float* logits, int32_t* idx, float* weights, int K,
                             void* out_per_k, void* out, int out_dtype, const void* residual,
                             void* workspace, size_t workspace_bytes, void* stream) {
    if (!t) return KQ_ERR_ARG;
    if (layer < 0 || layer >= t->d.num_layers) return KQ_ERR_ARG;
    if (T < 0 || K <= 0 || K > 32 || K > t->d.num_experts) return KQ_ERR_ARG;
    if (T == 0) return KQ_OK;
    if (!x || !valid_dtype(x_dtype)) return KQ_ERR_ARG;
    if (!logits && !idx) return KQ_ERR_ARG;
    if (!valid_dtype(out_dtype)) return KQ_ERR_ARG;
    if (out && !weights && !logits) return KQ_ERR_ARG;
    if (!out && !out_per_k) return KQ_ERR_ARG;
    if (logits && t->d.num_experts > 1024) return KQ_ERR_UNSUPPORTED;
    if (!workspace) return KQ_ERR_WORKSPACE;
    const MoeWs L = moe_ws_layout(t, T, K);
    if (workspace_bytes < L.total) return KQ_ERR_WORKSPACE;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    int32_t* idx_use = idx ? idx : reinterpret_cast<int32_t*>(ws + L.idx);
    float* w_use = weights ? weights : reinterpret_cast<float*>(ws + L.w);
    const bool pdl = true;
    if (logits) {
        if (launch_router(logits, T, t->d.num_experts, K, idx_use, w_use, s, false) != cudaSuccess)
            return KQ_ERR_CUDA;
    }
    GemvParams p{};
    p.base = t->base + (size_t)layer * t->layer_bytes;
    p.expert_bytes = t->expert_bytes;
    p.E = t->d.num_experts;
    p.T = T;
    p.K = K;
    p.idx = idx_use;
    p.w = w_use;
    p.act = reinterpret_cast<float*>(ws + L.act);
    p.amax = reinterpret_cast<float*>(ws + L.amax);
    p.nrt_up = t->i8;
    p.I = t->d.inter;
    p.y = reinterpret_cast<float*>(ws + L.y);
    p.cnt = reinterpret_cast<uint32_t*>(ws + L.cnt);
    p.cnt_per_token = t->h16;
    p.status = reinterpret_cast<uint32_t*>(ws + L.status);
    p.act_kind = t->d.activation;
    p.x = x;
    p.x_dtype = x_dtype;
    // gate/up
    p.mode = MODE_GATEUP;
    p.mat_off = 0;
    p.nrt = t->i8;
    p.nst = t->nst_h;
    p.ncols = t->d.hidden;
    p.prefetch_before_wait = 0;
    if (dispatch_gemv(t->d.bits, t->d.sb_dtype, false, p, s, pdl) != cudaSuccess) return KQ_ERR_CUDA;
    // down (+ combine)
    p.mode = MODE_DOWN;
    p.mat_off = t->gateup_bytes;
    p.nrt = t->h16;
    p.nst = t->nst_i;
    p.ncols = t->d.inter;
    p.H = t->d.hidden;
    p.out_per_k = out_per_k;
    p.out = out;
    p.out_dtype = out_dtype;
    p.residual = residual;
    p.prefetch_before_wait = 1;
    if (dispatch_gemv(t->d.bits, t->d.sb_dtype, true, p, s, true) != cudaSuccess) return KQ_ERR_CUDA;
    return KQ_OK;
}

// ---- dense quantized matrices ---------------------------------------------------------

extern "C" int kq_qmat_create(int rows, int cols, int bits, int sb_dtype, int pair, kq_qmat** out) {
    if (!out) return KQ_ERR_ARG;
    *out = nullptr;
    if (bits != 3 && bits != 4) return KQ_ERR_UNSUPPORTED;
    if (sb_dtype != KQ_DT_F16 && sb_dtype != KQ_DT_BF16) return KQ_ERR_ARG;
    if (rows <= 0 || cols <= 0 || cols % 64) return KQ_ERR_ARG;
    if (pair ? rows % 8 : rows % 16) return KQ_ERR_ARG;
    kq_qmat* m = new (std::nothrow) kq_qmat();
    if (!m) return KQ_ERR_ALLOC;
    m->rows = rows;
    m->cols = cols;
    m->bits = bits;
    m->sb_dtype = sb_dtype;
    m->pair = pair ? 1 : 0;
    m->nrt = pair ? rows / 8 : rows / 16;
    m->nst = (cols + TILE_COLS - 1) / TILE_COLS;
    m->tb = tile_bytes(bits);
    m->bytes = (size_t)m->nrt * m->nst * m->tb;
    if (cudaMalloc(&m->base, m->bytes) != cudaSuccess) {
        cudaGetLastError();
        delete m;
        return KQ_ERR_ALLOC;
    }
    cudaMemset(m->base, 0, m->bytes);
    *out = m;
    return KQ_OK;
}

extern "C" int kq_qmat_destroy(kq_qmat* m) {
    if (!m) return KQ_OK;
    if (m->base) cudaFree(m->base);
    delete m;
    return KQ_OK;
}

namespace kq {
int qmat_repack(kq_qmat* m, const kq_mlx_matrix* a, const kq_mlx_matrix* b, cudaStream_t s);
}

extern "C" int kq_dense_gemv(const kq_qmat* m, const void* x, int x_dtype, int T, const void* norm_w,
                             float eps, int activation, void* y, int y_dtype, void* stream) {
    if (!m || !x || !y) return KQ_ERR_ARG;
    if (!valid_dtype(x_dtype) || !valid_dtype(y_dtype)) return KQ_ERR_ARG;
    if (norm_w && x_dtype == KQ_DT_F32) return KQ_ERR_ARG;
    if (activation != KQ_ACT_SILU && activation != KQ_ACT_GELU_TANH) return KQ_ERR_ARG;
    if (T < 0) return KQ_ERR_ARG;
    if (T == 0) return KQ_OK;
    GemvParams p{};
    p.base = m->base;
    p.E = 1;
    p.T = T;
    p.K = 1;
    p.x = x;
    p.x_dtype = x_dtype;
    p.norm_w = norm_w;
    p.eps = eps;
    p.nrt = m->nrt;
    p.nst = m->nst;
    p.ncols = m->cols;
    p.out = y;
    p.out_dtype = y_dtype;
    p.act_kind = activation;
    p.H = m->rows;
    p.mode = m->pair ? MODE_DENSE_PAIR : MODE_DENSE;
    p.prefetch_before_wait = 1;
    return dispatch_gemv(m->bits, m->sb_dtype, false, p, static_cast<cudaStream_t>(stream), true) ==
                   cudaSuccess
               ? KQ_OK
               : KQ_ERR_CUDA;
}
