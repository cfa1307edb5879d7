// kq_moe.cu -- routed-expert decode path and dense quantized GEMV on sm_100a.
//
// Kernels
//   router_topk_kernel  softmax / top-K / renormalise, one warp per token
//                       (kandiga/metal/moe_block.metal:419-505), built on
//                       warp_topk (REDUX max/min on order-preserving keys).
//   qunit_kernel        one CTA per 16-row unit of a quantized matrix: the unit's
//                       512-column tiles are spread over the CTA's warps, each
//                       tile fetched by its own TMA bulk copy into shared memory
//                       and consumed by the 32-MMA tile engine (kq_qtile.cuh);
//                       the input vector is staged once per CTA; warp partials
//                       are reduced through shared memory.  Epilogues:
//     MODE_GATEUP      routed experts' gate+up rows -> act = silu(g) * u (fp32
//                      scratch) + per-unit max|act|
//                      (kandiga/metal/kandiga_cpu_expert.m:372-394)
//     MODE_DENSE       y = W x, optional RMSNorm prologue
//     MODE_DENSE_PAIR  y = act(Wg x) * (Wu x)
//   moe_down_kernel     one CTA per (token, 16 hidden rows) owning all K
//                       experts: each warp streams its experts' down tiles
//                       (issued before the programmatic-dependent-launch wait on
//                       the gate/up grid), and the CTA forms the per-expert
//                       outputs and the weighted combine (+ residual) in shared
//                       memory (kandiga/metal/kandiga_cpu_expert.m:396-398,
//                       kandiga/metal/moe_block.metal:556-584).
//
// For small token counts the routing runs inside the prologues of both expert
// kernels (no separate router launch); otherwise router_topk_kernel runs first.
#include <cstdio>

#include "kq_internal.h"
#include "kq_route.cuh"

namespace kq {

enum { MODE_GATEUP = 0, MODE_DOWN = 1, MODE_DENSE = 2, MODE_DENSE_PAIR = 3 };

constexpr int MAX_K = 32;
constexpr int ROUTE_INLINE_MAX_T = 8;

struct GemvParams {
    const uint8_t* base;  // layer base (MoE) or matrix base (dense)
    size_t expert_bytes;  // MoE: bytes per expert
    size_t mat_off;       // matrix offset inside an expert
    int nrt, nst;         // row-tiles per vector, column tiles of the matrix
    int E;                // experts (1 for dense)
    int ncols;            // real input length
    int T, K;             // tokens, experts per token (dense: 1)
    const void* x;
    int x_dtype;
    const void* norm_w;
    float eps;
    const float* logits;  // [T][E] when routing runs in the prologues, else null
    int32_t* idx;         // [T*K]
    float* w;             // [T*K]
    float* act;           // [T*K][I]
    float* amax;          // [T*K][I/8] per gate/up unit max |act|
    int nrt_up;           // gate/up units per (token, k): I/8
    int I;
    void* out_per_k;      // [T*K][H] (out_dtype) or null
    void* out;            // [T][rows] (out_dtype) or null
    int out_dtype;
    const void* residual; // [T][H] (out_dtype) or null
    int act_kind;
    int H;                // output rows
    uint32_t* status;
    int mode;
};

__host__ __device__ constexpr size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

__global__ void router_topk_kernel(const float* __restrict__ logits, int T, int E, int K,
                                   int32_t* __restrict__ idx, float* __restrict__ wout) {
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    pdl_wait();
    pdl_launch_dependents();
    if (t >= T) return;
    int i;
    float w;
    warp_topk_any(logits + (size_t)t * E, E, K, i, w);
    if (lane < K) {
        idx[(size_t)t * K + lane] = i;
        wout[(size_t)t * K + lane] = w;
    }
}

// ---- block-wide input staging ----------------------------------------------------------


// Stage input vector `vec` (x row, optional RMSNorm) into xs/cx, using the
// threads [t0, t0 + nthr) of the CTA (whole warps, sharing named barrier 1).
// Returns 1/scale.
template <int BITS>
__device__ __forceinline__ float block_stage_x(const GemvParams& p, int vec, int npad, __half* xs,
                                               float2* cx, float* scratch, int t0, int nthr) {
    const int rank = threadIdx.x - t0, lane = rank & 31, wl = rank >> 5;
    const size_t off = (size_t)vec * p.ncols;
    const int nch = p.ncols / 8;
    float scale = 1.f, rinv = 1.f;
    if (p.norm_w != nullptr || p.x_dtype != KQ_DT_F16) {
        float amax = 0.f, ss = 0.f;
        for (int c = rank; c < nch; c += nthr) {
            float v[8], wv[8];
            load8(p.x, p.x_dtype, off + (size_t)c * 8, false, v);
            if (p.norm_w) load8(p.norm_w, p.x_dtype, (size_t)c * 8, false, wv);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                ss += v[k] * v[k];
                amax = fmaxf(amax, fabsf(p.norm_w ? v[k] * wv[k] : v[k]));
            }
        }
        amax = warp_max(amax);
        ss = warp_sum(ss);
        if (lane == 0) {
            scratch[wl] = amax;
            scratch[16 + wl] = ss;
        }
        named_barrier_sync(1, nthr);
        amax = 0.f;
        ss = 0.f;
        for (int w = 0; w < nthr / 32; ++w) {
            amax = fmaxf(amax, scratch[w]);
            ss += scratch[16 + w];
        }
        if (p.norm_w) rinv = rsqrtf(ss / (float)p.ncols + p.eps);
        scale = pow2_scale(amax * rinv);
    }
    stage_fused<BITS, 2>(p.x, p.x_dtype, off, p.ncols, npad, rinv * scale, false, rank, nthr, xs, cx, p.norm_w);
    return 1.f / scale;
}

// ---- qunit_kernel: gate/up and dense matrices ---------------------------------------------

// Tile slots of a CTA: NBUF per warp, reused round-robin, one mbarrier each;
// or, with PA ("prefetch all"), one per tile of the CTA's RT row tiles in the
// matrix's own order, filled by one bulk copy per row tile (its nst tiles are
// contiguous) issued before the programmatic-dependent-launch wait, one
// mbarrier per row tile.  A copy engine completes a few bulk copies per
// microsecond per SM whatever their size, so whole rows (18-64 KB) instead of
// 3.5 KB tiles keep it off the critical path.
template <int NW, int NBUF, int RT, bool PA>
__host__ __device__ constexpr int qunit_slots(int nst) {
    return PA ? RT * nst : NW * NBUF;
}
template <int NW, int NBUF, int RT, bool PA>
__host__ __device__ constexpr int qunit_bars(int nst) {
    return PA ? RT : NW * NBUF;
}

template <int BITS, int NW, int NBUF, int RT = 1, bool PA = false>
__host__ __device__ constexpr size_t qunit_smem(int nst) {
    return align_up((size_t)qunit_slots<NW, NBUF, RT, PA>(nst) * TileT<BITS>::BYTES, 128) +  // tiles
           align_up((size_t)nst * TILE_COLS * 2, 128) +                  // xs
           align_up((size_t)nst * TILE_GROUPS * 8, 128) +                // cx
           align_up((size_t)NW * 32 * 8, 128) +                          // warp partials
           align_up((size_t)qunit_bars<NW, NBUF, RT, PA>(nst) * 8, 128) +   // mbarriers
           256;                                                           // scratch
}

// RT > 1 (dense matrices only): RT row tiles per CTA, NW / RT warps each,
// sharing one staged input.  PA (dense matrices only): every tile of the CTA
// has its own slot, so no copy is issued after the wait.
template <int BITS, int SB_DT, int NW, int NBUF, int RT = 1, bool PA = false>
__global__ void __launch_bounds__(NW * 32) qunit_kernel(const GemvParams p) {
    constexpr int WPG = NW / RT;  // warps per row tile
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int TB = TileT<BITS>::BYTES;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int npad = p.nst * TILE_COLS, ng = npad / GS;
    const int nslot = qunit_slots<NW, NBUF, RT, PA>(p.nst), nbar = qunit_bars<NW, NBUF, RT, PA>(p.nst);
    uint8_t* sp = smem;
    uint8_t* tiles = sp;
    sp += align_up((size_t)nslot * TB, 128);
    __half* xs = reinterpret_cast<__half*>(sp);
    sp += align_up((size_t)npad * 2, 128);
    float2* cx = reinterpret_cast<float2*>(sp);
    sp += align_up((size_t)ng * 8, 128);
    float2* red = reinterpret_cast<float2*>(sp);
    sp += align_up((size_t)NW * 32 * 8, 128);
    uint64_t* bars = reinterpret_cast<uint64_t*>(sp);
    sp += align_up((size_t)nbar * 8, 128);
    float* scratch = reinterpret_cast<float*>(sp);   // 2*NW floats
    int* s_e = reinterpret_cast<int*>(sp + 192);     // expert id of this unit

    float* s_inv = reinterpret_cast<float*>(sp + 196);  // 1/scale of the staged input

    const int mode = p.mode;
    const int u = blockIdx.x;
    const int nrtc = (p.nrt + RT - 1) / RT;  // CTAs per token
    const int tk = u / nrtc;
    const int grp = warp / WPG, wg = warp % WPG;
    const int rt = (u % nrtc) * RT + grp;    // this warp's row tile
    const bool rt_ok = rt < p.nrt;
    const int t = tk / p.K, k = tk % p.K;
    if (tid == 0) {  // every warp's barriers, so warp 0 may issue copies for all of them
        for (int b = 0; b < nbar; ++b) mbar_init(&bars[b], 1);
        fence_mbar_init();
    }
    __syncthreads();
    // warp w's tiles: column tiles st = w % WPG, + WPG, ... of row tile (u % nrtc) * RT + w / WPG
    auto ntiles_of = [&](int w) {
        const int wl = w % WPG;
        if ((u % nrtc) * RT + w / WPG >= p.nrt) return 0;
        return wl < p.nst ? (p.nst - 1 - wl) / WPG + 1 : 0;
    };
    const int ntl = ntiles_of(warp);
    // slot of warp w's i-th tile (column tile w % WPG + i * WPG of its row tile)
    auto slot_of = [&](int w, int i) {
        return PA ? (w / WPG) * p.nst + w % WPG + i * WPG : w * NBUF + i % NBUF;
    };
    const uint64_t pol = policy_evict_first();
    auto issue_for = [&](int w, int i, const uint8_t* mb) {  // per-warp ring (not PA)
        const int st = w % WPG + i * WPG, slot = slot_of(w, i);
        const int rtw = (u % nrtc) * RT + w / WPG;
        uint64_t* bar = bars + slot;
        mbar_expect_tx(bar, TB);
        bulk_g2s(tiles + (size_t)slot * TB, mb + ((size_t)rtw * p.nst + st) * TB, TB, bar, pol);
    };
    auto issue_row = [&](int g, const uint8_t* mb) {  // PA: row tile g of the CTA, all its tiles
        const int rtw = (u % nrtc) * RT + g;
        if (rtw >= p.nrt) return;
        const uint32_t bytes = (uint32_t)p.nst * TB;
        mbar_expect_tx(&bars[g], bytes);
        bulk_g2s(tiles + (size_t)g * p.nst * TB, mb + (size_t)rtw * p.nst * TB, bytes, &bars[g], pol);
    };

    bool valid = true;
    const uint8_t* mbase = p.base + p.mat_off;
    float inv = 1.f;
    if (mode == MODE_GATEUP) {
        pdl_wait();  // routing inputs and x come from earlier work on the stream
        pdl_launch_dependents();
        if (warp == 0) {
            // routing, then every warp's first tiles; warps 1.. stage x meanwhile
            int e;
            if (p.logits) {
                int ix;
                float wt;
                warp_topk<8>(p.logits + (size_t)t * p.E, p.E, p.K, ix, wt);
                if (rt == 0 && k == 0 && lane < p.K) {  // one CTA per token publishes the routing
                    p.idx[(size_t)t * p.K + lane] = ix;
                    p.w[(size_t)t * p.K + lane] = wt;
                }
                e = __shfl_sync(0xffffffffu, ix, k);
            } else {
                e = __ldcg(p.idx + tk);
            }
            if (lane == 0) {
                *s_e = e;
                const uint8_t* mb = mbase + (size_t)((unsigned)e < (unsigned)p.E ? e : 0) * p.expert_bytes;
                if constexpr (PA) {
                    for (int g = 0; g < RT; ++g) issue_row(g, mb);
                } else {
                    for (int w = 0; w < NW; ++w)
                        for (int i = 0; i < NBUF && i < ntiles_of(w); ++i) issue_for(w, i, mb);
                }
            }
        } else {
            const float iv = block_stage_x<BITS>(p, t, npad, xs, cx, scratch, 32, (NW - 1) * 32);
            if (tid == 32) *s_inv = iv;
        }
        __syncthreads();
        int e = *s_e;
        inv = *s_inv;
        valid = (unsigned)e < (unsigned)p.E;
        if (!valid) {  // rows are zeroed; an id other than -1 (an empty slot) is latched
            if (tid == 0 && e != -1) set_status(p.status, KQ_DEV_BAD_EXPERT);
            e = 0;         // a real expert is addressed
        }
        mbase += (size_t)e * p.expert_bytes;
    } else {
        if (lane == 0) {  // dense weights do not depend on earlier work: fetch before the wait
            if constexpr (PA) {
                if (wg == 0) issue_row(grp, mbase);
            } else {
                for (int i = 0; i < NBUF && i < ntl; ++i) issue_for(warp, i, mbase);
            }
        }
        pdl_wait();
        pdl_launch_dependents();
        inv = block_stage_x<BITS>(p, tk, npad, xs, cx, scratch, 0, NW * 32);
        __syncthreads();
    }

    float y0 = 0.f, y1 = 0.f;
    if (PA && ntl > 0) mbar_wait(&bars[grp], 0u, p.status);
    for (int i = 0; i < ntl; ++i) {
        const int slot = slot_of(warp, i);
        if (!PA) mbar_wait(&bars[slot], (uint32_t)((i / NBUF) & 1), p.status);
        TileRegs<BITS> R;
        tile_load<BITS>(tiles + (size_t)slot * TB, R);
        __syncwarp();
        if (!PA && lane == 0 && i + NBUF < ntl) {
            fence_proxy_async_smem();
            issue_for(warp, i + NBUF, mbase);
        }
        tile_compute<BITS, SB_DT>(R, wg + i * WPG, xs, cx, y0, y1);
    }
    red[warp * 32 + lane] = make_float2(y0, y1);
    __syncthreads();
    if (wg != 0 || !rt_ok) return;  // the first warp of each row tile finishes it
    y0 = 0.f;
    y1 = 0.f;
#pragma unroll
    for (int w = 0; w < WPG; ++w) {
        const float2 v = red[(grp * WPG + w) * 32 + lane];
        y0 += v.x;
        y1 += v.y;
    }
    quad_reduce(y0, y1);
    const int r = lane >> 2;
    const float g = valid ? y0 * inv : 0.f, h = valid ? y1 * inv : 0.f;
    if (mode == MODE_DENSE) {
        if ((lane & 3) == 0) {
            const size_t o0 = (size_t)tk * p.H + rt * 16 + r, o1 = o0 + 8;
            // residual (out_dtype, may alias out): out = residual + W x
            const float r0 = p.residual ? load_as_float(p.residual, p.out_dtype, o0) : 0.f;
            const float r1 = p.residual ? load_as_float(p.residual, p.out_dtype, o1) : 0.f;
            store_from_float(p.out, p.out_dtype, o0, p.residual ? r0 + g : g);
            store_from_float(p.out, p.out_dtype, o1, p.residual ? r1 + h : h);
        }
        return;
    }
    const float a = valid ? activate(g, h, p.act_kind) : 0.f;
    if (mode == MODE_DENSE_PAIR) {
        if ((lane & 3) == 0) store_from_float(p.out, p.out_dtype, (size_t)tk * p.H + rt * 8 + r, a);
        return;
    }
    if ((lane & 3) == 0) p.act[(size_t)tk * p.I + rt * 8 + r] = a;
    const float m = warp_max(fabsf(a));
    if (lane == 0) p.amax[(size_t)tk * p.nrt + rt] = m;
}

// ---- moe_down_kernel ------------------------------------------------------------------------

constexpr int DOWN_NW = 8;
constexpr int DOWN_NBUF = 2;

template <int BITS>
__host__ __device__ constexpr size_t down_warp_smem(int nst) {
    return align_up((size_t)DOWN_NBUF * TileT<BITS>::BYTES + (size_t)nst * TILE_COLS * 2 +
                        (size_t)nst * TILE_GROUPS * 8 + DOWN_NBUF * 8,
                    128);
}
template <int BITS>
__host__ __device__ constexpr size_t down_smem(int nst) {
    return DOWN_NW * down_warp_smem<BITS>(nst) + MAX_K * 16 * 4 + MAX_K * 8 + 128;
}

template <int BITS, int SB_DT>
__global__ void __launch_bounds__(DOWN_NW * 32, 1) moe_down_kernel(const GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int TB = TileT<BITS>::BYTES;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int npad = p.nst * TILE_COLS, ng = npad / GS;
    uint8_t* wb = smem + (size_t)warp * down_warp_smem<BITS>(p.nst);
    uint8_t* tiles = wb;
    __half* xs = reinterpret_cast<__half*>(wb + DOWN_NBUF * TB);
    float2* cx = reinterpret_cast<float2*>(wb + DOWN_NBUF * TB + (size_t)npad * 2);
    uint64_t* bars = reinterpret_cast<uint64_t*>(wb + DOWN_NBUF * TB + (size_t)npad * 2 + (size_t)ng * 8);
    float* red = reinterpret_cast<float*>(smem + DOWN_NW * down_warp_smem<BITS>(p.nst));  // [MAX_K][16]
    int* s_idx = reinterpret_cast<int*>(red + MAX_K * 16);
    float* s_w = reinterpret_cast<float*>(s_idx + MAX_K);

    const int t = blockIdx.x / p.nrt, rt = blockIdx.x % p.nrt;
    if (lane == 0) {
#pragma unroll
        for (int b = 0; b < DOWN_NBUF; ++b) mbar_init(&bars[b], 1);
        fence_mbar_init();
    }
    // Routing of token t.  The gate/up grid may still be running: routing is
    // recomputed from the logits (or read from idx, written before that grid
    // started), so the down weights can be fetched before the dependency wait.
    if (p.logits) {
        if (warp == 0) {
            int ix;
            float wt;
            warp_topk<8>(p.logits + (size_t)t * p.E, p.E, p.K, ix, wt);
            if (lane < p.K) {
                s_idx[lane] = ix;
                s_w[lane] = wt;
            }
        }
    } else if (tid < p.K) {
        s_idx[tid] = __ldcg(p.idx + (size_t)t * p.K + tid);
        s_w[tid] = p.w ? __ldcg(p.w + (size_t)t * p.K + tid) : 0.f;
    }
    __syncthreads();
    // this warp's experts: k = warp, warp + DOWN_NW, ...; tiles f = j * nst + st
    const int nexp = warp < p.K ? (p.K - 1 - warp) / DOWN_NW + 1 : 0;
    const int ntl = nexp * p.nst;
    const uint64_t pol = policy_evict_first();
    auto issue = [&](int f) {
        const int kk = warp + (f / p.nst) * DOWN_NW, st = f % p.nst;
        int e = s_idx[kk];
        if ((unsigned)e >= (unsigned)p.E) e = 0;
        const uint8_t* src = p.base + (size_t)e * p.expert_bytes + p.mat_off + ((size_t)rt * p.nst + st) * TB;
        const int slot = f % DOWN_NBUF;
        mbar_expect_tx(&bars[slot], TB);
        bulk_g2s(tiles + (size_t)slot * TB, src, TB, &bars[slot], pol);
    };
    if (lane == 0)
        for (int f = 0; f < DOWN_NBUF && f < ntl; ++f) issue(f);
    pdl_launch_dependents();
    pdl_wait();  // gate/up activations are complete and visible

    for (int j = 0; j < nexp; ++j) {
        const int kk = warp + j * DOWN_NW;
        const size_t tk = (size_t)t * p.K + kk;
        const bool valid = (unsigned)s_idx[kk] < (unsigned)p.E;
        const float inv = stage_act_warp<BITS>(p.act + tk * p.I, p.amax + tk * p.nrt_up, p.nrt_up, p.ncols,
                                               npad, xs, cx);
        float y0 = 0.f, y1 = 0.f;
        for (int st = 0; st < p.nst; ++st) {
            const int f = j * p.nst + st, slot = f % DOWN_NBUF;
            mbar_wait(&bars[slot], (uint32_t)((f / DOWN_NBUF) & 1), p.status);
            TileRegs<BITS> R;
            tile_load<BITS>(tiles + (size_t)slot * TB, R);
            __syncwarp();
            if (lane == 0 && f + DOWN_NBUF < ntl) {
                fence_proxy_async_smem();
                issue(f + DOWN_NBUF);
            }
            tile_compute<BITS, SB_DT>(R, st, xs, cx, y0, y1);
        }
        quad_reduce(y0, y1);
        const float g = valid ? y0 * inv : 0.f, h = valid ? y1 * inv : 0.f;
        if (!valid && lane == 0 && s_idx[kk] != -1) set_status(p.status, KQ_DEV_BAD_EXPERT);
        if ((lane & 3) == 0) {
            const int r = lane >> 2;
            if (p.out_per_k) {
                const size_t o = tk * p.H + rt * 16 + r;
                store_from_float(p.out_per_k, p.out_dtype, o, g);
                store_from_float(p.out_per_k, p.out_dtype, o + 8, h);
            }
            red[kk * 16 + r] = g;
            red[kk * 16 + r + 8] = h;
        }
    }
    if (!p.out) return;
    __syncthreads();
    if (tid < 16) {
        const int row = rt * 16 + tid;
        float acc = 0.f;
        for (int kk = 0; kk < p.K; ++kk) acc += red[kk * 16 + tid] * s_w[kk];
        if (p.residual) acc = load_as_float(p.residual, p.out_dtype, (size_t)t * p.H + row) + acc;
        store_from_float(p.out, p.out_dtype, (size_t)t * p.H + row, acc);
    }
}

// ---- launch helpers -----------------------------------------------------------------------------

// Raise a kernel's dynamic shared-memory limit once per device.
template <typename Kern>
static cudaError_t smem_attr(Kern kern, size_t bytes, int* /*unused*/) {
    return raise_smem_limit(reinterpret_cast<const void*>(kern), bytes);
}

template <typename Kern>
static cudaError_t launch_pdl(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              const GemvParams& p) {
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
    return cudaLaunchKernelEx(&cfg, kern, p);
}

constexpr int QUNIT_NW = 4;
constexpr int QUNIT_NBUF = 2;

template <int BITS, int SB_DT>
static cudaError_t launch_qunit_t(const GemvParams& p, cudaStream_t s) {
    static int configured[64] = {0};
    auto kern = qunit_kernel<BITS, SB_DT, QUNIT_NW, QUNIT_NBUF>;
    const size_t smem = qunit_smem<BITS, QUNIT_NW, QUNIT_NBUF>(p.nst);
    cudaError_t err = smem_attr(kern, smem, configured);
    if (err != cudaSuccess) return err;
    const long units = (long)p.T * p.K * p.nrt;
    return launch_pdl(kern, dim3((unsigned)units), dim3(QUNIT_NW * 32), smem, s, p);
}

template <int BITS, int SB_DT>
static cudaError_t launch_down_t(const GemvParams& p, cudaStream_t s) {
    static int configured[64] = {0};
    auto kern = moe_down_kernel<BITS, SB_DT>;
    const size_t smem = down_smem<BITS>(p.nst);
    cudaError_t err = smem_attr(kern, smem, configured);
    if (err != cudaSuccess) return err;
    return launch_pdl(kern, dim3((unsigned)(p.T * p.nrt)), dim3(DOWN_NW * 32), smem, s, p);
}

// Dense matrices (MODE_DENSE / MODE_DENSE_PAIR): warps per CTA and tile
// buffers per warp of the same kernel, tuned apart from the routed path.
#ifndef KQ_DENSE_NW
#define KQ_DENSE_NW 4
#endif
#ifndef KQ_DENSE_NBUF
#define KQ_DENSE_NBUF 2
#endif

#ifndef KQ_WIDE_MIN_NST
#define KQ_WIDE_MIN_NST 8  // column tiles from which a matrix gets wide CTAs
#endif

template <int BITS, int SB_DT, int NW, int NBUF, int RT = 1, bool PA = false>
static cudaError_t launch_dense_nw(const GemvParams& p, cudaStream_t s) {
    auto kern = qunit_kernel<BITS, SB_DT, NW, NBUF, RT, PA>;
    const size_t smem = qunit_smem<BITS, NW, NBUF, RT, PA>(p.nst);
    cudaError_t err = smem_attr(kern, smem, nullptr);
    if (err != cudaSuccess) return err;
    const long units = (long)p.T * p.K * ((p.nrt + RT - 1) / RT);
    return launch_pdl(kern, dim3((unsigned)units), dim3(NW * 32), smem, s, p);
}

#ifndef KQ_SHORT_RT
#define KQ_SHORT_RT 4  // row tiles per CTA for short rows with many row tiles
#endif
#ifndef KQ_SHORT_NBUF
#define KQ_SHORT_NBUF 1
#endif

#ifndef KQ_DENSE_PA
#define KQ_DENSE_PA 1
#endif
#ifndef KQ_PA_NW
#define KQ_PA_NW 16
#endif
constexpr size_t PA_MAX_TILE_BYTES = 100 * 1024;  // tile slots of one CTA in prefetch-all mode

// Prefetch-all (a matrix row of at most PA_MAX_TILE_BYTES): every tile of a
// CTA is in flight before the wait, so after the previous launch completes
// only the input staging and the arithmetic remain.  RT is the smallest of 1,
// 2, 4 that fits the launch in one wave at two CTAs per SM.
// Otherwise: long rows (K >= 4096) with few row tiles (one wave at two CTAs per
// SM) get 16 warps per CTA: each thread stages and multiplies a quarter as much.
template <int BITS, int SB_DT>
static cudaError_t launch_dense_t(const GemvParams& p, cudaStream_t s) {
    const long units = (long)p.T * p.K * p.nrt;
    const size_t row_bytes = (size_t)p.nst * TileT<BITS>::BYTES;
    if (KQ_DENSE_PA && row_bytes <= PA_MAX_TILE_BYTES) {
        if (units <= 2L * 148 || 2 * row_bytes > PA_MAX_TILE_BYTES)
            return launch_dense_nw<BITS, SB_DT, KQ_PA_NW, 1, 1, true>(p, s);
        if (units <= 4L * 148 || 4 * row_bytes > PA_MAX_TILE_BYTES)
            return launch_dense_nw<BITS, SB_DT, KQ_PA_NW, 1, 2, true>(p, s);
        return launch_dense_nw<BITS, SB_DT, KQ_PA_NW, 1, 4, true>(p, s);
    }
    if (p.nst >= KQ_WIDE_MIN_NST && units <= 2L * 148) return launch_dense_nw<BITS, SB_DT, 16, 1>(p, s);
    if (KQ_SHORT_RT > 1 && p.nst < KQ_WIDE_MIN_NST && units > 2L * 148)
        return launch_dense_nw<BITS, SB_DT, 4 * KQ_SHORT_RT, KQ_SHORT_NBUF, KQ_SHORT_RT>(p, s);
    return launch_dense_nw<BITS, SB_DT, KQ_DENSE_NW, KQ_DENSE_NBUF>(p, s);
}

static cudaError_t launch_qunit(int bits, int sb_dt, const GemvParams& p, cudaStream_t s) {
    if (p.mode == MODE_DENSE || p.mode == MODE_DENSE_PAIR) {
        if (bits == 3)
            return sb_dt == KQ_DT_F16 ? launch_dense_t<3, KQ_DT_F16>(p, s) : launch_dense_t<3, KQ_DT_BF16>(p, s);
        return sb_dt == KQ_DT_F16 ? launch_dense_t<4, KQ_DT_F16>(p, s) : launch_dense_t<4, KQ_DT_BF16>(p, s);
    }
    if (bits == 3) return sb_dt == KQ_DT_F16 ? launch_qunit_t<3, KQ_DT_F16>(p, s) : launch_qunit_t<3, KQ_DT_BF16>(p, s);
    return sb_dt == KQ_DT_F16 ? launch_qunit_t<4, KQ_DT_F16>(p, s) : launch_qunit_t<4, KQ_DT_BF16>(p, s);
}

static cudaError_t launch_down(int bits, int sb_dt, const GemvParams& p, cudaStream_t s) {
    if (bits == 3) return sb_dt == KQ_DT_F16 ? launch_down_t<3, KQ_DT_F16>(p, s) : launch_down_t<3, KQ_DT_BF16>(p, s);
    return sb_dt == KQ_DT_F16 ? launch_down_t<4, KQ_DT_F16>(p, s) : launch_down_t<4, KQ_DT_BF16>(p, s);
}

static cudaError_t launch_router(const float* logits, int T, int E, int K, int32_t* idx, float* w,
                                 cudaStream_t s) {
    const int warps = 4;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((T + warps - 1) / warps);
    cfg.blockDim = dim3(warps * 32);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, router_topk_kernel, logits, T, E, K, idx, w);
}

// One token's routing plus a fixed shared expert: top-K of logits[0, E)
// (softmax, strict '>', lowest index on ties, renormalised), then assignment K
// = (shared_id, sigmoid(logits[E])) -- the shared expert's gate logit computed
// by the same GEMV as the router (moe_block.metal:335-404, 515-584).
__global__ void route_shared_kernel(const float* __restrict__ logits, int E, int K, int shared_id,
                                    int32_t* __restrict__ idx, float* __restrict__ wout) {
    pdl_wait();
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31;
    int i;
    float w;
    warp_topk_any(logits, E, K, i, w);
    if (lane < K) {
        idx[lane] = i;
        wout[lane] = w;
    }
    if (lane == 0) {
        idx[K] = shared_id;
        wout[K] = 1.f / (1.f + expf(-__ldcg(logits + E)));
    }
}

int route_with_shared(const float* logits, int E, int K, int shared_id, int32_t* idx, float* w,
                      cudaStream_t s) {
    if (E > 1024 || K + 1 > MAX_K || K > 32) return KQ_ERR_UNSUPPORTED;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(32);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, route_shared_kernel, logits, E, K, shared_id, idx, w) == cudaSuccess ? KQ_OK
                                                                                                       : KQ_ERR_CUDA;
}

int launch_router_ext(const float* logits, int T, int E, int K, int32_t* idx, float* w, cudaStream_t s) {
    if (E > 1024 || K > MAX_K) return KQ_ERR_UNSUPPORTED;
    return launch_router(logits, T, E, K, idx, w, s) == cudaSuccess ? KQ_OK : KQ_ERR_CUDA;
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
    L.amax = o;
    o = align_up(o + (size_t)T * K * t->i8 * 4, 256);
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
    if (T < 0 || E <= 0 || E > 1024 || K <= 0 || K > E || K > MAX_K) return KQ_ERR_ARG;
    if (T == 0) return KQ_OK;
    if (!logits || !idx || !weights) return KQ_ERR_ARG;
    return launch_router(logits, T, E, K, idx, weights, static_cast<cudaStream_t>(stream)) == cudaSuccess
               ? KQ_OK
               : KQ_ERR_CUDA;
}

extern "C" int kq_moe_decode(const kq_table* t, int layer, const void* x, int x_dtype, int T,
                             const float* logits, int32_t* idx, float* weights, int K,
                             void* out_per_k, void* out, int out_dtype, const void* residual,
                             void* workspace, size_t workspace_bytes, void* stream) {
    return kq::moe_decode_ex(t, layer, x, x_dtype, T, logits, idx, weights, K, out_per_k, out, out_dtype, residual,
                             nullptr, 0.f, workspace, workspace_bytes, stream);
}

int kq::moe_decode_ex(const kq_table* t, int layer, const void* x, int x_dtype, int T, const float* logits,
                      int32_t* idx, float* weights, int K, void* out_per_k, void* out, int out_dtype,
                      const void* residual, const void* norm_w, float eps, void* workspace, size_t workspace_bytes,
                      void* stream) {
    if (!t) return KQ_ERR_ARG;
    if (norm_w && x_dtype != KQ_DT_F16) return KQ_ERR_ARG;
    if (layer < 0 || layer >= t->d.num_layers) return KQ_ERR_ARG;
    if (T < 0 || K <= 0 || K > MAX_K || K > t->d.num_experts) return KQ_ERR_ARG;
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
    const bool inline_route = logits && T <= ROUTE_INLINE_MAX_T && t->d.num_experts <= 256;
    if (logits && !inline_route) {
        if (launch_router(logits, T, t->d.num_experts, K, idx_use, w_use, s) != cudaSuccess) return KQ_ERR_CUDA;
    }
    GemvParams p{};
    p.base = t->base + (size_t)layer * t->layer_bytes;
    p.expert_bytes = t->expert_bytes;
    p.E = t->d.num_experts;
    p.T = T;
    p.K = K;
    p.logits = inline_route ? logits : nullptr;
    p.idx = idx_use;
    p.w = w_use;
    p.act = reinterpret_cast<float*>(ws + L.act);
    p.amax = reinterpret_cast<float*>(ws + L.amax);
    p.nrt_up = t->i8;
    p.I = t->d.inter;
    p.status = reinterpret_cast<uint32_t*>(ws + L.status);
    p.act_kind = t->d.activation;
    p.x = x;
    p.x_dtype = x_dtype;
    p.norm_w = norm_w;  // RMSNorm of x in the gate/up staging (the down pass reads the activations)
    p.eps = eps;
    // gate/up + SwiGLU
    p.mode = MODE_GATEUP;
    p.mat_off = 0;
    p.nrt = t->i8;
    p.nst = t->nst_h;
    p.ncols = t->d.hidden;
    if (launch_qunit(t->d.bits, t->d.sb_dtype, p, s) != cudaSuccess) return KQ_ERR_CUDA;
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
    if (launch_down(t->d.bits, t->d.sb_dtype, p, s) != cudaSuccess) return KQ_ERR_CUDA;
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

extern "C" int kq_dense_gemv(const kq_qmat* m, const void* x, int x_dtype, int T, const void* norm_w,
                             float eps, int activation, void* y, int y_dtype, void* stream) {
    return kq::dense_gemv_res(m, x, x_dtype, T, norm_w, eps, activation, y, y_dtype, nullptr, stream);
}

int kq::dense_gemv_res(const kq_qmat* m, const void* x, int x_dtype, int T, const void* norm_w, float eps,
                       int activation, void* y, int y_dtype, const void* residual, void* stream) {
    if (!m || !x || !y) return KQ_ERR_ARG;
    if (residual && m->pair) return KQ_ERR_ARG;
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
    p.residual = residual;
    p.mode = m->pair ? MODE_DENSE_PAIR : MODE_DENSE;
    return launch_qunit(m->bits, m->sb_dtype, p, static_cast<cudaStream_t>(stream)) == cudaSuccess
               ? KQ_OK
               : KQ_ERR_CUDA;
}
