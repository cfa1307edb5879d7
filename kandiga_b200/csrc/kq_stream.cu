// kq_stream.cu -- routed-expert decode of many independent single-token items
// in one persistent launch.
//
// Each item (token t of layer l) is the reference's per-token expert path:
// softmax top-K routing (kandiga/metal/moe_block.metal:419-505), then per
// routed expert gate/up + SwiGLU + down (kandiga/metal/kandiga_cpu_expert.m:
// 355-401, 471-552), then the weighted blend (moe_block.metal:556-584).
//
// Work unit = (item j, expert slot k): one CTA streams that expert's whole
// matrix pair through its shared memory -- gate/up row tiles, the SwiGLU
// activations kept on chip, then down row tiles -- and writes w_k * y_k into
// a partial-sum ring.  The K work units of an item run on K different CTAs;
// the last of them to finish adds the K partial rows in slot order (plus the
// residual), so the result does not depend on timing.  Work units are taken
// round robin, CTA c doing units c, c + P, c + 2P ... (one CTA per SM).  No
// CTA ever waits for another except to reuse a partial-sum slot RP items
// later, which in this order has long been released.
//
// Weights arrive by TMA bulk copies of up to 4 tiles (14-18 KB): each SM's
// copy engine completes only a few bulk copies per microsecond whatever their
// size (measured on B200: 3.5 KB copies stream ~17 GB/s per SM, 14 KB copies
// ~49 GB/s), so per-tile copies would cap the whole GPU far below HBM peak.
//
// Warp roles inside a CTA:
//   warp 0    units: routing of the unit's item (top-K of its logits, or the
//             given routing) and its input row staged as fp16 + per-group
//             constants (optional RMSNorm), RW units ahead
//   warps 1+  CW consumers.  Warp w owns gate/up row tiles rt = w, w + CW, ...
//             and down row-tile blocks b = w, w + CW, ... (a block: as many
//             consecutive down row tiles as make up to 4 tiles), so it
//             finishes every row tile it starts and no partial sums cross
//             warps.  Its lane 0 streams the warp's copies through a private
//             ring of 2 slots, running into the next units' copies once their
//             routing is published.  Gate/up rows give the SwiGLU activations
//             (kept in shared memory; after the phase one power-of-two scale
//             per unit from their maximum, staged to fp16); down rows give 16
//             outputs each.
#include <cstdio>

#include "kq_internal.h"
#include "kq_route.cuh"

namespace kq {

constexpr int EX_MAXCW = 8;                    // consumer warps at most
constexpr int EX_W_AUX = 0, EX_CW0 = 1;
constexpr int EX_MAXTHREADS = (EX_CW0 + EX_MAXCW) * 32;
constexpr int EX_CT = 4;                       // tiles per copy at most
constexpr int EX_NW = 2;                       // slots in each consumer warp's ring
constexpr int EX_RW = 3;                       // work units in the per-CTA routing / input ring
constexpr int EX_RP = 64;                      // items in the global partial-sum ring
constexpr int EX_MAXK = 32;
constexpr int EX_BAR = 1;                      // named barrier of the consumer warps
constexpr size_t EX_SMEM_MAX = 227 * 1024;

struct ExParams {
    const uint8_t* base;        // table
    size_t layer_bytes, expert_bytes, gateup_bytes;
    int E, K, H, I;
    int nst_h, nst_i;           // column tiles of gate/up and down
    int nrt_up, nrt_dn;         // gate/up row tiles (I / 8) and down row tiles (H / 16)
    int db;                     // down row tiles per block
    int cw;                     // consumer warps
    int n;                      // items
    const int32_t* layers;      // [n] or null: every item uses `layer`
    int layer;
    const void* x;              // [n][H]
    int x_dtype;
    const float* logits;        // [n][E] or null
    const int32_t* idx_in;      // [n][K] (logits null)
    const float* w_in;          // [n][K] (logits null; may be null when out is null)
    int32_t* idx_out;           // [n][K] or null
    float* w_out;               // [n][K] or null
    const void* norm_w;         // [H] RMSNorm weight (x dtype) or null
    float eps;
    void* out;                  // [n][H] or null
    void* out_per_k;            // [n][K][H] or null
    int out_dtype;
    const void* residual;       // [n][H] (out_dtype) or null
    int act_kind;
    float* part;                // [RP][K][H] w_k y_k
    unsigned* pcnt;             // [RP] units of the slot's items done
    unsigned* pgen;             // [RP] combines done (item / RP + 1 after item's)
    uint32_t* status;
    // shared-memory layout (bytes)
    uint32_t slot_bytes, unit_bytes;  // a consumer warp's ring slot (4 tiles), a unit record
    uint32_t off_unit, off_act, off_xd, off_misc, off_bar;
};

__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned ld_relaxed(const unsigned* p) {
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release(unsigned* p, unsigned v) {
    asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_cta(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_cta(unsigned* p, unsigned v) {
    asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(smem_u32(p)), "r"(v) : "memory");
}

__device__ __forceinline__ bool wait_timed_out(uint64_t t0, uint32_t* status) {
    if (*reinterpret_cast<volatile uint32_t*>(status) & KQ_DEV_WAIT_TIMEOUT) return true;
    if (global_ns() - t0 > KQ_WAIT_NS) {
        set_status(status, KQ_DEV_WAIT_TIMEOUT);
        return true;
    }
    return false;
}

// Wait until *p >= target (global; bounded by KQ_WAIT_NS): relaxed polls with
// a growing pause, then one acquire fence.
__device__ __forceinline__ bool wait_count(const unsigned* p, unsigned target, uint32_t* status) {
    if (ld_acquire(p) >= target) return true;
    const uint64_t t0 = global_ns();
    unsigned pause = 64;
    for (;;) {
        __nanosleep(pause);
        if (ld_relaxed(p) >= target) {
            asm volatile("fence.acq_rel.gpu;" ::: "memory");
            return true;
        }
        if (pause < 1024) pause *= 2;
        if (wait_timed_out(t0, status)) return false;
    }
}

// Wait until *p > v (shared, this CTA; bounded by KQ_WAIT_NS).
__device__ __forceinline__ bool wait_cta_above(const unsigned* p, unsigned v, uint32_t* status) {
    if (ld_acquire_cta(p) > v) return true;
    const uint64_t t0 = global_ns();
    unsigned pause = 32;
    for (;;) {
        __nanosleep(pause);
        if (*reinterpret_cast<const volatile unsigned*>(p) > v) {
            __threadfence_block();
            return true;
        }
        if (pause < 256) pause *= 2;
        if (wait_timed_out(t0, status)) return false;
    }
}

// The first wait of a launch that gives up records where: words 4..6 of the
// status region hold (site, work unit, CTA).
enum { EX_SITE_PROD_UNIT = 1, EX_SITE_PROD_SLOT, EX_SITE_AUX_FREE, EX_SITE_CONS_UNIT, EX_SITE_CONS_SLOT,
       EX_SITE_PART };
__device__ __forceinline__ void note_site(uint32_t* status, bool ok, int site, int what) {
    if (ok) return;
    if (atomicCAS(status + 4, 0u, (uint32_t)site) == 0u) {
        status[5] = (uint32_t)what;
        status[6] = blockIdx.x;
    }
}

// One work unit's record in the per-CTA ring.
struct UnitView {
    int* meta;      // expert, item, slot k
    float* fw;      // weight w_k, 1 / input scale
    __half* xs;     // npad_h inputs, padded rows (kq_qtile.cuh PAD_ROW)
    float2* cx;     // [npad_h / 64]
};
__device__ __forceinline__ UnitView unit_view(uint8_t* sm, const ExParams& p, int slot) {
    uint8_t* b = sm + p.off_unit + (size_t)slot * p.unit_bytes;
    const int npad = p.nst_h * TILE_COLS;
    UnitView v;
    v.meta = reinterpret_cast<int*>(b);
    v.fw = reinterpret_cast<float*>(b + 16);
    v.xs = reinterpret_cast<__half*>(b + 32);
    v.cx = reinterpret_cast<float2*>(b + 32 + pad_bytes(npad));
    return v;
}

// Activations (fp32 in shared memory) -> fp16 x scale (padded rows) + per-group
// constants, by the nthr threads of rank 0..nthr-1 (whole warps).
template <int BITS>
__device__ __forceinline__ void stage_act_smem(const float* act, int n, int npad, float scale, int rank, int nthr,
                                               __half* xs, float2* cx) {
    const int nch = n / 8, npch = npad / 8;
    float offv[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) offv[k] = chunk_offset<BITS>(rank & 7, k);
    for (int c0 = 0; c0 < npch; c0 += nthr) {
        const int c = c0 + rank;
        // npch is a multiple of 64 and threads come in whole warps: the condition is warp-uniform
        if (c0 + (rank & ~31) < npch) {
            float v[8];
            if (c < nch) {
                const float4 a = *reinterpret_cast<const float4*>(act + (size_t)c * 8);
                const float4 b = *reinterpret_cast<const float4*>(act + (size_t)c * 8 + 4);
                v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
                v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
            } else {
#pragma unroll
                for (int k = 0; k < 8; ++k) v[k] = 0.f;
            }
            const float2 part = store_chunk_pad<BITS>(v, scale, offv, xs, c);
            group_reduce_store(part, rank, c, cx, 0xffffffffu);
        }
    }
}

__device__ __forceinline__ const uint8_t* expert_base(const ExParams& p, int item, int e) {
    const int l = p.layers ? p.layers[item] : p.layer;
    return p.base + (size_t)l * p.layer_bytes + (size_t)e * p.expert_bytes;
}

// Copies of consumer warp w in one unit.  Gate/up: each of its row tiles in
// runs of up to EX_CT column tiles.  Down: blocks of db row tiles (whole
// rows, db * nst_i <= EX_CT) or, when a row alone exceeds EX_CT tiles, each
// of its row tiles in runs like gate/up.
struct ExCopy {
    int ph, rt0, nrt, st0, nst;  // nrt row tiles x nst column tiles from column st0
};
__device__ __forceinline__ int ex_runs(int nst) { return (nst + EX_CT - 1) / EX_CT; }
__device__ __forceinline__ int ex_nrows(int n, int w, int cw) { return n > w ? (n - w - 1) / cw + 1 : 0; }
__device__ __forceinline__ int ex_ncopies(const ExParams& p, int w, int ph) {
    if (ph == 0) return ex_nrows(p.nrt_up, w, p.cw) * ex_runs(p.nst_h);
    const int nblk = (p.nrt_dn + p.db - 1) / p.db;
    return ex_nrows(nblk, w, p.cw) * (p.db > 1 ? 1 : ex_runs(p.nst_i));
}
__device__ __forceinline__ ExCopy ex_copy(const ExParams& p, int w, int ph, int i) {
    if (ph == 0 || p.db == 1) {
        const int nst = ph ? p.nst_i : p.nst_h, rr = ex_runs(nst);
        const int rt = w + (i / rr) * p.cw, st0 = (i % rr) * EX_CT;
        return {ph, rt, 1, st0, min(EX_CT, nst - st0)};
    }
    const int rt0 = (w + i * p.cw) * p.db;
    return {1, rt0, min(p.db, p.nrt_dn - rt0), 0, p.nst_i};
}

template <int BITS, int SB_DT>
__global__ void __launch_bounds__(EX_MAXTHREADS, 1) moe_expert_stream_kernel(const ExParams p) {
    extern __shared__ __align__(128) uint8_t sm[];
    constexpr int TB = TileT<BITS>::BYTES;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int c = blockIdx.x, P = gridDim.x, CW = p.cw;
    const int nunits_all = p.n * p.K;
    const int nunits = nunits_all > c ? (nunits_all - c - 1) / P + 1 : 0;  // this CTA's units
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + p.off_bar);  // [CW][EX_NW]
    unsigned* u_ready = reinterpret_cast<unsigned*>(full + CW * EX_NW);  // [EX_RW] unit published (t + 1)
    unsigned* u_free = u_ready + EX_RW;                                   // [EX_RW] unit released (t + 1)
    float* act = reinterpret_cast<float*>(sm + p.off_act);                // [I]
    __half* xd = reinterpret_cast<__half*>(sm + p.off_xd);                // npad_i, padded rows
    float2* cxd = reinterpret_cast<float2*>(sm + p.off_xd + pad_bytes(p.nst_i * TILE_COLS));
    const __half* zrow = reinterpret_cast<const __half*>(sm + p.off_misc);  // PAD_ROW zero bytes
    float* wmax = reinterpret_cast<float*>(sm + p.off_misc + 256);           // [EX_MAXCW] per-warp max |act|
    int* s_last = reinterpret_cast<int*>(wmax + EX_MAXCW);                   // this unit completes its item

    if (tid == 0) {
        for (int i = 0; i < CW * EX_NW; ++i) mbar_init(&full[i], 1);
        for (int i = 0; i < EX_RW; ++i) u_ready[i] = u_free[i] = 0u;
        fence_mbar_init();
    }
    if (tid < PAD_ROW / 4) reinterpret_cast<uint32_t*>(sm + p.off_misc)[tid] = 0u;
    __syncthreads();

    if (warp == EX_W_AUX) {
        // ---------------- units: routing and staged input ----------------
        const int npad = p.nst_h * TILE_COLS;
        for (int t = 0; t < nunits; ++t) {
            const int rs = t % EX_RW;
            if (lane == 0 && t >= EX_RW)
                note_site(p.status, wait_cta_above(&u_free[rs], (unsigned)(t - EX_RW), p.status), EX_SITE_AUX_FREE, t);
            __syncwarp();
            const int wu = c + t * P, j = wu / p.K, k = wu % p.K;
            const UnitView uv = unit_view(sm, p, rs);
            int ix = -1;
            float wt = 0.f;
            if (p.logits) {
                warp_topk_any(p.logits + (size_t)j * p.E, p.E, p.K, ix, wt);
            } else if (lane < p.K) {
                ix = __ldg(p.idx_in + (size_t)j * p.K + lane);
                wt = p.w_in ? __ldg(p.w_in + (size_t)j * p.K + lane) : 0.f;
            }
            if (k == 0 && lane < p.K) {  // the item's first unit publishes its routing
                if (p.idx_out) p.idx_out[(size_t)j * p.K + lane] = ix;
                if (p.w_out) p.w_out[(size_t)j * p.K + lane] = wt;
            }
            const int e = __shfl_sync(0xffffffffu, ix, k);
            const float w = __shfl_sync(0xffffffffu, wt, k);
            float mul = 1.f, inv = 1.f;
            if (p.norm_w || p.x_dtype != KQ_DT_F16) {  // RMSNorm and / or a power-of-two scale into fp16
                float am, ss;
                vec_stats(p.x, p.x_dtype, (size_t)j * p.H, p.H, p.norm_w, false, am, ss);
                const float rinv = p.norm_w ? rsqrtf(ss / (float)p.H + p.eps) : 1.f;
                const float sc = pow2_scale(am * rinv);
                mul = rinv * sc;
                inv = 1.f / sc;
            }
            stage_fused_pad<BITS, 8>(p.x, p.x_dtype, (size_t)j * p.H, p.H, npad, mul, false, lane, 32, uv.xs,
                                     uv.cx, p.norm_w);
            if (lane == 0) {
                uv.meta[0] = e;
                uv.meta[1] = j;
                uv.meta[2] = k;
                uv.fw[0] = w;
                uv.fw[1] = inv;
            }
            __syncwarp();
            if (lane == 0) st_release_cta(&u_ready[rs], (unsigned)(t + 1));
        }
    } else if (warp - EX_CW0 < CW) {
        // ---------------- consumers ----------------
        const int w = warp - EX_CW0;
        const int ctid = tid - EX_CW0 * 32;  // 0 .. CW * 32 - 1
        const int npad_i = p.nst_i * TILE_COLS;
        const int ncg = ex_ncopies(p, w, 0), ncd = ex_ncopies(p, w, 1);
        uint64_t* myfull = full + w * EX_NW;
        uint8_t* myslots = sm + (size_t)w * EX_NW * p.slot_bytes;
        // lane 0 issues this warp's copies in consumption order, EX_NW ahead
        const uint64_t pol = policy_evict_first();
        int issued = 0, done = 0;                // copies issued / consumed
        int it_t = 0, it_ph = 0, it_i = 0;       // next copy to issue
        const uint8_t* it_base = nullptr;        // its unit's expert
        int it_base_t = -1;
        auto it_norm = [&]() {  // past the last copy of a phase: next phase / unit
            while (it_t < nunits && it_i >= (it_ph ? ncd : ncg)) {
                it_i = 0;
                if (it_ph == 0) it_ph = 1;
                else {
                    it_ph = 0;
                    ++it_t;
                }
            }
        };
        auto try_issue = [&](bool block) -> bool {
            if (it_t >= nunits) return false;
            if (it_base_t != it_t) {
                const int rs = it_t % EX_RW;
                if (block) {
                    note_site(p.status, wait_cta_above(&u_ready[rs], (unsigned)it_t, p.status), EX_SITE_CONS_UNIT, it_t);
                } else if (ld_acquire_cta(&u_ready[rs]) <= (unsigned)it_t) {
                    return false;
                }
                const UnitView uv = unit_view(sm, p, rs);
                int e = uv.meta[0];
                if ((unsigned)e >= (unsigned)p.E) e = 0;  // outputs are zeroed
                it_base = expert_base(p, uv.meta[1], e);
                it_base_t = it_t;
            }
            const ExCopy cp = ex_copy(p, w, it_ph, it_i);
            const int nst = it_ph ? p.nst_i : p.nst_h;
            const uint8_t* src = it_base + (it_ph ? p.gateup_bytes : 0) + ((size_t)cp.rt0 * nst + cp.st0) * TB;
            const uint32_t bytes = (uint32_t)(cp.nrt * cp.nst * TB);
            const int s = issued % EX_NW;
            mbar_expect_tx(&myfull[s], bytes);
            bulk_g2s(myslots + (size_t)s * p.slot_bytes, src, bytes, &myfull[s], pol);
            ++issued;
            ++it_i;
            it_norm();
            return true;
        };
        it_norm();
        if (lane == 0 && try_issue(true))
            while (issued < EX_NW && try_issue(false)) {
            }
        __syncwarp();
        for (int t = 0; t < nunits; ++t) {
            const int rs = t % EX_RW;
            if (lane == 0) note_site(p.status, wait_cta_above(&u_ready[rs], (unsigned)t, p.status), EX_SITE_CONS_UNIT, t);
            __syncwarp();
            const UnitView uv = unit_view(sm, p, rs);
            const int e = uv.meta[0], j = uv.meta[1], kk = uv.meta[2];
            const float wk = uv.fw[0], xinv = uv.fw[1];
            const bool valid = (unsigned)e < (unsigned)p.E;
            const int ps = j % EX_RP;
            float* prow = p.part + ((size_t)ps * p.K + kk) * p.H;
            float m = 0.f, dinv = 1.f;
            for (int ph = 0; ph < 2; ++ph) {
                if (ph == 1) {
                    // gate/up complete: one scale for the unit's activations, staged to fp16
                    m = warp_max(m);
                    if (lane == 0) wmax[w] = m;
                    named_barrier_sync(EX_BAR, CW * 32);
                    if (ctid == 0) st_release_cta(&u_free[rs], (unsigned)(t + 1));  // input consumed
                    float am = 0.f;
                    for (int v = 0; v < CW; ++v) am = fmaxf(am, wmax[v]);
                    const float sc = pow2_scale(am);
                    dinv = 1.f / sc;
                    stage_act_smem<BITS>(act, p.I, npad_i, sc, ctid, CW * 32, xd, cxd);
                    // item j's partial-sum slot is free once the item RP before has been combined
                    if (ctid == 0 && p.out && j >= EX_RP)
                        note_site(p.status, wait_count(&p.pgen[ps], (unsigned)(j / EX_RP), p.status), EX_SITE_PART, j);
                    named_barrier_sync(EX_BAR, CW * 32);
                }
                const __half* xs = ph ? xd : uv.xs;
                const float2* cx = ph ? cxd : uv.cx;
                const int nst = ph ? p.nst_i : p.nst_h;
                const int ncp = ph ? ncd : ncg;
                float y0 = 0.f, y1 = 0.f;  // running sums of the current row tile
                for (int i = 0; i < ncp; ++i) {
                    const ExCopy cp = ex_copy(p, w, ph, i);
                    if (lane == 0 && issued == done) try_issue(true);  // the copy needed now is of this unit
                    __syncwarp();
                    const int s = done % EX_NW;
                    note_site(p.status, mbar_wait(&myfull[s], (done / EX_NW) & 1, p.status), EX_SITE_CONS_SLOT, done);
                    const uint8_t* slot = myslots + (size_t)s * p.slot_bytes;
                    for (int r = 0; r < cp.nrt; ++r) {
                        for (int st = 0; st < cp.nst; ++st) {
                            TileRegs<BITS> R;
                            tile_load<BITS>(slot + ((size_t)r * cp.nst + st) * TB, R);
                            tile_compute_pad<BITS, SB_DT>(R, cp.st0 + st, xs, cx, zrow, y0, y1);
                        }
                        if (cp.st0 + cp.nst == nst) {  // the row tile is complete
                            float g = y0, u = y1;
                            quad_reduce(g, u);
                            y0 = y1 = 0.f;
                            const int rt = cp.rt0 + r;
                            if (ph == 0) {
                                const float a = valid ? activate(g * xinv, u * xinv, p.act_kind) : 0.f;
                                if ((lane & 3) == 0) act[rt * 8 + (lane >> 2)] = a;
                                m = fmaxf(m, fabsf(a));
                            } else {
                                g = valid ? g * dinv : 0.f;
                                u = valid ? u * dinv : 0.f;
                                if ((lane & 3) == 0) {
                                    const int row = rt * 16 + (lane >> 2);
                                    if (p.out_per_k) {
                                        const size_t o = ((size_t)j * p.K + kk) * p.H + row;
                                        store_from_float(p.out_per_k, p.out_dtype, o, g);
                                        store_from_float(p.out_per_k, p.out_dtype, o + 8, u);
                                    }
                                    if (p.out) {
                                        __stcg(prow + row, wk * g);
                                        __stcg(prow + row + 8, wk * u);
                                    }
                                }
                            }
                        }
                    }
                    ++done;
                    __syncwarp();  // the slot's tiles have been read and used
                    if (lane == 0)
                        while (issued < done + EX_NW && try_issue(false)) {
                        }
                }
            }
            if (!valid && ctid == 0) set_status(p.status, KQ_DEV_BAD_EXPERT);
            if (p.out) {
                // the last of the item's K units adds their partial rows in slot order
                __threadfence();
                named_barrier_sync(EX_BAR, CW * 32);
                if (ctid == 0) {
                    const unsigned dn = atomicAdd(&p.pcnt[ps], 1u) + 1;
                    *s_last = dn == (unsigned)p.K * (unsigned)(j / EX_RP + 1);
                }
                named_barrier_sync(EX_BAR, CW * 32);
                const bool last = *s_last != 0;
                if (last) {
                    __threadfence();  // acquire side of the other units' increments
                    for (int h = ctid; h < p.H; h += CW * 32) {
                        float acc = 0.f;
                        for (int q2 = 0; q2 < p.K; ++q2) acc += __ldcg(p.part + ((size_t)ps * p.K + q2) * p.H + h);
                        if (p.residual) acc = load_as_float(p.residual, p.out_dtype, (size_t)j * p.H + h) + acc;
                        store_from_float(p.out, p.out_dtype, (size_t)j * p.H + h, acc);
                    }
                    __threadfence();
                }
                named_barrier_sync(EX_BAR, CW * 32);  // s_last is read by every warp before it changes
                if (last && ctid == 0) st_release(&p.pgen[ps], (unsigned)(j / EX_RP + 1));
            }
        }
        if (lane == 0)  // copies still in flight (only after a wait gave up) land before the CTA exits
            for (int f = done; f < issued; ++f) mbar_drain(&myfull[f % EX_NW], (f / EX_NW) & 1);
    }
}

// Workspace: status region, counters (zeroed before each launch), partial sums.
struct ExWs {
    size_t status, pcnt, pgen, cnt_end, part, total;
};

static ExWs ex_ws_layout(const kq_table* t, int K) {
    auto al = [](size_t v) { return (v + 255) / 256 * 256; };
    ExWs L{};
    size_t o = 0;
    L.status = o;
    o += 256;
    L.pcnt = o;
    o += (size_t)EX_RP * 4;
    L.pgen = o;
    o += (size_t)EX_RP * 4;
    L.cnt_end = o;
    o = al(o);
    L.part = o;
    o = al(o + (size_t)EX_RP * K * t->d.hidden * 4);
    L.total = o;
    return L;
}

// Shared-memory layout and consumer warps (as many as fit, up to EX_MAXCW);
// false if not even four consumer warps fit.
static bool ex_smem_layout(const kq_table* t, ExParams& p, size_t* bytes) {
    auto a128 = [](size_t v) { return (v + 127) / 128 * 128; };
    p.db = t->nst_i <= EX_CT ? std::max(1, EX_CT / t->nst_i) : 1;
    const size_t nh = (size_t)t->nst_h * TILE_COLS, ni = (size_t)t->nst_i * TILE_COLS;
    const size_t slot = a128((size_t)EX_CT * t->tb);
    const size_t unit = a128(32 + pad_bytes((int)nh) + (nh / GS) * 8);
    const size_t actb = a128((size_t)t->d.inter * 4);
    const size_t xd = a128(pad_bytes((int)ni) + (ni / GS) * 8);
    const size_t misc = 384;  // zero row, per-warp maxima, flag
    const size_t fixed = (size_t)EX_RW * unit + actb + xd + misc;
    auto bars = [&](int cw) { return (size_t)cw * EX_NW * 8 + (size_t)2 * EX_RW * 4; };
    int cw = EX_MAXCW;
    while (cw >= 4 && (size_t)cw * EX_NW * slot + fixed + bars(cw) > EX_SMEM_MAX) --cw;
    if (cw < 4) return false;
    p.cw = cw;
    p.slot_bytes = (uint32_t)slot;
    p.unit_bytes = (uint32_t)unit;
    p.off_unit = (uint32_t)(cw * EX_NW * slot);
    p.off_act = p.off_unit + (uint32_t)(EX_RW * unit);
    p.off_xd = p.off_act + (uint32_t)actb;
    p.off_misc = p.off_xd + (uint32_t)xd;
    p.off_bar = p.off_misc + (uint32_t)misc;
    *bytes = p.off_bar + bars(cw);
    return true;
}

template <int BITS, int SB_DT>
static cudaError_t launch_ex_t(const ExParams& p, size_t smem, cudaStream_t s) {
    auto kern = moe_expert_stream_kernel<BITS, SB_DT>;
    cudaError_t err = raise_smem_limit(reinterpret_cast<const void*>(kern), smem);
    if (err != cudaSuccess) return err;
    int dev = 0, nsm = 0, per_sm = 0;
    if ((err = cudaGetDevice(&dev)) != cudaSuccess) return err;
    if ((err = cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return err;
    const int threads = (EX_CW0 + p.cw) * 32;
    if ((err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem)) != cudaSuccess)
        return err;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)nsm);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // partial-sum slots are reused across CTAs: all resident
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

static cudaError_t launch_ex(int bits, int sb, const ExParams& p, size_t smem, cudaStream_t s) {
    if (bits == 3)
        return sb == KQ_DT_F16 ? launch_ex_t<3, KQ_DT_F16>(p, smem, s) : launch_ex_t<3, KQ_DT_BF16>(p, smem, s);
    return sb == KQ_DT_F16 ? launch_ex_t<4, KQ_DT_F16>(p, smem, s) : launch_ex_t<4, KQ_DT_BF16>(p, smem, s);
}

static bool ex_dtype_ok(int d) { return d == KQ_DT_F16 || d == KQ_DT_BF16 || d == KQ_DT_F32; }

}  // namespace kq

using namespace kq;

extern "C" size_t kq_moe_decode_batch_workspace_size(const kq_table* t, int top_k) {
    if (!t || top_k <= 0 || top_k > EX_MAXK) return 0;
    return ex_ws_layout(t, top_k).total;
}

extern "C" int kq_moe_decode_batch(const kq_table* t, int n, const int32_t* layers, int layer, const void* x,
                                   int x_dtype, const float* logits, int32_t* idx, float* weights, int K,
                                   void* out_per_k, void* out, int out_dtype, const void* residual,
                                   const void* norm_w, float eps, void* workspace, size_t workspace_bytes,
                                   void* stream) {
    if (!t) return KQ_ERR_ARG;
    if (n < 0 || K <= 0 || K > EX_MAXK || K > t->d.num_experts) return KQ_ERR_ARG;
    if (!layers && (layer < 0 || layer >= t->d.num_layers)) return KQ_ERR_ARG;
    if (n == 0) return KQ_OK;
    if ((long)n * K >= (1L << 31)) return KQ_ERR_ARG;
    if (!x || !ex_dtype_ok(x_dtype) || !ex_dtype_ok(out_dtype)) return KQ_ERR_ARG;
    if (norm_w && x_dtype == KQ_DT_F32) return KQ_ERR_ARG;
    if (!logits && !idx) return KQ_ERR_ARG;
    if (out && !weights && !logits) return KQ_ERR_ARG;
    if (!out && !out_per_k) return KQ_ERR_ARG;
    if (logits && t->d.num_experts > 1024) return KQ_ERR_UNSUPPORTED;
    if (t->d.hidden % 16 || t->d.inter % 8) return KQ_ERR_UNSUPPORTED;
    if (!workspace) return KQ_ERR_WORKSPACE;
    const ExWs L = ex_ws_layout(t, K);
    if (workspace_bytes < L.total) return KQ_ERR_WORKSPACE;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    ExParams p{};
    p.base = t->base;
    p.layer_bytes = t->layer_bytes;
    p.expert_bytes = t->expert_bytes;
    p.gateup_bytes = t->gateup_bytes;
    p.E = t->d.num_experts;
    p.K = K;
    p.H = t->d.hidden;
    p.I = t->d.inter;
    p.nst_h = t->nst_h;
    p.nst_i = t->nst_i;
    p.nrt_up = t->i8;
    p.nrt_dn = t->h16;
    p.n = n;
    p.layers = layers;
    p.layer = layer;
    p.x = x;
    p.x_dtype = x_dtype;
    p.logits = logits;
    p.idx_in = logits ? nullptr : idx;
    p.w_in = logits ? nullptr : weights;
    p.idx_out = logits ? idx : nullptr;
    p.w_out = logits ? weights : nullptr;
    p.norm_w = norm_w;
    p.eps = eps;
    p.out = out;
    p.out_per_k = out_per_k;
    p.out_dtype = out_dtype;
    p.residual = residual;
    p.act_kind = t->d.activation;
    p.part = reinterpret_cast<float*>(ws + L.part);
    p.pcnt = reinterpret_cast<unsigned*>(ws + L.pcnt);
    p.pgen = reinterpret_cast<unsigned*>(ws + L.pgen);
    p.status = reinterpret_cast<uint32_t*>(ws + L.status);
    size_t smem = 0;
    if (!ex_smem_layout(t, p, &smem)) return KQ_ERR_UNSUPPORTED;
    if (cudaMemsetAsync(ws + L.pcnt, 0, L.cnt_end - L.pcnt, s) != cudaSuccess) return KQ_ERR_CUDA;
    if (cudaMemsetAsync(ws + L.status + 16, 0, 12, s) != cudaSuccess) return KQ_ERR_CUDA;  // wait-site record
    const cudaError_t e = launch_ex(t->d.bits, t->d.sb_dtype, p, smem, s);
    if (e != cudaSuccess) {
        fprintf(stderr, "[kq] decode batch launch failed: %s\n", cudaGetErrorString(e));
        return KQ_ERR_CUDA;
    }
    return KQ_OK;
}
