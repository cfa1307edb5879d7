// kq_common.cuh -- shared device helpers for the sm_100a kernels of libkq.
//
// Inline-PTX wrappers: mbarrier (bounded waits), cp.async.bulk (TMA bulk copy
// global -> shared), programmatic dependent launch, the m16n8k16 f16 MMA used
// as the dot-product engine of the dequant GEMV, and 16-bit float helpers.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "kq.h"

#ifndef KQ_WAIT_LIMIT
// upper bound on polls of one mbarrier phase (each try_wait already blocks
// for a hardware-defined time slice); reaching it latches KQ_DEV_WAIT_TIMEOUT
#define KQ_WAIT_LIMIT (1u << 22)
#endif

namespace kq {

// ---- status word -------------------------------------------------------------
__device__ __forceinline__ void set_status(uint32_t* status, uint32_t bit) {
    if (status) atomicOr(status, bit);
}

// ---- shared-memory address ----------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier -------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait: returns false (and latches the timeout bit) if the phase never
// completed within KQ_WAIT_LIMIT polls.  Once any wait of the launch has timed
// out (bit latched in *status), later waits return at once, so a stalled
// pipeline drains in one wait limit instead of one per stage.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* status) {
    for (uint32_t i = 0; i < KQ_WAIT_LIMIT; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 1023u) == 1023u && status &&
            (*reinterpret_cast<volatile uint32_t*>(status) & KQ_DEV_WAIT_TIMEOUT))
            return false;
    }
    set_status(status, KQ_DEV_WAIT_TIMEOUT);
    return false;
}

// try_wait that lets the hardware suspend the thread for up to `ns`
// nanoseconds; the thread resumes as soon as the phase completes.
__device__ __forceinline__ bool mbar_try_wait_hint(uint64_t* bar, uint32_t parity, uint32_t ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

#ifndef KQ_WAIT_NS
#define KQ_WAIT_NS 1000000000ull  // 1 s: a phase that takes longer latches KQ_DEV_WAIT_TIMEOUT
#endif

// Bounded wait for waits that are often long (pipeline roles of persistent
// kernels): sleeping try_wait instead of a hot poll, so waiting warps leave
// the issue slots to the working ones.  Bounded by KQ_WAIT_NS of wall time
// (%globaltimer); returns false, with the timeout bit latched, if exceeded,
// and at once if another wait of the launch already timed out.
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t* status) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (;;) {
        if (mbar_try_wait_hint(bar, parity, 200000u)) return true;
        if (status && (*reinterpret_cast<volatile uint32_t*>(status) & KQ_DEV_WAIT_TIMEOUT)) return false;
        if (global_ns() - t0 > KQ_WAIT_NS) {
            set_status(status, KQ_DEV_WAIT_TIMEOUT);
            return false;
        }
    }
}

#ifndef KQ_DRAIN_NS
#define KQ_DRAIN_NS 100000000ull  // 100 ms
#endif

// Exit-path wait for this thread's own asynchronous work (a TMA fill or an
// MMA commit) on a barrier: ignores the timeout latch, so a role that gave up
// early still lets its copies and MMAs finish before the CTA frees its shared
// and tensor memory.  Bounded by KQ_DRAIN_NS.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return;
    const uint64_t t0 = global_ns();
    while (!mbar_try_wait_hint(bar, parity, 100000u))
        if (global_ns() - t0 > KQ_DRAIN_NS) return;
}

// plain arrive (one count) on a shared-memory mbarrier
__device__ __forceinline__ void mbar_arrive_local(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// ---- TMA bulk copy (non-tensor): global -> shared, completion on an mbarrier ----
// dst, src 16-byte aligned, bytes a multiple of 16.  Streamed data: L2 evict-first.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// ---- programmatic dependent launch ---------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- MMA m16n8k16, f16 inputs, f32 accumulate -----------------------------------
__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                        uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ---- 16-bit helpers --------------------------------------------------------------
template <int SB_DT>
__device__ __forceinline__ float sb_lo(uint32_t v);  // low 16 bits as float
template <int SB_DT>
__device__ __forceinline__ float sb_hi(uint32_t v);  // high 16 bits as float

template <>
__device__ __forceinline__ float sb_lo<KQ_DT_F16>(uint32_t v) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(v & 0xFFFFu)));
}
template <>
__device__ __forceinline__ float sb_hi<KQ_DT_F16>(uint32_t v) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(v >> 16)));
}
template <>
__device__ __forceinline__ float sb_lo<KQ_DT_BF16>(uint32_t v) {
    return __uint_as_float(v << 16);
}
template <>
__device__ __forceinline__ float sb_hi<KQ_DT_BF16>(uint32_t v) {
    return __uint_as_float(v & 0xFFFF0000u);
}

__device__ __forceinline__ float load_as_float(const void* p, int dtype, size_t i) {
    if (dtype == KQ_DT_F16) return __half2float(reinterpret_cast<const __half*>(p)[i]);
    if (dtype == KQ_DT_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
    return reinterpret_cast<const float*>(p)[i];
}

__device__ __forceinline__ void store_from_float(void* p, int dtype, size_t i, float v) {
    if (dtype == KQ_DT_F16)
        reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
    else if (dtype == KQ_DT_BF16)
        reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
    else
        reinterpret_cast<float*>(p)[i] = v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

}  // namespace kq
