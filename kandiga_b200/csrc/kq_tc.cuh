// kq_tc.cuh -- 5th-generation tensor core (tcgen05) building blocks for sm_100a.
//
// Operand staging follows the K-major, 128-byte-swizzled shared-memory layout:
// a tile of R rows x 64 16-bit elements (128 B per row) is R/8 atoms of
// 8 rows x 128 B (1 KB, 1024-byte aligned); inside an atom, 16-byte chunk c of
// row r sits at chunk position c ^ (r % 8).  Operands longer than 64 elements
// along K are stored as consecutive [R x 128 B] blocks, one per 64-element
// K-chunk.  The MMA for the K-slice s (16 elements) of a chunk starts 32*s
// bytes into the chunk's block.
//
// Shared-memory matrix descriptor (64 bits): start address >> 4 in bits 0-13,
// leading-dimension byte offset >> 4 in 16-29 (unused by swizzled K-major
// layouts), stride byte offset >> 4 in 32-45 (1024 B between 8-row atoms),
// descriptor version 1 in 46-47, layout type in 61-63 (2 = 128-byte swizzle).
//
// Instruction descriptor for kind::f16 (32 bits): D format in bits 4-5
// (1 = f32), A format 7-9 and B format 10-12 (0 = f16, 1 = bf16), A/B major
// in bits 15/16 (0 = K-major), N >> 3 in bits 17-22, M >> 4 in bits 24-28.
#pragma once

#include "kq_common.cuh"

namespace kq {
namespace tc {

// byte offset of 16-bit element (r, k), k < 64, inside a swizzled [rows x 128 B] block
__host__ __device__ __forceinline__ uint32_t sw128_offset(int r, int k) {
    return (uint32_t)(r * 128 + (((k >> 3) ^ (r & 7)) << 4) + ((k & 7) << 1));
}

__device__ __forceinline__ uint64_t smem_desc_sw128(const void* base) {
    const uint64_t addr = (uint64_t)(smem_u32(base) >> 4) & 0x3FFFull;
    const uint64_t lbo = 1ull;          // 16 B (unused for swizzled K-major)
    const uint64_t sbo = 1024ull >> 4;  // 8-row atoms are 1 KB apart
    return addr | (lbo << 16) | (sbo << 32) | (1ull << 46) | (2ull << 61);
}

// advance a descriptor's start address by `bytes` (multiple of 16)
__device__ __forceinline__ uint64_t desc_advance(uint64_t d, uint32_t bytes) {
    return d + (uint64_t)(bytes >> 4);
}

__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, bool bf16) {
    return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((uint32_t)(N >> 3) << 17) |
           ((uint32_t)(M >> 4) << 24);
}

// ---- tensor memory -----------------------------------------------------------------
// Whole warp: allocate `ncols` (power of two >= 32) columns; the TMEM address
// lands in *slot (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void fence_before_sync() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, one thread issues
__device__ __forceinline__ void mma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate ? 1u : 0u)
        : "memory");
}

// Warp-converged forms: the whole warp executes the instruction, predicated
// on `leader` (one lane).  Keeping the issuing warp converged lets the
// descriptors live in uniform registers, which the MMA issue rate depends on.
__device__ __forceinline__ void mma_f16_ss_warp(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                bool accumulate, uint32_t leader) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "setp.ne.b32 e, %5, 0;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate ? 1u : 0u), "r"(leader)
        : "memory");
}

__device__ __forceinline__ void mma_commit_warp(uint64_t* bar, uint32_t leader) {
    asm volatile(
        "{\n\t.reg .pred e;\n\t"
        "setp.ne.b32 e, %1, 0;\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(
            smem_u32(bar)),
        "r"(leader)
        : "memory");
}

// arrive on an mbarrier when all previously issued MMAs of this thread complete
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

// 32 lanes x 32 bits x 16 columns: thread t of warp w gets lane (32w + t), columns [col, col+16)
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

}  // namespace tc
}  // namespace kq

namespace kq {
namespace tc {

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// 2D tiled TMA load (tensor map in kernel-parameter space), completion on an mbarrier.
// x (innermost, elements) must be a multiple of 16 bytes' worth of elements.
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// same with an L2 cache policy (createpolicy)
__device__ __forceinline__ void tma_load_2d_hint(void* dst, const void* tmap, int x, int y, uint64_t* bar,
                                                 uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// 3D tiled TMA load with an L2 cache policy
__device__ __forceinline__ void tma_load_3d_hint(void* dst, const void* tmap, int x, int y, int z, uint64_t* bar,
                                                 uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}

}  // namespace tc
}  // namespace kq
