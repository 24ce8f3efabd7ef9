// tc.cuh — 5th-generation tensor core (tcgen05) building blocks for sm_100a:
// TMEM allocation, UMMA shared-memory / instruction descriptors, the MMA issue,
// its commit to an mbarrier, and TMEM -> register loads.  Field layouts follow
// the PTX ISA's tcgen05 matrix-descriptor and instruction-descriptor formats.
#pragma once
#include "common.cuh"

namespace llmdiy {

// ---------------- TMEM allocation (one full warp) ----------------
LLMDIY_DEV void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
                 "r"(ncols)
                 : "memory");
}
LLMDIY_DEV void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::); }
LLMDIY_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
LLMDIY_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
LLMDIY_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// ---------------- descriptors ----------------
// Shared-memory matrix descriptor, K-major operand staged by a TMA load with
// 128-byte swizzling: rows of 64 fp16 (128 B) at a 128-byte pitch, 8-row
// groups 1024 B apart (SBO), leading offset unused for this layout (1),
// descriptor version 1, layout type 2 (SWIZZLE_128B).  `addr` is the shared
// address of the tile (1024-byte aligned) plus the K offset in bytes.
LLMDIY_DEV uint64_t umma_desc_sw128(uint32_t addr) {
    uint64_t d = 0;
    d |= (uint64_t)((addr & 0x3FFFFu) >> 4);
    d |= (uint64_t)1 << 16;             // leading byte offset (16 B >> 4)
    d |= (uint64_t)(1024 >> 4) << 32;   // stride byte offset
    d |= (uint64_t)1 << 46;             // version
    d |= (uint64_t)2 << 61;             // SWIZZLE_128B
    return d;
}
// Shared-memory matrix descriptor of an MN-major operand staged with 128-byte
// swizzling: atoms of 64 MN-elements x 8 K-rows (1024 B); `lbo` = bytes
// between atoms adjacent in MN, `sbo` = bytes between the 8-row K groups.
LLMDIY_DEV uint64_t umma_desc_sw128_mn(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((addr & 0x3FFFFu) >> 4);
    d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}
// Instruction descriptor of kind::f16 with fp16 A (K-major) and B (K-major, or
// MN-major when b_mn), fp32 accumulator of M x N.
__host__ __device__ constexpr uint32_t umma_idesc_f16_f32(int M, int N, bool b_mn = false) {
    return (1u << 4)                          // D format: f32
           | (0u << 7) | (0u << 10)           // A, B format: f16
           | (0u << 15)                       // A K-major
           | ((b_mn ? 1u : 0u) << 16)         // B major-ness
           | ((uint32_t)(N >> 3) << 17)       // N / 8
           | ((uint32_t)(M >> 4) << 24);      // M / 16
}

// ---------------- MMA issue (one thread) ----------------
// D[tmem] (+)= A[smem] * B[smem]^T, 128 x N x 16 per instruction.
LLMDIY_DEV void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}\n"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}
// As umma_f16 with the A operand in TMEM (M rows in lanes, K elements packed two 16-bit values per
// 32-bit column: a K = 16 step spans 8 columns starting at `tmem_a`).
LLMDIY_DEV void umma_f16_tmem_a(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}\n"
        ::"r"(tmem_d), "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}

// Arrive on `bar` once every MMA this thread issued so far has completed.
LLMDIY_DEV void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// ---------------- TMEM -> registers ----------------
// Warp w reads TMEM lanes 32w..32w+31 (thread t: lane 32w+t), 16 consecutive
// 32-bit columns starting at column `col` of the allocation at `base`.
LLMDIY_DEV void tmem_ld16(uint32_t taddr, uint32_t* r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
LLMDIY_DEV void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// registers -> TMEM, the same 32-lane x 16-column shape as tmem_ld16.
LLMDIY_DEV void tmem_st16(uint32_t taddr, const uint32_t* r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
        ::"r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
          "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}
LLMDIY_DEV void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

}  // namespace llmdiy
