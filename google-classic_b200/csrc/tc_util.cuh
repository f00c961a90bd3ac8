// tc_util.cuh -- 5th-generation tensor core (tcgen05) building blocks shared
// by the prompt matmul (prefill.cu) and the prompt attention
// (prompt_attn.cu): fences, the 128-byte-swizzled K-major shared-memory
// layout and its descriptor, the f16 instruction descriptor, MMA issue,
// commit to an mbarrier, and TMEM loads.
#pragma once
#include "holo_common.cuh"

namespace holo_tc {

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// shared-memory descriptor of a K-major, 128-byte-swizzled operand: rows of
// 128 bytes, 8-row atoms 1024 bytes apart (SBO), 16-byte LBO, version 1
__device__ __forceinline__ uint64_t sw128_desc(const void *smem) {
    const uint32_t a = smem_addr(smem);
    return (uint64_t)((a >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// instruction descriptor: fp16 x fp16 -> fp32, both operands K-major, M x N
__host__ __device__ constexpr uint32_t tc_idesc_f16(int m, int n) {
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void tc_mma(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, bool acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        :: "r"(tmem_d), "l"(a), "l"(b), "r"(idesc), "r"((uint32_t)acc) : "memory");
}

// D (+)= A . B with A (M x 16 fp16, row m in TMEM lane m, two K values a
// 32-bit column, the lower K in the low half) read from TMEM, B from shared
// memory through its descriptor
__device__ __forceinline__ void tc_mma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t b, uint32_t idesc, bool acc) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
        :: "r"(tmem_d), "r"(tmem_a), "l"(b), "r"(idesc), "r"((uint32_t)acc) : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(smem_addr(bar)) : "memory");
}

// 16 consecutive fp32 columns of this warp's 32 TMEM lanes.  The load and
// its wait are one asm statement: tcgen05.ld writes the destination
// registers asynchronously, so the compiler must not see them as defined
// (and move or read them) before tcgen05.wait::ld has returned.
__device__ __forceinline__ void tc_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t"
        "tcgen05.wait::ld.sync.aligned;"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr)
        : "memory");
}

// 16 consecutive 32-bit columns of this warp's 32 TMEM lanes from registers,
// and the wait until they have landed, in one asm statement: tcgen05.st may
// read its source registers after it issues, so the compiler must not reuse
// them before tcgen05.wait::st has returned.
__device__ __forceinline__ void tc_st16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n\t"
        "tcgen05.wait::st.sync.aligned;"
        :: "r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
           "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}

// byte offset of element (row r, column c) of a [rows][64] fp16 tile in the
// 128-byte-swizzled K-major layout (16-byte chunk index XOR row mod 8)
__host__ __device__ __forceinline__ uint32_t sw128_off(int r, int c) {
    return (uint32_t)((r >> 3) * 1024 + (r & 7) * 128 + ((((c >> 3) ^ (r & 7)) & 7) << 4) + (c & 7) * 2);
}

// TMEM columns for this CTA (a power of two >= 32), written to *slot by the
// calling warp; tc_dealloc releases them (same warp, same count)
__device__ __forceinline__ void tc_alloc(uint32_t *slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_addr(slot)), "r"(ncols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tc_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(taddr), "r"(ncols) : "memory");
}

}  // namespace holo_tc
