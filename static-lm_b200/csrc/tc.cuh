// tc.cuh -- 5th-generation tensor core (tcgen05) helpers for sm_100a: TMEM
// allocation, kind::tf32 MMA on shared-memory operands, completion through an
// mbarrier, TMEM loads and the fences that order them with thread barriers.
#pragma once

#include "async.cuh"

namespace slm {

// Byte offset of element (r, k) in a K-major operand of R rows in the 128-byte
// swizzled canonical layout: the K extent is cut into atoms of 32 f32 (128 B),
// atom kb holds R rows of 128 B at kb*R*128, and the 16-byte chunk c of row r
// is stored at chunk c ^ (r & 7).  R is a multiple of 8; every atom's base is
// 1024-byte aligned when the operand's base is.
__device__ __forceinline__ unsigned sw128_off(int r, int k, int R) {
    const int kb = k >> 5, c = (k & 31) >> 2;
    return (unsigned)(kb * R * 128 + r * 128 + ((c ^ (r & 7)) << 4) + ((k & 3) << 2));
}

// Shared-memory matrix descriptor of such an operand: start address >> 4,
// leading byte offset 1 (unused by swizzled K-major layouts), stride byte
// offset 1024 B between groups of 8 rows, descriptor version 1, layout
// SWIZZLE_128B.  The K step of a kind::tf32 MMA is 8 elements = 32 B, taken
// inside an atom by adding 32 B to the start address.
__device__ __forceinline__ uint64_t umma_desc_sw128(unsigned saddr) {
    uint64_t d = (uint64_t)((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t)1u << 16;
    d |= (uint64_t)(1024u >> 4) << 32;
    d |= (uint64_t)1u << 46;
    d |= (uint64_t)2u << 61;
    return d;
}

// Instruction descriptor: f32 accumulator (bits 4-5 = 1), tf32 A and B (bits
// 7-9, 10-12 = 2), both K-major (bits 15, 16 = 0), N >> 3 at bit 17, M >> 4
// at bit 24.
__host__ __device__ constexpr unsigned umma_idesc_tf32(int M, int N) {
    return (1u << 4) | (2u << 7) | (2u << 10) | ((unsigned)(N >> 3) << 17) | ((unsigned)(M >> 4) << 24);
}

// D[M x N] (+)= A[M x K=8] . B[N x K=8]^T, issued by one thread.
__device__ __forceinline__ void tc_mma_tf32(unsigned d_tmem, uint64_t adesc, uint64_t bdesc,
                                            unsigned idesc, bool accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"((unsigned)accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}

// Instruction descriptor of kind::i8: s32 accumulator (bits 4-5 = 2), signed
// 8-bit A and B (bits 7-9, 10-12 = 1), both K-major, N >> 3 at bit 17, M >> 4
// at bit 24.  The K of one MMA is 32 elements (32 bytes).
__host__ __device__ constexpr unsigned umma_idesc_s8(int M, int N) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((unsigned)(N >> 3) << 17) | ((unsigned)(M >> 4) << 24);
}

// D[M x N] (+)= A[M x K=32] . B[N x K=32]^T over signed 8-bit operands into
// s32 TMEM, issued by one thread.
__device__ __forceinline__ void tc_mma_s8(unsigned d_tmem, uint64_t adesc, uint64_t bdesc, unsigned idesc,
                                          bool accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"((unsigned)accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}

// Arrive once on `bar` when every MMA this thread issued so far has completed.
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
                     smem_addr(bar))
                 : "memory");
}

// Warp-wide: allocate `ncols` TMEM columns (power of two >= 32), address to *dst.
__device__ __forceinline__ void tc_alloc(unsigned *dst, unsigned ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_addr(dst)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}
// Warp-wide: free the columns.
__device__ __forceinline__ void tc_dealloc(unsigned taddr, unsigned ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
}
// Generic-proxy writes to shared memory become visible to the tensor core.
__device__ __forceinline__ void fence_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}

// Warp-wide: 32 consecutive f32 columns of this thread's TMEM lane (lane
// field of taddr = 32 * (warp % 4)), waited for.
__device__ __forceinline__ void tc_ld32(unsigned taddr, float (&v)[32]) {
    unsigned r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
          "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
          "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
          "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
#pragma unroll
    for (int j = 0; j < 32; j++) v[j] = __uint_as_float(r[j]);
}

// Warp-wide: 32 / 16 consecutive 32-bit columns of this thread's TMEM lane as
// raw bits (s32 accumulators), waited for.
__device__ __forceinline__ void tc_ld32_u32(unsigned taddr, unsigned (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
          "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
          "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
          "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tc_ld16_u32(unsigned taddr, unsigned (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
          "=r"(r[15])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
}

// 3xTF32: x = hi + lo with hi = x cut to tf32 (10 mantissa bits) and lo the
// exact f32 remainder; a.b ~ ah.bh + ah.bl + al.bh with ~2^-21 relative error.
__device__ __forceinline__ float tf32_hi(float x) {
    return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
}

}  // namespace slm
