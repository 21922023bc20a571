// async.cuh -- asynchronous copies and mbarriers (sm_100a, CTA scope),
// shared by the GEMV and attention kernels.
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace slm {

// 16-byte global -> shared copy through the LSU (cp.async, L2 only).
__device__ __forceinline__ void cp_async16(void *smem_dst, const void *gsrc) {
    unsigned d = (unsigned)__cvta_generic_to_shared(smem_dst);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(d), "l"(gsrc));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// ---- mbarriers and bulk (TMA) copies ------------------------------------
__device__ __forceinline__ unsigned smem_addr(const void *p) {
    return (unsigned)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_addr(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_addr(bar)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_test(uint64_t *bar, unsigned parity) {
    unsigned ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Wait for phase `parity` of `bar`, giving up after ~1 s (2e9 cycles) or as
// soon as another thread of the CTA gave up (*abort set): on a timeout the
// thread sets *abort and the kernel's error flag, and returns false.
constexpr long long WAIT_LIMIT = 2000000000LL;
__device__ __forceinline__ bool mbar_wait_limit(uint64_t *bar, unsigned parity, volatile int *abort,
                                                int32_t *err, long long limit) {
    if (mbar_test(bar, parity)) return true;  // fast path: the phase is already complete
    const long long t0 = clock64();
    while (!mbar_test(bar, parity)) {
        if (*abort) return false;
        if (clock64() - t0 > limit) {
            *abort = 1;
            if (err) atomicExch(err, 3);
            return false;
        }
    }
    return true;
}
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, unsigned parity, volatile int *abort,
                                          int32_t *err) {
    return mbar_wait_limit(bar, parity, abort, err, WAIT_LIMIT);
}
// One row copy global -> shared through the TMA engine, completing bytes on bar.
__device__ __forceinline__ void bulk_copy(void *dst, const void *src, unsigned bytes,
                                          uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::
            "r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// One tile (box) of a 3-D tensor map global -> shared through the TMA
// engine, completing its bytes on bar.  x is a multiple of 4 floats (16 B).
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int x, int y, int z,
                                            uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4}], [%5];\n" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_addr(bar))
        : "memory");
}

// Hint: bring one tile (box) of a 3-D tensor map from global memory into L2,
// without a destination or a completion (no shared memory, nothing to wait on).
__device__ __forceinline__ void tma_prefetch_3d(const CUtensorMap *map, int x, int y, int z) {
    asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];\n" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(x), "r"(y), "r"(z)
                 : "memory");
}

// ---- programmatic dependent launch ---------------------------------------
// A kernel launched with the programmatic-serialization attribute may start
// while its predecessor in the stream is still running.  It runs only work
// that does not depend on the predecessor (constant weights, shared-memory
// set-up, data written two or more kernels back), then pdl_wait() (returns
// once the predecessor has completed and its writes are visible; a no-op for
// a normal launch), then pdl_release() so that its own successor may start.
// Releasing only after the wait keeps "two kernels back" complete whenever a
// successor starts.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_release() {
    asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}

// ---- thread-block clusters -------------------------------------------------
// This CTA's rank in its cluster, the address of a shared variable in CTA
// `rank` of the cluster, a load from / a store to such an address, and the
// cluster-wide barrier.  Every thread of every CTA of the cluster arrives once
// per barrier phase, then waits; arrive and wait alternate in each thread.
// The forms without .aligned let the threads of a warp reach them apart.
__device__ __forceinline__ unsigned cluster_rank() {
    unsigned r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ unsigned cluster_map(unsigned saddr, unsigned rank) {
    unsigned r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}
__device__ __forceinline__ float cluster_ld(unsigned addr) {
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}
__device__ __forceinline__ void cluster_st(unsigned addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n barrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
// arrive without ordering (only "this CTA is running"), arrive that publishes
// this thread's earlier stores, and the wait that sees every arrived thread's
__device__ __forceinline__ void cluster_arrive_relaxed() {
    asm volatile("barrier.cluster.arrive.relaxed;\n" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive.release;\n" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.acquire;\n" ::: "memory"); }

// `count` arrivals on an mbarrier at once.
__device__ __forceinline__ void mbar_arrive_cnt(uint64_t *bar, unsigned count) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// Shared-memory loads and stores at 32-bit shared-window addresses
// (smem_addr): no generic-address conversion per access.  The loads are
// volatile, so they keep their order with the mbarrier waits (also volatile)
// that make the data they read ready, while the arithmetic around them is
// free to move.
__device__ __forceinline__ float lds_f32(unsigned a) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ float2 lds_f32x2(unsigned a) {
    float2 v;
    asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ float4 lds_f32x4(unsigned a) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ void sts_f32(unsigned a, float v) {
    asm volatile("st.shared.f32 [%0], %1;" ::"r"(a), "f"(v) : "memory");
}
__device__ __forceinline__ void sts_f32x4(unsigned a, float4 v) {
    asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(a), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                 : "memory");
}

// Barrier `id` over `count` threads (whole warps), without a result.
__device__ __forceinline__ void named_bar_sync(int id, int count) {
    asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(count) : "memory");
}

// Named barrier `id` over `count` threads (whole warps) that also returns the
// OR of `pred` over them, so every participant takes the same branch after it.
__device__ __forceinline__ bool named_bar_or(int id, int count, bool pred) {
    int r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.s32 p, %1, 0;\n"
        " bar.red.or.pred q, %2, %3, p;\n selp.s32 %0, 1, 0, q;\n}\n"
        : "=r"(r)
        : "r"((int)pred), "r"(id), "r"(count)
        : "memory");
    return r != 0;
}

}  // namespace slm
