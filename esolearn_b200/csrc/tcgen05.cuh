// 5th-generation tensor-core helpers (tcgen05, cta_group::1) shared by the
// batched int8 GEMM (qgemm.cu) and the persistent decode step.
//
// Shared-memory operands use the K-major, no-swizzle canonical layout: a core
// matrix is 8 rows x 16 bytes stored contiguously (rows 16 B apart); LBO is
// the byte distance between core matrices along K, SBO between 8-row groups.
#pragma once

#include "pipeline.cuh"

namespace sb {

__device__ __forceinline__ uint64_t umma_sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    // start, LBO and SBO in 16-byte units; descriptor version 1 (bit 46); no swizzle
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | ((uint64_t)1 << 46);
}
// Instruction descriptor of kind::i8 with an s32 accumulator, M = m, N = n,
// both operands K-major; a_signed / b_signed pick s8 (1) or u8 (0).
__device__ __forceinline__ uint32_t umma_idesc_i8(int m, int n, int a_signed, int b_signed) {
    return (2u << 4) | ((uint32_t)a_signed << 7) | ((uint32_t)b_signed << 10) | ((uint32_t)(n >> 3) << 17) |
           ((uint32_t)(m >> 4) << 24);
}
// D[tmem] (+)= A[da] . B[db]^T, issued by one thread.
__device__ __forceinline__ void umma_i8(uint32_t tmem, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
    asm volatile("{ .reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p; }" ::"r"(
                     tmem),
                 "l"(da), "l"(db), "r"(idesc), "r"(acc)
                 : "memory");
}
// The mbarrier at `bar` receives one arrival once every tcgen05 operation
// this thread issued before has completed.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
// Generic-proxy shared-memory writes made visible to the async proxy (the
// tensor core reading an operand this thread wrote with st.shared).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t *r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, uint32_t *r) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(taddr));
}

// Wait for this thread's tcgen05.ld results, then pass the registers
// through an empty asm so no use of them can be scheduled before the wait
// (the loads write their registers asynchronously).
template <int N>
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&d)[N]) {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < N; i++) asm volatile("" : "+r"(d[i]));
}

// TMEM allocation of ncols columns (a power of two >= 32) by one full warp;
// the base address lands in *dst (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t *dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

}  // namespace sb
