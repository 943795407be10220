// Shared-memory pipeline primitives (mbarriers, 1-D TMA bulk copies) and
// the exact fixed-point dot product of the int8 GEMVs.
#pragma once

#include "sb_common.cuh"

namespace sb {

// Every spin on an mbarrier or a flag gives up after this long.
constexpr unsigned long long SB_WAIT_NS = 2000000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("{ .reg .b64 st; mbarrier.arrive.shared::cta.b64 st, [%0]; }" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("{ .reg .b64 st; mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1; }" ::"r"(bar), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Bounded wait for the phase with the given parity; false when it timed out.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    uint64_t t0 = 0;
    for (uint32_t it = 0;; it++) {
        uint32_t done;
        asm volatile(
            "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
            : "=r"(done)
            : "r"(bar), "r"(parity)
            : "memory");
        if (done) return true;
        if ((it & 63) == 0) {
            const uint64_t t = global_ns();
            if (it == 0) t0 = t;
            else if (t - t0 > SB_WAIT_NS) return false;
        }
    }
}
// 1-D bulk copy global -> shared, completion counted on an mbarrier.
__device__ __forceinline__ void tma_load_1d(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
                 "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

// L2 policy for data read once per pass (weights, KV rows): evict first, so
// the stream does not push out what is reused (code, activations, sums).
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
// tma_load_1d with an L2 cache policy.
__device__ __forceinline__ void tma_load_1d_hint(uint32_t dst, const void *src, uint32_t bytes, uint32_t bar,
                                                 uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            dst),
        "l"(src), "r"(bytes), "r"(bar), "l"(policy)
        : "memory");
}

// Named barrier over the first N threads of the block (the consumer warps).
template <int N>
__device__ __forceinline__ void named_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(N) : "memory");
}

// Activation fixed point: a = A0 + 2^8 A1 + 2^16 A2 with A0, A1 unsigned
// bytes and A2 a signed byte; dot16 accumulates the three byte planes of 16
// consecutive k against 16 int8 weights (one uint4) with dp4a.
__device__ __forceinline__ long long combine_planes(int a0, int a1, int a2) {
    return (long long)a0 + ((long long)a1 << 8) + ((long long)a2 << 16);
}

__device__ __forceinline__ void dot16(const uint4 &w, const uint4 &p0, const uint4 &p1, const uint4 &p2, int &a0,
                                      int &a1, int &a2) {
    a0 = dp4a_su(w.x, p0.x, a0);
    a0 = dp4a_su(w.y, p0.y, a0);
    a0 = dp4a_su(w.z, p0.z, a0);
    a0 = dp4a_su(w.w, p0.w, a0);
    a1 = dp4a_su(w.x, p1.x, a1);
    a1 = dp4a_su(w.y, p1.y, a1);
    a1 = dp4a_su(w.z, p1.z, a1);
    a1 = dp4a_su(w.w, p1.w, a1);
    a2 = dp4a_ss(w.x, p2.x, a2);
    a2 = dp4a_ss(w.y, p2.y, a2);
    a2 = dp4a_ss(w.z, p2.z, a2);
    a2 = dp4a_ss(w.w, p2.w, a2);
}

// Output of an exact int64 column sum t: y = (f32)(t * f) with the f64
// factor f = 2^-shift * scale * rstd computed once per column kind.  The
// int64 -> f64 conversion adds t into the mantissa of 1.5 * 2^52 (exact for
// |t| < 2^51; column sums stay below 2^43), which keeps the per-element
// work off the conversion unit.
__device__ __forceinline__ double pow2_neg(int s) { return __longlong_as_double((long long)(1023 - s) << 52); }
__device__ __forceinline__ double gemv_factor(int shift, float scale, double rstd) {
    return pow2_neg(shift) * (double)scale * rstd;
}
__device__ __forceinline__ double i64_to_f64(long long t) {
    return __longlong_as_double(0x4338000000000000LL + t) - 6755399441055744.0;
}
__device__ __forceinline__ float gemv_out(long long t, double f) { return (float)(i64_to_f64(t) * f); }

}  // namespace sb
