// Internal helpers shared by every translation unit of libscryb200.so.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <utility>

#include "sb_api.h"

namespace sb {

// Records the failure message for sb_last_error() on this thread.
int set_error(int code, const char *fmt, ...);

// Device properties cached per device.
struct DeviceProps {
    int sm_count = 0;
    int max_smem_optin = 0;
    int cc_major = 0, cc_minor = 0;
};
const DeviceProps &device_props();

#define SB_CUDA_TRY(expr)                                                                   \
    do {                                                                                    \
        cudaError_t _e = (expr);                                                            \
        if (_e != cudaSuccess)                                                              \
            return sb::set_error(SB_ERR_CUDA, "%s: %s (%s:%d)", #expr, cudaGetErrorString(_e), \
                                 __FILE__, __LINE__);                                       \
    } while (0)

#define SB_CHECK(cond, code, ...)                       \
    do {                                                \
        if (!(cond)) return sb::set_error(code, __VA_ARGS__); \
    } while (0)

#define SB_TRY(expr)                   \
    do {                               \
        int _s = (expr);               \
        if (_s != SB_OK) return _s;    \
    } while (0)

// Programmatic dependent launch: a kernel lets its dependent start early
// (only loads of immutable data may precede pdl_wait()), then waits until
// every prerequisite grid has completed and its writes are visible.
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// cudaLaunchKernelEx with the programmatic-serialization attribute.
template <typename... KArgs, typename... Args>
inline cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                          cudaStream_t st, bool pdl, Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Streaming 16-byte load that bypasses L1 (weights are read once per step).
__device__ __forceinline__ uint4 ldg_stream(const uint4 *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// 4-way int8 dot products with int32 accumulate.
__device__ __forceinline__ int dp4a_su(unsigned w_s8x4, unsigned a_u8x4, int c) {
    int d;
    asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(w_s8x4), "r"(a_u8x4), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_ss(unsigned w_s8x4, unsigned a_s8x4, int c) {
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(w_s8x4), "r"(a_s8x4), "r"(c));
    return d;
}

__device__ __forceinline__ float warp_sum_f(float v) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ double warp_max_d(double v) {
    for (int o = 16; o > 0; o >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_max_f(float v) {
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// silu_scalar (cpu.rs:1119-1122), evaluated in f64 like the reference.
__device__ __forceinline__ float silu_f64(float x) {
    double x64 = (double)x;
    return (float)(x64 / (1.0 + exp(-x64)));
}

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Raise a kernel's dynamic shared-memory limit to what the device allows
// next to the kernel's static shared memory (once per device and kernel).
template <typename K>
inline int allow_max_dynamic_smem(K kern, int *limit_out) {
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, kern);
    if (e != cudaSuccess) return set_error(SB_ERR_CUDA, "cudaFuncGetAttributes: %s", cudaGetErrorString(e));
    const int limit = device_props().max_smem_optin - (int)fa.sharedSizeBytes;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, limit);
    if (e != cudaSuccess) return set_error(SB_ERR_CUDA, "cudaFuncSetAttribute(%d): %s", limit, cudaGetErrorString(e));
    if (limit_out) *limit_out = limit;
    return SB_OK;
}
inline int ceil_div(int a, int b) { return (a + b - 1) / b; }

}  // namespace sb
