// Embedding, argmax, standalone MathBackend ops, device quantizer and the
// seeded on-device weight generator.
#include "misc.cuh"

#include <cuda_fp16.h>

#include <algorithm>

namespace sb {

// ---------------------------------------------------------------------------
// embedding / argmax around the decode step

__global__ void embed_kernel(const float *__restrict__ embed, int h, int V, SeqState s, float *x) {
    pdl_launch_dependents();
    pdl_wait();
    const int b = blockIdx.x;
    const int pos = s.pos[b];
    int tok = (s.prompt_len && pos < s.prompt_len[b]) ? s.prompt[(size_t)b * s.max_prompt + pos] : s.tok[b];
    tok = min(max(tok, 0), V - 1);  // the reference asserts idx < vocab (cpu.rs:486-491)
    const float *src = embed + (size_t)tok * h;
    float *dst = x + (size_t)b * h;
    if ((h & 3) == 0) {  // rows are 16-byte aligned when h % 4 == 0
        const float4 *s4 = reinterpret_cast<const float4 *>(src);
        float4 *d4 = reinterpret_cast<float4 *>(dst);
        for (int i = threadIdx.x; i < h / 4; i += blockDim.x) d4[i] = __ldg(s4 + i);
    } else {
        for (int i = threadIdx.x; i < h; i += blockDim.x) dst[i] = src[i];
    }
}

int embed_launch(const float *embed, int h, int V, SeqState s, int B, float *x, cudaStream_t st, bool pdl) {
    SB_CUDA_TRY(launch(embed_kernel, dim3(B), dim3(1024), 0, st, pdl, embed, h, V, s, x));
    return SB_OK;
}

// (value, index) pair reduction: larger value wins; equal values -> larger index.
__device__ __forceinline__ void amax_merge(float &v, int &i, float ov, int oi) {
    if (oi < 0) return;
    if (i < 0 || ov > v || (ov == v && oi > i)) v = ov, i = oi;
}

__device__ void block_amax(float &v, int &i) {
    __shared__ float sv[32];
    __shared__ int si[32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, i, o);
        amax_merge(v, i, ov, oi);
    }
    if (lane == 0) sv[warp] = v, si[warp] = i;
    __syncthreads();
    if (warp == 0) {
        const int nw = blockDim.x >> 5;
        v = lane < nw ? sv[lane] : -INFINITY;
        i = lane < nw ? si[lane] : -1;
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, v, o);
            const int oi = __shfl_xor_sync(0xffffffffu, i, o);
            amax_merge(v, i, ov, oi);
        }
    }
}

__global__ void argmax_step_kernel(const float *__restrict__ cv, const int *__restrict__ ci, int ntiles,
                                   SeqState s, int tp, int rank_stride, int idx_stride) {
    pdl_launch_dependents();
    pdl_wait();
    const int b = blockIdx.x;
    float v = -INFINITY;
    int idx = -1;
    for (int j = threadIdx.x; j < tp * ntiles; j += blockDim.x) {
        const int r = j / ntiles, t = j - r * ntiles;
        const size_t o = (size_t)r * rank_stride + (size_t)b * ntiles + t;
        const int i = ci[o];
        amax_merge(v, idx, cv[o], i < 0 ? i : i + r * idx_stride);
    }
    block_amax(v, idx);
    if (threadIdx.x == 0) {
        const int next = idx < 0 ? 0 : idx;
        const int pos = s.pos[b];
        const int plen = s.prompt_len ? s.prompt_len[b] : 0;
        s.last[b] = next;
        // generate.rs:72-75: sample after the last prompt token (a step at
        // position -1 is a graph capture's warm-up and records nothing)
        if (pos >= 0 && pos >= plen - 1) {
            const int g = s.ngen[b];
            if (g < s.max_gen) s.out[(size_t)b * s.max_gen + g] = next;
            s.ngen[b] = g + 1;
        }
        s.tok[b] = next;
        s.pos[b] = pos + 1;
    }
}

int argmax_step_launch(const float *cand_val, const int *cand_idx, int ntiles, SeqState s, int B,
                       cudaStream_t st, bool pdl, int tp, int rank_stride, int idx_stride) {
    SB_CUDA_TRY(launch(argmax_step_kernel, dim3(B), dim3(256), 0, st, pdl, cand_val, cand_idx, ntiles, s, tp,
                       rank_stride, idx_stride));
    return SB_OK;
}

// ---------------------------------------------------------------------------
// standalone ops

__global__ void rmsnorm_kernel(const float *__restrict__ x, const float *__restrict__ w, int d, float eps,
                               float *__restrict__ out) {
    // cpu.rs:574-599: f64 mean of squares, out = (f32)(x * rstd * w) in f64.
    __shared__ double sh[32];
    const float *xr = x + (size_t)blockIdx.x * d;
    double s = 0.0;
    for (int j = threadIdx.x; j < d; j += blockDim.x) s += (double)xr[j] * (double)xr[j];
    s = warp_sum_d(s);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) sh[warp] = s;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int i = 0; i < (int)(blockDim.x >> 5); i++) t += sh[i];
        sh[0] = 1.0 / sqrt(t / (double)d + (double)eps);
    }
    __syncthreads();
    const double rstd = sh[0];
    for (int j = threadIdx.x; j < d; j += blockDim.x)
        out[(size_t)blockIdx.x * d + j] = (float)(__dmul_rn(__dmul_rn((double)xr[j], rstd), (double)w[j]));
}

int rmsnorm_launch(const float *x, const float *w, int rows, int d, float eps, float *out, cudaStream_t st) {
    if (rows <= 0) return SB_OK;
    rmsnorm_kernel<<<rows, 256, 0, st>>>(x, w, d, eps, out);
    SB_CUDA_TRY(cudaGetLastError());
    return SB_OK;
}

__global__ void rope_kernel(const float *__restrict__ x, int seq, int n_heads, int hd, int start_pos,
                            const float *__restrict__ freqs, float scale, float *__restrict__ out) {
    // cpu.rs:635-664, then the trait-default scale (backend/mod.rs:219-230).
    const int half = hd / 2;
    const size_t total = (size_t)seq * n_heads * half;
    for (size_t t = blockIdx.x * (size_t)blockDim.x + threadIdx.x; t < total; t += (size_t)gridDim.x * blockDim.x) {
        const int i = (int)(t % half);
        const size_t sh = t / half;  // (s, h)
        const int s = (int)(sh / n_heads);
        const double angle = __dmul_rn((double)(start_pos + s), (double)freqs[i]);
        const float cs = (float)cos(angle), sn = (float)sin(angle);
        const size_t base = sh * hd + 2 * i;
        const float x0 = x[base], x1 = x[base + 1];
        const float o0 = __fsub_rn(__fmul_rn(x0, cs), __fmul_rn(x1, sn));
        const float o1 = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, cs));
        out[base] = __fmul_rn(o0, scale);
        out[base + 1] = __fmul_rn(o1, scale);
    }
}

int rope_launch(const float *x, int seq, int n_heads, int hd, int start_pos, const float *freqs, float scale,
                float *out, cudaStream_t st) {
    const size_t total = (size_t)seq * n_heads * (hd / 2);
    if (total == 0) return SB_OK;
    const int blocks = (int)std::min<size_t>((total + 255) / 256, 65535);
    rope_kernel<<<blocks, 256, 0, st>>>(x, seq, n_heads, hd, start_pos, freqs, scale, out);
    SB_CUDA_TRY(cudaGetLastError());
    return SB_OK;
}

__global__ void swiglu_kernel(const float *__restrict__ g, const float *__restrict__ u, size_t n,
                              float *__restrict__ out) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = __fmul_rn(silu_f64(g[i]), u[i]);  // cpu.rs:666-678
}

int swiglu_launch(const float *g, const float *u, size_t n, float *out, cudaStream_t st) {
    if (n == 0) return SB_OK;
    const int blocks = (int)std::min<size_t>((n + 255) / 256, 65535);
    swiglu_kernel<<<blocks, 256, 0, st>>>(g, u, n, out);
    SB_CUDA_TRY(cudaGetLastError());
    return SB_OK;
}

__global__ void argmax_rows_kernel(const float *__restrict__ x, int n, int *out) {
    float v = -INFINITY;
    int idx = -1;
    const float *xr = x + (size_t)blockIdx.x * n;
    for (int j = threadIdx.x; j < n; j += blockDim.x) amax_merge(v, idx, xr[j], j);
    block_amax(v, idx);
    if (threadIdx.x == 0) out[blockIdx.x] = idx < 0 ? 0 : idx;
}

int argmax_rows_launch(const float *x, int rows, int n, int *out, cudaStream_t st) {
    if (rows <= 0) return SB_OK;
    argmax_rows_kernel<<<rows, 1024, 0, st>>>(x, n, out);
    SB_CUDA_TRY(cudaGetLastError());
    return SB_OK;
}

// ---------------------------------------------------------------------------
// quantize_symmetric on device (quantize.rs:16-32)

__device__ __forceinline__ int8_t quant_one(float w, float inv) {
    const float r = roundf(__fmul_rn(w, inv));  // f32::round: half away from zero
    // f32::clamp keeps NaN and `as i8` maps it to 0 (a NaN weight, or every
    // weight once one is infinite: inv = 0 and inf * 0 = NaN)
    if (r != r) return 0;
    return (int8_t)fminf(fmaxf(r, -127.0f), 127.0f);
}

__global__ void absmax_kernel(const float *__restrict__ w, size_t n, unsigned *amax) {
    float m = 0.0f;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        m = fmaxf(m, fabsf(w[i]));
    m = warp_max_f(m);
    if ((threadIdx.x & 31) == 0) atomicMax(amax, __float_as_uint(m));  // non-negative floats order as uints
}

__global__ void quantize_kernel(const float *__restrict__ w, size_t n, const unsigned *amax, int8_t *q,
                                float *scale_out) {
    const float am = __uint_as_float(*amax);
    const float scale = am / 127.0f;   // f32 division (IEEE, no fast-math)
    const float inv = 1.0f / scale;
    if (blockIdx.x == 0 && threadIdx.x == 0) *scale_out = am == 0.0f ? 0.0f : scale;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        q[i] = am == 0.0f ? (int8_t)0 : quant_one(w[i], inv);
}

int quantize_device(const float *w, size_t n, int8_t *q, float *scale_dev, unsigned *amax, cudaStream_t st) {
    SB_CUDA_TRY(cudaMemsetAsync(amax, 0, sizeof(unsigned), st));
    const int blocks = (int)std::min<size_t>((n + 255) / 256, (size_t)device_props().sm_count * 8);
    if (n > 0) absmax_kernel<<<std::max(blocks, 1), 256, 0, st>>>(w, n, amax);
    quantize_kernel<<<std::max(blocks, 1), 256, 0, st>>>(w, n, amax, q, scale_dev);
    SB_CUDA_TRY(cudaGetLastError());
    return SB_OK;
}

// ---------------------------------------------------------------------------
// seeded weights: fastrand 2.3.0 wyrand + Box-Muller (nn/init.rs:2-14)
//
// The generator's state after d draws is seed + d*C0 (mod 2^64), so normal
// sample i (draws 2i+1 and 2i+2 of the stream) is computed independently.

constexpr uint64_t WY0 = 0x2d358dccaa6c78a5ULL;
constexpr uint64_t WY1 = 0x8bb84b93962eacc9ULL;

__device__ __forceinline__ uint64_t wy_mix(uint64_t s) {
    const uint64_t t = s ^ WY1;
    return (s * t) ^ __umul64hi(s, t);
}

__device__ __forceinline__ double unit_f64(uint64_t r) {
    return __longlong_as_double((long long)(0x3FF0000000000000ULL + (r >> 12))) - 1.0;
}

__device__ __forceinline__ float normal_at(uint64_t seed, uint64_t i) {
    const uint64_t s1 = seed + (2 * i + 1) * WY0;
    const uint64_t s2 = s1 + WY0;
    double u1 = unit_f64(wy_mix(s1));
    const double u2 = unit_f64(wy_mix(s2));
    if (u1 < 1e-30) u1 = 1e-30;
    const double z = __dmul_rn(sqrt(__dmul_rn(-2.0, log(u1))), cos(__dmul_rn(2.0 * 3.14159265358979323846, u2)));
    return (float)__dadd_rn(0.0, __dmul_rn((double)0.02f, z));  // mean 0, std 0.02 (llama.rs:599)
}

__device__ __forceinline__ float gen_value(const GenSpec &g, uint64_t seed, int r, int c) {
    if (g.src) return g.transposed ? g.src[(size_t)c * g.K + r] : g.src[(size_t)r * g.N + c];
    int i = 0;
    if (g.nseg > 1 && c >= g.c0[1]) i = 1;
    if (g.nseg > 2 && c >= g.c0[2]) i = 2;
    const int cc = c - g.c0[i];
    const uint64_t idx = g.transposed ? g.base[i] + (uint64_t)cc * g.K + r : g.base[i] + (uint64_t)r * g.width[i] + cc;
    return normal_at(seed, idx);
}

__global__ void gen_absmax_kernel(GenSpec g, uint64_t seed, unsigned *amax) {
    const size_t n = (size_t)g.K * g.N;
    float m = 0.0f;
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < n; e += (size_t)gridDim.x * blockDim.x)
        m = fmaxf(m, fabsf(gen_value(g, seed, (int)(e / g.N), (int)(e % g.N))));
    m = warp_max_f(m);
    if ((threadIdx.x & 31) == 0) atomicMax(amax, __float_as_uint(m));
}

__global__ void gen_quantize_kernel(GenSpec g, uint64_t seed, const unsigned *amax, int8_t *q, float *scale_out) {
    const float am = __uint_as_float(*amax);
    const float scale = am / 127.0f;
    const float inv = 1.0f / scale;
    if (blockIdx.x == 0 && threadIdx.x == 0) *scale_out = am == 0.0f ? 0.0f : scale;
    const size_t n = (size_t)g.K * g.N;
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < n; e += (size_t)gridDim.x * blockDim.x)
        q[e] = am == 0.0f ? (int8_t)0 : quant_one(gen_value(g, seed, (int)(e / g.N), (int)(e % g.N)), inv);
}

static int gen_blocks(size_t n) {
    return (int)std::max<size_t>(1, std::min<size_t>((n + 255) / 256, (size_t)device_props().sm_count * 16));
}

int gen_absmax(const GenSpec &g, uint64_t seed, unsigned *amax, cudaStream_t st) {
    SB_CUDA_TRY(cudaMemsetAsync(amax, 0, sizeof(unsigned), st));
    gen_absmax_kernel<<<gen_blocks((size_t)g.K * g.N), 256, 0, st>>>(g, seed, amax);
    SB_CUDA_TRY(cudaGetLastError());
    return SB_OK;
}

int gen_quantize(const GenSpec &g, uint64_t seed, const unsigned *amax, int8_t *q, float *scale_out,
                 cudaStream_t st) {
    gen_quantize_kernel<<<gen_blocks((size_t)g.K * g.N), 256, 0, st>>>(g, seed, amax, q, scale_out);
    SB_CUDA_TRY(cudaGetLastError());
    return SB_OK;
}

__global__ void gen_normal_kernel(uint64_t seed, uint64_t first, size_t n, float *out) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = normal_at(seed, first + i);
}

int gen_normal_f32(uint64_t seed, uint64_t first_sample, size_t n, float *out, cudaStream_t st) {
    gen_normal_kernel<<<gen_blocks(n), 256, 0, st>>>(seed, first_sample, n, out);
    SB_CUDA_TRY(cudaGetLastError());
    return SB_OK;
}

// ---------------------------------------------------------------------------
// checkpoint tensors (LlamaModel::from_safetensors, llama.rs:768-958): the
// F32 / BF16 / F16 -> f32 conversion (llama.rs:795-808, exact), the [out, in]
// -> [in, out] transpose (llama.rs:815-825) and the q|k|v concatenation
// (llama.rs:1009-1029) are folded into the index map of SrcSpec.

__device__ __forceinline__ float src_elem(const void *p, int dtype, long long i) {
    if (dtype == SB_DTYPE_BF16) return __uint_as_float((uint32_t)static_cast<const uint16_t *>(p)[i] << 16);
    if (dtype == SB_DTYPE_F16) return __half2float(static_cast<const __half *>(p)[i]);
    return static_cast<const float *>(p)[i];
}

__device__ __forceinline__ float src_value(const SrcSpec &g, int r, int c) {
    int i = 0;
    if (g.nseg > 1 && c >= g.c0[1]) i = 1;
    if (g.nseg > 2 && c >= g.c0[2]) i = 2;
    const long long row = g.row0[i] + (c - g.c0[i]);
    return src_elem(g.p[i], g.dtype, row * g.ld[i] + g.k0 + r);
}

__global__ void src_absmax_kernel(SrcSpec g, unsigned *amax) {
    const size_t n = (size_t)g.K * g.N;
    float m = 0.0f;
    // consecutive threads take consecutive k of one source row (coalesced)
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < n; e += (size_t)gridDim.x * blockDim.x)
        m = fmaxf(m, fabsf(src_value(g, (int)(e % g.K), (int)(e / g.K))));
    m = warp_max_f(m);
    if ((threadIdx.x & 31) == 0) atomicMax(amax, __float_as_uint(m));
}

__global__ void src_quantize_kernel(SrcSpec g, const unsigned *amax, int8_t *q, float *scale_out) {
    const float am = __uint_as_float(*amax);
    const float scale = am / 127.0f;
    const float inv = 1.0f / scale;
    if (blockIdx.x == 0 && threadIdx.x == 0) *scale_out = am == 0.0f ? 0.0f : scale;
    const size_t n = (size_t)g.K * g.N;
    // q is [N, K] (the source's row order): reads and writes both coalesced
    for (size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x; e < n; e += (size_t)gridDim.x * blockDim.x) {
        const int r = (int)(e % g.K), c = (int)(e / g.K);
        q[e] = am == 0.0f ? (int8_t)0 : quant_one(src_value(g, r, c), inv);
    }
}

int src_absmax(const SrcSpec &g, unsigned *amax, cudaStream_t st) {
    SB_CUDA_TRY(cudaMemsetAsync(amax, 0, sizeof(unsigned), st));
    src_absmax_kernel<<<gen_blocks((size_t)g.K * g.N), 256, 0, st>>>(g, amax);
    SB_CUDA_TRY(cudaGetLastError());
    return SB_OK;
}

int src_quantize(const SrcSpec &part, const unsigned *amax, int8_t *q, float *scale_out, cudaStream_t st) {
    src_quantize_kernel<<<gen_blocks((size_t)part.K * part.N), 256, 0, st>>>(part, amax, q, scale_out);
    SB_CUDA_TRY(cudaGetLastError());
    return SB_OK;
}

__global__ void src_to_f32_kernel(const void *src, int dtype, size_t n, float *out) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = src_elem(src, dtype, (long long)i);
}

int src_to_f32(const void *src, int dtype, size_t n, float *out, cudaStream_t st) {
    if (n == 0) return SB_OK;
    src_to_f32_kernel<<<gen_blocks(n), 256, 0, st>>>(src, dtype, n, out);
    SB_CUDA_TRY(cudaGetLastError());
    return SB_OK;
}

}  // namespace sb
