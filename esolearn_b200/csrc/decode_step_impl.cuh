// Device code of the persistent decode step, included by the four
// instantiation units (one per head_dim x KV-cache type) and compiled in
// parallel.  The design notes are in decode_step.cu.
//
// Code layout matters here: the kernel runs for a whole step, so every phase
// body exists once (the GEMV consumer loop and the residual input stage are
// out-of-line functions shared by all their call sites), and hot loops keep
// their state in registers with no 64-bit division per stage.
#pragma once

#include "decode_step.cuh"

#include <algorithm>

#include "pipeline.cuh"

namespace sb {
namespace {

extern __shared__ __align__(1024) uint8_t ds_smem[];

// Per-CTA state shared by the consumer warps.
struct DsShared {
    double red_d[8][2];
    float cand_v[8];
    int cand_i[8];
    double rstd;  // of the last GEMV input stage
    int shift;
    int abort;  // a bounded wait ran out: skip the rest of the step
    int last;
};
__shared__ DsShared ds_sh;

__device__ __forceinline__ void ds_sync() { named_sync<DS_CONSUMERS>(); }

// ---- small device helpers ---------------------------------------------------
__device__ __forceinline__ float4 ldcg4(const float *p) { return __ldcg(reinterpret_cast<const float4 *>(p)); }
__device__ __forceinline__ longlong2 ldcg_ll2(const long long *p) {
    return __ldcg(reinterpret_cast<const longlong2 *>(p));
}
__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
// CTA owning unit u when U units are split into G contiguous ranges
// [c*U/G, (c+1)*U/G).
// (U * G < 2^31 for every shape the step accepts.)
__device__ __forceinline__ int ds_owner(unsigned u, unsigned U, unsigned G) { return (int)(((u + 1) * G + U - 1) / U) - 1; }
__device__ __forceinline__ bool ds_empty(unsigned U, unsigned c, unsigned G) { return U * c / G == U * (c + 1) / G; }
// Pull n bytes at p into L2, the 128-byte lines spread over the CTAs:
// immutable vectors (norm weights, RoPE rows, the embedding row) that a
// later input stage reads, so that stage hits L2 instead of waiting for HBM
// behind the weight stream.
__device__ __forceinline__ void ds_prefetch_l2(const void *p, size_t n, int cta, int G) {
    const size_t lines = (n + 127) / 128;
    for (size_t li = (size_t)cta + (size_t)threadIdx.x * G; li < lines; li += (size_t)DS_CONSUMERS * G)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(static_cast<const char *>(p) + li * 128));
}

template <typename KV>
struct DsKv;
template <>
struct DsKv<__nv_bfloat16> {
    static constexpr int EPL = 8;
    __device__ static void load(const __nv_bfloat16 *p, float v[8]) {
        const uint4 u = *reinterpret_cast<const uint4 *>(p);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            v[2 * i] = __uint_as_float(w[i] << 16);
            v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
        }
    }
    __device__ static __nv_bfloat16 from(float f) { return __float2bfloat16_rn(f); }
    __device__ static float to(__nv_bfloat16 b) { return __bfloat162float(b); }
    // N consecutive elements (N = 2 or 4, 4- or 8-byte aligned) as floats.
    template <int N>
    __device__ static void load_n(const __nv_bfloat16 *p, float (&v)[N]) {
        if (N == 4) {
            const uint2 u = *reinterpret_cast<const uint2 *>(p);
            v[0] = __uint_as_float(u.x << 16), v[1] = __uint_as_float(u.x & 0xffff0000u);
            v[N > 2 ? 2 : 0] = __uint_as_float(u.y << 16), v[N > 3 ? 3 : 0] = __uint_as_float(u.y & 0xffff0000u);
        } else {
            const uint32_t u = *reinterpret_cast<const uint32_t *>(p);
            v[0] = __uint_as_float(u << 16), v[N > 1 ? 1 : 0] = __uint_as_float(u & 0xffff0000u);
        }
    }
};
template <>
struct DsKv<float> {
    static constexpr int EPL = 4;
    __device__ static void load(const float *p, float v[4]) {
        const float4 u = *reinterpret_cast<const float4 *>(p);
        v[0] = u.x, v[1] = u.y, v[2] = u.z, v[3] = u.w;
    }
    __device__ static float from(float f) { return f; }
    __device__ static float to(float f) { return f; }
    template <int N>
    __device__ static void load_n(const float *p, float (&v)[N]) {
        if (N == 4) {
            const float4 u = *reinterpret_cast<const float4 *>(p);
            v[0] = u.x, v[1] = u.y, v[N > 2 ? 2 : 0] = u.z, v[N > 3 ? 3 : 0] = u.w;
        } else {
            const float2 u = *reinterpret_cast<const float2 *>(p);
            v[0] = u.x, v[N > 1 ? 1 : 0] = u.y;
        }
    }
};

// ---- input stage -----------------------------------------------------------
// Every GEMV input stage leaves in ds_smem + pa_off the three fixed-point
// byte planes of its input row, and in ds_sh the row's exponent and rstd.
// Thread t owns quads t + 256 j, and every reduction order matches qgemv.cu's
// prologue for a single row, so planes, exponent and rstd are bit-identical
// to the per-kernel path.  v holds x*w (the norm-weighted row) and ssq the
// sum of squares of x.

template <int QMAX>
__device__ __forceinline__ void ds_quantize(const float4 (&v)[QMAX], float ssq, float amx, int K, int nq, bool norm,
                                            float eps, size_t pa_off) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    {
        const double s = warp_sum_d((double)ssq);
        const float mx = warp_max_f(amx);
        if (lane == 0) ds_sh.red_d[warp][0] = s, ds_sh.red_d[warp][1] = (double)mx;
    }
    ds_sync();
    if (tid == 0) {
        double s = 0.0, mx = 0.0;
        for (int w = 0; w < DS_CONSUMERS / 32; w++) s += ds_sh.red_d[w][0], mx = fmax(mx, ds_sh.red_d[w][1]);
        // rmsnorm (cpu.rs:582-588): mean of squares, rstd = 1/sqrt(mean+eps), f64.
        ds_sh.rstd = norm ? 1.0 / sqrt(s / (double)K + (double)eps) : 1.0;
        int e = 0;
        if (mx > 0.0) frexp(mx, &e);
        const int s2 = (mx > 0.0) ? 22 - e : 0;  // |a * 2^shift| < 2^22
        ds_sh.shift = s2 < -126 ? -126 : (s2 > 126 ? 126 : s2);
    }
    ds_sync();
    uint32_t *planes = reinterpret_cast<uint32_t *>(ds_smem + pa_off);
    const float sc = __int_as_float((ds_sh.shift + 127) << 23);  // 2^shift, exact
#pragma unroll
    for (int j = 0; j < QMAX; j++) {
        const int q = tid + j * DS_CONSUMERS;
        if (q >= nq) continue;
        const float xs4[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
        uint32_t w0 = 0, w1 = 0, w2 = 0;
#pragma unroll
        for (int i = 0; i < 4; i++) {
            // round to nearest even: |t| < 2^22, so t + 1.5*2^23 has ulp 1
            const float t = __fmul_rn(xs4[i], sc);
            const int A = __float_as_int(__fadd_rn(t, 12582912.0f)) - 0x4B400000;
            w0 |= (uint32_t)(A & 0xff) << (8 * i);
            w1 |= (uint32_t)((A >> 8) & 0xff) << (8 * i);
            w2 |= (uint32_t)((A >> 16) & 0xff) << (8 * i);
        }
        planes[0 * nq + q] = w0;
        planes[1 * nq + q] = w1;
        planes[2 * nq + q] = w2;
    }
    ds_sync();
}

__device__ __forceinline__ void ds_accum(float4 x, const float4 w, bool norm, float &ssq, float &amx, float4 &v) {
    if (norm) {
        ssq = fmaf(x.x, x.x, fmaf(x.y, x.y, fmaf(x.z, x.z, fmaf(x.w, x.w, ssq))));
        x = make_float4(__fmul_rn(x.x, w.x), __fmul_rn(x.y, w.y), __fmul_rn(x.z, w.z), __fmul_rn(x.w, w.w));
    }
    v = x;
    amx = fmaxf(amx, fmaxf(fmaxf(fabsf(x.x), fabsf(x.y)), fmaxf(fabsf(x.z), fabsf(x.w))));
}

// Input = a row in memory (embedding row: immutable; SwiGLU output: written
// by other CTAs in this step).  K % 4 == 0.  All loads issue before any use.
template <int QMAX>
__device__ __noinline__ void ds_in_rows(const float *row, bool immutable, const float *norm, int K, int KS,
                                           float eps, float *x_dst, size_t pa_off) {
    const int tid = threadIdx.x, nq = KS * 4;
    float4 v[QMAX], w[QMAX];
#pragma unroll
    for (int j = 0; j < QMAX; j++) {
        const int k0 = (tid + j * DS_CONSUMERS) * 4;
        v[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        w[j] = v[j];
        if (k0 < K) {
            v[j] = immutable ? __ldg(reinterpret_cast<const float4 *>(row + k0)) : ldcg4(row + k0);
            if (norm) w[j] = __ldg(reinterpret_cast<const float4 *>(norm + k0));
        }
    }
    if (x_dst) {
#pragma unroll
        for (int j = 0; j < QMAX; j++) {
            const int k0 = (tid + j * DS_CONSUMERS) * 4;
            if (k0 < K) *reinterpret_cast<float4 *>(x_dst + k0) = v[j];
        }
    }
    float ssq = 0.f, amx = 0.f;
#pragma unroll
    for (int j = 0; j < QMAX; j++) ds_accum(v[j], w[j], norm != nullptr, ssq, amx, v[j]);
    ds_quantize<QMAX>(v, ssq, amx, K, nq, norm != nullptr, eps, pa_off);
}

// Input = x + y(acc_prev): the residual add after a projection
// (llama.rs:564,568), then the fused RMSNorm.  x_dst (and trace) receive the
// new residual (CTA 0 passes them).  K % 4 == 0.  Loads go in batches of 4
// quads; within a batch all loads issue before any use.
template <int QMAX>
__device__ __noinline__ void ds_in_resid(const float *x_src, const long long *acc_prev, float scale_prev, int sh_prev,
                                         double rstd_prev, const float *norm, int K, int KS, float eps, float *x_dst,
                                         float *trace, size_t pa_off) {
    const int tid = threadIdx.x, nq = KS * 4;
    const double f = gemv_factor(sh_prev, scale_prev, rstd_prev);
    float4 v[QMAX];
    float ssq = 0.f, amx = 0.f;
#pragma unroll
    for (int j0 = 0; j0 < QMAX; j0 += 4) {
        float4 xb[4], wb[4];
        longlong2 ab[4][2];
#pragma unroll
        for (int jj = 0; jj < 4; jj++) {
            const int k0 = (tid + (j0 + jj) * DS_CONSUMERS) * 4;
            xb[jj] = make_float4(0.f, 0.f, 0.f, 0.f);
            wb[jj] = xb[jj];
            ab[jj][0] = ab[jj][1] = make_longlong2(0, 0);
            if (k0 < K) {
                xb[jj] = ldcg4(x_src + k0);
                ab[jj][0] = ldcg_ll2(acc_prev + k0);
                ab[jj][1] = ldcg_ll2(acc_prev + k0 + 2);
                if (norm) wb[jj] = __ldg(reinterpret_cast<const float4 *>(norm + k0));
            }
        }
#pragma unroll
        for (int jj = 0; jj < 4; jj++) {
            const int k0 = (tid + (j0 + jj) * DS_CONSUMERS) * 4;
            float4 x = xb[jj];
            if (k0 < K) {
                x.x = __fadd_rn(x.x, gemv_out(ab[jj][0].x, f));
                x.y = __fadd_rn(x.y, gemv_out(ab[jj][0].y, f));
                x.z = __fadd_rn(x.z, gemv_out(ab[jj][1].x, f));
                x.w = __fadd_rn(x.w, gemv_out(ab[jj][1].y, f));
                if (x_dst) *reinterpret_cast<float4 *>(x_dst + k0) = x;
                if (trace) *reinterpret_cast<float4 *>(trace + k0) = x;
            }
            ds_accum(x, wb[jj], norm != nullptr, ssq, amx, v[j0 + jj]);
        }
    }
    ds_quantize<QMAX>(v, ssq, amx, K, nq, norm != nullptr, eps, pa_off);
}

// Input stage after a tensor-parallel row projection (o or down): the
// residual x plus every rank's partial product, read from this rank's cells
// (cells + src * ld + k holds rank src's y_k, written with epoch e), waiting
// -- bounded -- for cells not yet written.  The ranks' values are added in
// rank order, (x + y_0) + y_1 + ..., so every rank gets the same bits.  Then
// RMSNorm and quantization as ds_in_resid.  Returns false when a wait ran
// out (the step is then abandoned).
template <int QMAX>
__device__ __noinline__ bool ds_in_resid_tp(const float *x_src, const uint2 *cells, int T, int ld, unsigned e,
                                            const float *norm, int K, int KS, float eps, float *x_dst, float *trace,
                                            size_t pa_off) {
    const int tid = threadIdx.x, nq = KS * 4;
    float4 v[QMAX];
    float ssq = 0.f, amx = 0.f;
    bool ok = true;
    uint64_t t0 = 0;
    uint32_t spins = 0;
#pragma unroll
    for (int j0 = 0; j0 < QMAX; j0 += 4) {
        // every load of four quads in flight together: x, the norm weight,
        // then one rank's 16 cells at a time (one round trip per rank)
        float4 xb[4], wb[4];
#pragma unroll
        for (int jj = 0; jj < 4; jj++) {
            const int k0 = (tid + (j0 + jj) * DS_CONSUMERS) * 4;
            xb[jj] = make_float4(0.f, 0.f, 0.f, 0.f);
            wb[jj] = xb[jj];
            if (k0 < K) {
                xb[jj] = ldcg4(x_src + k0);
                if (norm) wb[jj] = __ldg(reinterpret_cast<const float4 *>(norm + k0));
            }
        }
        // cells of two quads of two ranks per round trip (register budget);
        // the ranks' values are still added in rank order
#pragma unroll
        for (int jp = 0; jp < 4; jp += 2) {
            for (int r0 = 0; r0 < T; r0 += 2) {
                const int nr = min(2, T - r0);
                uint2 c[2][2][4];
#pragma unroll
                for (int rr = 0; rr < 2; rr++)
#pragma unroll
                    for (int u = 0; u < 2; u++) {
                        const int k0 = (tid + (j0 + jp + u) * DS_CONSUMERS) * 4;
#pragma unroll
                        for (int q = 0; q < 4; q++)
                            c[rr][u][q] = (rr < nr && k0 < K) ? ld_cell(cells + (size_t)(r0 + rr) * ld + k0 + q)
                                                              : make_uint2(0u, e);
                    }
                for (;;) {
                    bool all = true;
#pragma unroll
                    for (int rr = 0; rr < 2; rr++)
#pragma unroll
                        for (int u = 0; u < 2; u++)
#pragma unroll
                            for (int q = 0; q < 4; q++) all = all && c[rr][u][q].y == e;
                    if (all || !ok) break;
                    if ((spins++ & 63) == 0) {
                        const uint64_t t = global_ns();
                        if (t0 == 0) t0 = t;
                        else if (t - t0 > SB_WAIT_NS) ok = false;
                    }
#pragma unroll
                    for (int rr = 0; rr < 2; rr++)
#pragma unroll
                        for (int u = 0; u < 2; u++) {
                            const int k0 = (tid + (j0 + jp + u) * DS_CONSUMERS) * 4;
#pragma unroll
                            for (int q = 0; q < 4; q++)
                                if (c[rr][u][q].y != e) c[rr][u][q] = ld_cell(cells + (size_t)(r0 + rr) * ld + k0 + q);
                        }
                }
#pragma unroll
                for (int rr = 0; rr < 2; rr++) {
                    if (rr >= nr) break;
#pragma unroll
                    for (int u = 0; u < 2; u++) {
                        float4 &x = xb[jp + u];
                        x.x = __fadd_rn(x.x, __uint_as_float(c[rr][u][0].x));
                        x.y = __fadd_rn(x.y, __uint_as_float(c[rr][u][1].x));
                        x.z = __fadd_rn(x.z, __uint_as_float(c[rr][u][2].x));
                        x.w = __fadd_rn(x.w, __uint_as_float(c[rr][u][3].x));
                    }
                }
            }
        }
#pragma unroll
        for (int jj = 0; jj < 4; jj++) {
            const int k0 = (tid + (j0 + jj) * DS_CONSUMERS) * 4;
            if (k0 < K) {
                if (x_dst) *reinterpret_cast<float4 *>(x_dst + k0) = xb[jj];
                if (trace) *reinterpret_cast<float4 *>(trace + k0) = xb[jj];
            }
            ds_accum(xb[jj], wb[jj], norm != nullptr, ssq, amx, v[j0 + jj]);
        }
    }
    if (!ok) ds_sh.abort = 1;  // seen by the GEMV after the reductions below
    ds_quantize<QMAX>(v, ssq, amx, K, nq, norm != nullptr, eps, pa_off);
    return ok;
}

// Input = the attention output: each q head's partial records (one per CTA
// that worked on its kv head) combined in CTA order,
//   out = sum_c exp(m_c - M) o_c / sum_c exp(m_c - M) l_c,  M = max_c m_c.
// The (m, l) of all records first go to a table in shared memory (aliasing
// the planes, which are written only after the last read of the table).
template <int HD, int REP, int QMAX>
__device__ __forceinline__ void ds_in_att(const float *part, unsigned U, int nch, int G, int nh, int K, int KS,
                                          int rmax, size_t pa_off) {
    const int tid = threadIdx.x, nq = KS * 4;
    float *tab = reinterpret_cast<float *>(ds_smem + pa_off);  // [nh][rmax] (w, l), then [nh] sums
    float *lsum = tab + (size_t)2 * nh * rmax;
    for (int i = tid; i < nh * rmax; i += DS_CONSUMERS) {
        const int hq = i / rmax, k = i - hq * rmax;
        const int g = hq / REP, r = hq - g * REP;
        const unsigned ub = (unsigned)g * nch;
        const int c = ds_owner(ub, U, G) + k;
        float m = -INFINITY, l = 0.f;
        if (c <= ds_owner(ub + nch - 1, U, G) && !ds_empty(U, c, G)) {
            const float *rec = part + (((size_t)g * G + c) * REP + r) * DS_REC(HD);
            m = __ldcg(rec + HD);
            l = __ldcg(rec + HD + 1);
        }
        tab[2 * i] = m;
        tab[2 * i + 1] = l;
    }
    ds_sync();
    for (int hq = tid; hq < nh; hq += DS_CONSUMERS) {
        float *t = tab + (size_t)2 * hq * rmax;
        float M = -INFINITY;
        for (int k = 0; k < rmax; k++) M = fmaxf(M, t[2 * k]);
        float Ls = 0.f;
        for (int k = 0; k < rmax; k++) {
            const float mt = t[2 * k];
            const float w = mt == -INFINITY ? 0.f : expf(mt - M);
            Ls = fmaf(t[2 * k + 1], w, Ls);
            t[2 * k] = w;  // the record's weight
        }
        lsum[hq] = Ls;
    }
    ds_sync();
    // Each thread combines its QMAX quads; the loads of all its quads for
    // RCH records at a time are issued before any is used.
    constexpr int RCH = 3;
    float4 v[QMAX];
    float O[QMAX][4];
    const float *rec0[QMAX];
    const float *tq[QMAX];
#pragma unroll
    for (int j = 0; j < QMAX; j++) {
        const int k0 = (tid + j * DS_CONSUMERS) * 4;
        O[j][0] = O[j][1] = O[j][2] = O[j][3] = 0.f;
        rec0[j] = nullptr;
        tq[j] = tab;
        if (k0 < K) {
            const int hq = k0 / HD, d0 = k0 - hq * HD;
            const int g = hq / REP, r = hq - g * REP;
            const int cf = ds_owner((unsigned)g * nch, U, G);
            tq[j] = tab + (size_t)2 * hq * rmax;
            rec0[j] = part + (((size_t)g * G + cf) * REP + r) * DS_REC(HD) + d0;
        }
    }
    const size_t cstride = (size_t)REP * DS_REC(HD);
    for (int kb = 0; kb < rmax; kb += RCH) {
        float4 o[QMAX][RCH];
        float w[QMAX][RCH];
#pragma unroll
        for (int j = 0; j < QMAX; j++)
#pragma unroll
            for (int i = 0; i < RCH; i++) {
                w[j][i] = (rec0[j] && kb + i < rmax) ? tq[j][2 * (kb + i)] : 0.f;
                o[j][i] = w[j][i] != 0.f ? ldcg4(rec0[j] + (size_t)(kb + i) * cstride) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
        for (int j = 0; j < QMAX; j++)
#pragma unroll
            for (int i = 0; i < RCH; i++) {
                if (w[j][i] == 0.f) continue;
                O[j][0] = fmaf(o[j][i].x, w[j][i], O[j][0]);
                O[j][1] = fmaf(o[j][i].y, w[j][i], O[j][1]);
                O[j][2] = fmaf(o[j][i].z, w[j][i], O[j][2]);
                O[j][3] = fmaf(o[j][i].w, w[j][i], O[j][3]);
            }
    }
    float ssq = 0.f, amx = 0.f;
    const float4 one = make_float4(1.f, 1.f, 1.f, 1.f);
#pragma unroll
    for (int j = 0; j < QMAX; j++) {
        float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
        const int k0 = (tid + j * DS_CONSUMERS) * 4;
        if (k0 < K) {
            const float Ls = lsum[k0 / HD];
            if (Ls > 0.f) x = make_float4(O[j][0] / Ls, O[j][1] / Ls, O[j][2] / Ls, O[j][3] / Ls);
        }
        ds_accum(x, one, false, ssq, amx, v[j]);
    }
    ds_sync();  // the table is read; the planes may overwrite it
    ds_quantize<QMAX>(v, ssq, amx, K, nq, false, 0.f, pa_off);
}

// ---- GEMV consumer ------------------------------------------------------------
// The stages of one GEMV for CTA cta: its range [u0, u1) of the tile-major
// sequence of 16 KB units, grouped two units of one tile per stage (one at a
// tile edge).  The producer walks the same sequence.
struct DsWalk {
    int tile, ut, u, u1, upt, KS;
    __device__ DsWalk(int KS_, int ntiles, int G, int cta) : KS(KS_) {
        upt = (KS + DS_UNIT_KS - 1) / DS_UNIT_KS;
        const int U = ntiles * upt;
        u = (int)((long long)U * cta / G);
        u1 = (int)((long long)U * (cta + 1) / G);
        tile = u / upt;
        ut = u - tile * upt;
    }
    __device__ bool more() const { return u < u1; }
    // Current stage: first k-step and k-step count; then advance.
    __device__ void next(int &t, int &k0, int &nks) {
        const int n = (ut + 1 < upt && u + 1 < u1) ? 2 : 1;
        t = tile;
        k0 = ut * DS_UNIT_KS;
        nks = min(n * DS_UNIT_KS, KS - k0);
        u += n;
        ut += n;
        if (ut >= upt) ut = 0, tile++;
    }
};

// Consumes this CTA's stages of one GEMV and adds the exact column sums into
// out.  Returns the updated count of consumed ring stages.
__device__ __noinline__ uint32_t ds_gemv(uint32_t it, int nst, uint32_t bars, int KS, int ntiles, long long *out,
                                         int G, int cta, uint32_t pa_off, uint32_t red_off,
                                         unsigned long long *ready) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    DsWalk wk(KS, ntiles, G, cta);
    if (!wk.more()) return it;
    const uint4 *ring4 = reinterpret_cast<const uint4 *>(ds_smem);
    const uint4 *planes4 = reinterpret_cast<const uint4 *>(ds_smem + pa_off);
    long long *red = reinterpret_cast<long long *>(ds_smem + red_off);
    bool failed = ds_sh.abort != 0;
    uint32_t slot = it % nst, par = (it / nst) & 1;
    int acc[4][3];
#pragma unroll
    for (int j = 0; j < 4; j++) acc[j][0] = acc[j][1] = acc[j][2] = 0;
    auto flush = [&](int t) {
#pragma unroll
        for (int j = 0; j < 4; j++) {
            red[warp * DS_TN + lane + 32 * j] = combine_planes(acc[j][0], acc[j][1], acc[j][2]);
            acc[j][0] = acc[j][1] = acc[j][2] = 0;
        }
        ds_sync();
        if (tid < DS_TN && !failed) {
            long long s = 0;
#pragma unroll
            for (int w = 0; w < DS_CONSUMERS / 32; w++) s += red[w * DS_TN + tid];
            if (s != 0)
                atomicAdd(reinterpret_cast<unsigned long long *>(out + (size_t)t * DS_TN + tid), (unsigned long long)s);
        }
        ds_sync();
    };
    int cur = wk.tile;
#ifdef SB_STEP_TIMELINE
    bool first = true;
#else
    (void)ready;
#endif
    while (wk.more()) {
        int t, k0, nks;
        wk.next(t, k0, nks);
        if (t != cur) {
            flush(cur);
            cur = t;
        }
        if (!failed && !mbar_wait(bars + 8 * slot, par)) {
            failed = true;
            ds_sh.abort = 1;
        }
#ifdef SB_STEP_TIMELINE
        if (ready && tid == 0) {  // timeline: first and last weight stage ready
            const unsigned long long tn = global_ns();
            if (first) ready[0] = tn;
            ready[1] = tn;
        }
        first = false;
#endif
        if (!failed) {
            const uint4 *wst = ring4 + (size_t)slot * (DS_STAGE / 16) + warp * DS_TN + lane;
#pragma unroll
            for (int kk = 0; kk < DS_KPS / 8; kk++) {
                const int kl = warp + 8 * kk;
                if (kl < nks) {
                    const int ks = k0 + kl;
                    uint4 w[4];
#pragma unroll
                    for (int j = 0; j < 4; j++) w[j] = wst[kk * 8 * DS_TN + 32 * j];
                    const uint4 p0 = planes4[ks], p1 = planes4[KS + ks], p2 = planes4[2 * KS + ks];
#pragma unroll
                    for (int j = 0; j < 4; j++) dot16(w[j], p0, p1, p2, acc[j][0], acc[j][1], acc[j][2]);
                }
            }
        }
        __syncwarp();
        if (lane == 0 && !failed) mbar_arrive(bars + 8 * (nst + slot));
        if (++slot == (uint32_t)nst) slot = 0, par ^= 1;
        it++;
    }
    flush(cur);
    return it;
}

// ---- attention consumer -------------------------------------------------------
// Attention over this CTA's (kv head, chunk) units [u0, u1) of one layer, in
// the flash-decoding form: each warp owns rows w, w+8, ... of every chunk and
// keeps its own online-softmax state (m, l, o) per q head of the group, so
// scores, the running maximum and the weighted V sum need only warp
// shuffles (four rows per shuffle round); the eight warp states are merged
// once per head into the head's record.  Lane x holds dims
// [DPL*x, DPL*x + DPL) of q and o.  Out of line, so its state stays in
// registers.  Returns the updated count of consumed ring stages.
template <int HD, int REP, typename KV>
__device__ __noinline__ uint32_t ds_attention(uint32_t it, int nst, uint32_t bars, long long u0, long long u1, int nch,
                                              int ctx, int pos, bool has_new, const long long *accq, double fq,
                                              const float *cos_row, const float *sin_row, KV *kcl, KV *vcl,
                                              const int *page_table, float *part, int nkv, int q_dim, int kv_dim,
                                              int page_size, int chunk, float q_scale, int G, int cta,
                                              uint32_t qs_off, uint32_t kvnew_off, uint32_t pa_off) {
    using KL = DsKv<KV>;
    constexpr int DPL = HD / 32;  // dims per lane
    constexpr int BR = 4;         // rows per warp per shuffle round
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    uint8_t *smem = ds_smem;
    float *qs = reinterpret_cast<float *>(smem + qs_off);
    float *knew = reinterpret_cast<float *>(smem + kvnew_off);
    float *vnew = knew + HD;
    float *ared = reinterpret_cast<float *>(smem + pa_off);  // [8 warps][REP][HD + 2]
    bool failed = ds_sh.abort != 0;
    uint32_t slot = it % nst, par = (it / nst) & 1;
    float q[REP][DPL], o[REP][DPL], m[REP], ls[REP];
    int cur = -1;
    // RoPE of the element pair (d, d^1) of a head whose columns start at
    // col (rope_with_freqs_preloaded, cpu.rs:650-661).
    auto roped = [&](int col, int d) {
        const float y = gemv_out(__ldcg(accq + col + d), fq);
        const float partner = gemv_out(__ldcg(accq + col + (d ^ 1)), fq);
        const int i = d >> 1;
        const float cs = __ldg(cos_row + i), sn = __ldg(sin_row + i);
        return (d & 1) ? __fadd_rn(__fmul_rn(partner, sn), __fmul_rn(y, cs))
                       : __fsub_rn(__fmul_rn(y, cs), __fmul_rn(partner, sn));
    };
    // q of head group g (pre-scaled, llama.rs:394) and, when this CTA owns
    // the chunk holding the decoded position, the new K/V row (rounded to
    // the cache type, also stored in the cache) -- one pass of loads.
    auto begin = [&](int g) {
        const long long ulast = (long long)g * nch + nch - 1;
        const bool own_new = has_new && ulast >= u0 && ulast < u1;
        const int nq_el = REP * HD;
        for (int i = tid; i < nq_el + (own_new ? HD : 0); i += DS_CONSUMERS) {
            if (i < nq_el) {
                const int r = i / HD, d = i - r * HD;
                qs[i] = __fmul_rn(roped((g * REP + r) * HD, d), q_scale);
            } else {
                const int d = i - nq_el;
                const size_t row =
                    (((size_t)page_table[pos / page_size] * nkv + g) * page_size + pos % page_size) * HD;
                const KV kq = KL::from(roped(q_dim + g * HD, d));
                const KV vq = KL::from(gemv_out(__ldcg(accq + q_dim + kv_dim + g * HD + d), fq));
                knew[d] = KL::to(kq);
                vnew[d] = KL::to(vq);
                kcl[row + d] = kq;
                vcl[row + d] = vq;
            }
        }
        ds_sync();
#pragma unroll
        for (int r = 0; r < REP; r++) {
            m[r] = -INFINITY;
            ls[r] = 0.f;
#pragma unroll
            for (int e = 0; e < DPL; e++) q[r][e] = qs[r * HD + lane * DPL + e], o[r][e] = 0.f;
        }
    };
    // Merge the warp states: M = max_w m_w, o = sum_w e^(m_w - M) o_w,
    // l likewise; write the head's record.
    auto finish = [&](int g) {
#pragma unroll
        for (int r = 0; r < REP; r++) {
            float *aw = ared + ((size_t)warp * REP + r) * (HD + 2);
#pragma unroll
            for (int e = 0; e < DPL; e++) aw[lane * DPL + e] = o[r][e];
            if (lane == 0) aw[HD] = m[r], aw[HD + 1] = ls[r];
        }
        ds_sync();
        float *rec = part + ((size_t)g * G + cta) * REP * DS_REC(HD);
        for (int i = tid; i < REP * HD; i += DS_CONSUMERS) {
            const int r = i / HD, d = i - r * HD;
            float M = -INFINITY;
            for (int w = 0; w < 8; w++) M = fmaxf(M, ared[((size_t)w * REP + r) * (HD + 2) + HD]);
            float O = 0.f, Lz = 0.f;
            for (int w = 0; w < 8; w++) {
                const float *aw = ared + ((size_t)w * REP + r) * (HD + 2);
                if (aw[HD] == -INFINITY) continue;
                const float sw = expf(aw[HD] - M);
                O = fmaf(aw[d], sw, O);
                Lz = fmaf(aw[HD + 1], sw, Lz);
            }
            rec[(size_t)r * DS_REC(HD) + d] = O;
            if (d == 0) {
                rec[(size_t)r * DS_REC(HD) + HD] = M;
                rec[(size_t)r * DS_REC(HD) + HD + 1] = Lz;
            }
        }
        ds_sync();
    };
    for (long long u = u0; u < u1; u++) {
        const int g = (int)(u / nch), j = (int)(u - (long long)g * nch);
        if (g != cur) {
            if (cur >= 0) finish(cur);
            cur = g;
            begin(g);
        }
        const int p0 = j * chunk, np = min(chunk, ctx - p0);
        // one stage: K rows in the first half, V rows in the second
        if (!failed && !mbar_wait(bars + 8 * slot, par)) {
            failed = true;
            ds_sh.abort = 1;
        }
        KV *kst = reinterpret_cast<KV *>(smem + (size_t)slot * DS_STAGE);
        KV *vst = reinterpret_cast<KV *>(smem + (size_t)slot * DS_STAGE + DS_KV_HALF);
        if (has_new && j == nch - 1) {
            for (int d = tid; d < HD; d += DS_CONSUMERS) {
                kst[(size_t)(pos - p0) * HD + d] = KL::from(knew[d]);
                vst[(size_t)(pos - p0) * HD + d] = KL::from(vnew[d]);
            }
            ds_sync();
        }
        if (!failed) {
            for (int i0 = warp; i0 < np; i0 += 8 * BR) {
                float sc[BR][REP];
#pragma unroll
                for (int b = 0; b < BR; b++) {
                    const int i = i0 + 8 * b;
                    float kx[DPL];
                    if (i < np) KL::template load_n<DPL>(kst + (size_t)i * HD + lane * DPL, kx);
#pragma unroll
                    for (int r = 0; r < REP; r++) {
                        float t = 0.f;
                        if (i < np) {
#pragma unroll
                            for (int e = 0; e < DPL; e++) t = fmaf(q[r][e], kx[e], t);
                        }
                        sc[b][r] = t;
                    }
                }
#pragma unroll
                for (int off = 16; off > 0; off >>= 1)
#pragma unroll
                    for (int b = 0; b < BR; b++)
#pragma unroll
                        for (int r = 0; r < REP; r++) sc[b][r] += __shfl_xor_sync(0xffffffffu, sc[b][r], off);
#pragma unroll
                for (int r = 0; r < REP; r++) {
                    float mn = m[r];
#pragma unroll
                    for (int b = 0; b < BR; b++)
                        if (i0 + 8 * b < np) mn = fmaxf(mn, sc[b][r]);
                    const float al = m[r] == -INFINITY ? 0.f : expf(m[r] - mn);
                    ls[r] *= al;
#pragma unroll
                    for (int e = 0; e < DPL; e++) o[r][e] *= al;
                    m[r] = mn;
#pragma unroll
                    for (int b = 0; b < BR; b++) sc[b][r] = (i0 + 8 * b < np) ? expf(sc[b][r] - mn) : 0.f;
                }
#pragma unroll
                for (int b = 0; b < BR; b++) {
                    const int i = i0 + 8 * b;
                    if (i >= np) continue;
                    float vx[DPL];
                    KL::template load_n<DPL>(vst + (size_t)i * HD + lane * DPL, vx);
#pragma unroll
                    for (int r = 0; r < REP; r++) {
                        ls[r] += sc[b][r];
#pragma unroll
                        for (int e = 0; e < DPL; e++) o[r][e] = fmaf(sc[b][r], vx[e], o[r][e]);
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0 && !failed) mbar_arrive(bars + 8 * (nst + slot));
        if (++slot == (uint32_t)nst) slot = 0, par ^= 1;
        it++;
    }
    if (cur >= 0) finish(cur);
    return it;
}

// ---- the kernel ----------------------------------------------------------------
// Tensor parallelism: this CTA's slice of a row projection's h outputs,
// y = sum * f (this rank's partial product), into slot [e & 1][rank] of
// every rank's cells, each value paired with the exchange's epoch e in one
// store.
__device__ __forceinline__ void ds_tp_push(const DsArgs &a, const long long *sums, double f, unsigned e, int G, int cta) {
    const int tid = threadIdx.x, ld = a.h + 2;
    const int c0 = (int)((long long)a.h * cta / G), c1 = (int)((long long)a.h * (cta + 1) / G);
    const size_t slot = ((size_t)(e & 1u) * a.tp + a.tp_rank) * ld;
    for (int col = c0 + tid; col < c1; col += DS_CONSUMERS) {
        const float y = gemv_out(__ldcg(sums + col), f);
        for (int r = 0; r < a.tp; r++) st_cell(a.cells[r] + slot + col, y, e);
    }
}

// Tensor parallelism, one thread: this rank's argmax candidate (best, bi
// local to its vocabulary rows) to every rank, then every rank's candidate
// merged in rank order with the argmax tie rule (ties -> the larger index);
// best / bi become the global argmax.  The argmax exchange of the step uses
// cells h and h+1 of slot [e & 1][rank].  Returns false when a wait ran out.
__device__ __forceinline__ bool ds_tp_argmax(const DsArgs &a, float &best, int &bi) {
    const unsigned e = a.epoch0 + 2 * a.L + 1;
    const int ld = a.h + 2;
    const size_t slot = ((size_t)(e & 1u) * a.tp + a.tp_rank) * ld + a.h;
    const unsigned gi = bi < 0 ? 0xffffffffu : (unsigned)(bi + a.v_off);
    for (int r = 0; r < a.tp; r++) {
        st_cell(a.cells[r] + slot, best, e);
        st_cell_u(a.cells[r] + slot + 1, gi, e);
    }
    best = -INFINITY;
    bi = -1;
    const uint2 *mine = a.cells[a.tp_rank] + (size_t)(e & 1u) * a.tp * ld;
    uint64_t t0 = 0;
    for (int r = 0; r < a.tp; r++) {
        const uint2 *c = mine + (size_t)r * ld + a.h;
        uint2 cv = ld_cell(c), ci = ld_cell(c + 1);
        for (uint32_t it = 0; cv.y != e || ci.y != e; it++) {
            if ((it & 63) == 0) {
                const uint64_t t = global_ns();
                if (it == 0) t0 = t;
                else if (t - t0 > SB_WAIT_NS) return false;
            }
            if (cv.y != e) cv = ld_cell(c);
            if (ci.y != e) ci = ld_cell(c + 1);
        }
        const float ov = __uint_as_float(cv.x);
        const int oi = ci.x == 0xffffffffu ? -1 : (int)ci.x;
        if (oi >= 0 && (bi < 0 || ov > best || (ov == best && oi > bi))) best = ov, bi = oi;
    }
    return true;
}

// TP: the tensor-parallel variant (a.tp > 1); the single-GPU kernel carries none of its code.
template <int HD, int REP, typename KV, bool TP>
__global__ void __launch_bounds__(DS_THREADS, 1) decode_step_kernel(const DsArgs a) {
    using KL = DsKv<KV>;
    static_assert(HD % 64 == 0, "head_dim must give each lane 2 or 4 dims");

    uint8_t *smem = ds_smem;
    DsShared &sh = ds_sh;
    const int G = gridDim.x, cta = blockIdx.x, tid = threadIdx.x;
    const int lane = tid & 31, warp = tid >> 5;
    const int nst = a.nst;
    const int ksmax = max(max(a.ks_h, a.ks_q), a.ks_f);
    const DsSmem L = ds_layout(nst, ksmax, REP, HD, a.chunk, a.mtab_bytes);
    const uint32_t bars = smem_u32(smem + L.bars);  // full[nst], empty[nst]
    const uint32_t ring = smem_u32(smem + L.ring);
    unsigned *const abort_flag = a.sync + 2;

    if (tid == 0) {
        for (int i = 0; i < nst; i++) {
            mbar_init(bars + 8 * i, 1);
            mbar_init(bars + 8 * (nst + i), DS_CONSUMERS / 32);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        sh.abort = 0;
        sh.shift = 0;
        sh.rstd = 1.0;
        sh.last = 0;
    }
    __syncthreads();

    // Step constants: the position decoded, the context and its KV chunks.
    const int pos = a.pos_in >= 0 ? a.pos_in : a.seq.pos[0];
    const int cap = min(a.max_pos, a.max_pages * a.page_size);
    const bool has_new = pos >= 0 && pos < cap;
    const int ctx = max(1, min(pos + 1, cap));
    const int nch = (ctx + a.chunk - 1) / a.chunk;
    const long long att_U = (long long)a.nkv * nch;
    const size_t kv_row = (size_t)HD * sizeof(KV);

    if (tid >= DS_CONSUMERS) {
        // ---- producer: one thread issues every stage of the step in order
        if (tid != DS_CONSUMERS) return;
        uint32_t it = 0, slot = 0, par = 0;
        bool ok = true;
        // Every streamed byte is read once per step: keep it from evicting
        // the step's code, activations and column sums from L2.
        const uint64_t stream_policy = l2_evict_first_policy();
        // One stage: a copy of bytes0 at src0 into the slot, and optionally
        // a second copy of bytes1 at src1 into its second half.
        auto issue = [&](const void *src0, uint32_t bytes0, const void *src1 = nullptr, uint32_t bytes1 = 0) {
            if (it >= (uint32_t)nst) {
                if (*(volatile int *)&sh.abort || !mbar_wait(bars + 8 * (nst + slot), par ^ 1)) {
                    ok = false;
                    return;
                }
            }
            mbar_expect_tx(bars + 8 * slot, bytes0 + bytes1);
            tma_load_1d_hint(ring + slot * DS_STAGE, src0, bytes0, bars + 8 * slot, stream_policy);
            if (src1) tma_load_1d_hint(ring + slot * DS_STAGE + DS_KV_HALF, src1, bytes1, bars + 8 * slot, stream_policy);
            it++;
            if (++slot == (uint32_t)nst) slot = 0, par ^= 1;
        };
        auto gemv_stream = [&](const uint4 *w, int KS, int ntiles) {
            DsWalk wk(KS, ntiles, G, cta);
            while (wk.more() && ok) {
                int t, k0, nks;
                wk.next(t, k0, nks);
                issue(w + ((size_t)t * KS + k0) * DS_TN, (uint32_t)nks * DS_TN * 16);
            }
        };
        const int *ptab = a.page_table;  // sequence 0
        const long long au0 = att_U * cta / G, au1 = att_U * (cta + 1) / G;
        for (int l = 0; l < a.L && ok; l++) {
            const DsLayer &ly = a.layers[l];
            gemv_stream(ly.w[0], a.ks_h, a.nt_qkv);
            {
                const char *kc = static_cast<const char *>(a.kc) + (size_t)l * a.layer_kv_bytes;
                const char *vc = static_cast<const char *>(a.vc) + (size_t)l * a.layer_kv_bytes;
                for (long long u = au0; u < au1 && ok; u++) {
                    const int g = (int)(u / nch), j = (int)(u - (long long)g * nch);
                    const int p0 = j * a.chunk, np = min(a.chunk, ctx - p0);
                    const int page = ptab[p0 / a.page_size];
                    const size_t off = (((size_t)page * a.nkv + g) * a.page_size + p0 % a.page_size) * kv_row;
                    issue(kc + off, (uint32_t)(np * kv_row), vc + off, (uint32_t)(np * kv_row));
                }
            }
            gemv_stream(ly.w[1], a.ks_q, a.nt_o);
            gemv_stream(ly.w[2], a.ks_h, a.nt_gu);
            gemv_stream(ly.w[3], a.ks_f, a.nt_down);
        }
        gemv_stream(a.lm_w, a.ks_h, a.nt_lm);
        if (!ok) {
            atomicExch(abort_flag, 1u);
            // Let the copies already issued land before the CTA can exit.
            const uint32_t first = it > (uint32_t)nst ? it - nst : 0;
            for (uint32_t s = first; s < it; s++) mbar_wait(bars + 8 * (s % nst), (s / nst) & 1);
        }
        return;
    }

    // ---- consumers (warps 0-7)
    uint32_t it = 0;     // stages consumed; mirrors the producer's count
    unsigned phase = 0;  // phases completed by this CTA

    // Optional timeline, per phase p and CTA: %globaltimer at the phase's
    // start (after its barrier), after its input stage, when its first and
    // its last weight stage were ready (GEMV phases), and at its end (before
    // the arrival): stamps[(p * G + cta) * DS_STAMPS + i], i = 0, 1, 2, 3, 4.
    // Compiled in only with SB_STEP_TIMELINE (a profiling build): the default
    // kernel carries no trace of it.
    auto mark = [&](int i) {
#ifdef SB_STEP_TIMELINE
        if (a.stamps && tid == 0) a.stamps[((size_t)phase * G + cta) * DS_STAMPS + i] = global_ns();
#endif
    };
    auto ready_slot = [&]() -> unsigned long long * {
#ifdef SB_STEP_TIMELINE
        return a.stamps ? a.stamps + ((size_t)phase * G + cta) * DS_STAMPS + 2 : nullptr;
#else
        return nullptr;
#endif
    };
    // Arrive at the end of the current phase.
    auto arrive = [&]() {
        ds_sync();
        mark(4);
        // release at gpu scope: the CTA's writes (ordered before this thread by
        // the named barrier) are visible to whoever acquires the new count
        if (tid == 0) asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(a.sync), "r"(1u) : "memory");
        phase++;
    };
    // Wait until every CTA has arrived at the end of the previous phase.
    // Returns false (uniformly) when the step is being abandoned.
    auto wait_all = [&]() -> bool {
        if (tid == 0 && !sh.abort) {
            const unsigned target = (unsigned)G * phase;
            uint64_t t0 = 0;
            for (uint32_t i = 0;; i++) {
                if (ld_acquire(a.sync) >= target) break;
                if ((i & 31) == 0) {
                    if (ld_acquire(abort_flag)) {
                        sh.abort = 1;
                        break;
                    }
                    const uint64_t t = global_ns();
                    if (i == 0) t0 = t;
                    else if (t - t0 > SB_WAIT_NS) {
                        sh.abort = 1;
                        break;
                    }
                }
            }
        }
        ds_sync();
        const bool go = !sh.abort;
        ds_sync();
        if (!go && tid == 0) atomicExch(abort_flag, 1u);
        mark(0);
        return go;
    };
    // Zero this CTA's share of an int64 column-sum buffer (n columns).
    auto zero_acc = [&](long long *buf, int n) {
        const int z0 = (int)((long long)n * cta / G), z1 = (int)((long long)n * (cta + 1) / G);
        for (int i = z0 + tid; i < z1; i += DS_CONSUMERS) buf[i] = 0;
    };

    // Tensor parallelism: this CTA's slice of a row projection's h outputs,
    // y = sum * f (this rank's partial product), into slot [e & 1][rank] of
    // every rank's cells, paired with the exchange's epoch e in one store.
    const int tp_ld = a.h + 2;
    auto tp_push = [&](const long long *sums, double f, unsigned e) { ds_tp_push(a, sums, f, e, G, cta); };
    // This rank's cells of exchange e: [src][tp_ld].
    auto tp_cells = [&](unsigned e) -> const uint2 * {
        return a.cells[a.tp_rank] + (size_t)(e & 1u) * a.tp * tp_ld;
    };

    // Attention over this CTA's (kv head, chunk) units of layer l.
    auto attention = [&](int l) {
        const long long u0 = att_U * cta / G, u1 = att_U * (cta + 1) / G;
        const int rp = min(max(pos, 0), a.max_pos - 1);  // rope table row
        it = ds_attention<HD, REP, KV>(
            it, nst, bars, u0, u1, nch, ctx, pos, has_new, a.acc + (size_t)((4 * l) % 3) * a.acc_n,
            gemv_factor(sh.shift, a.layers[l].scale[0], sh.rstd), a.rope_cos + (size_t)rp * (HD / 2),
            a.rope_sin + (size_t)rp * (HD / 2),
            reinterpret_cast<KV *>(static_cast<char *>(a.kc) + (size_t)l * a.layer_kv_bytes),
            reinterpret_cast<KV *>(static_cast<char *>(a.vc) + (size_t)l * a.layer_kv_bytes), a.page_table, a.part,
            a.nkv, a.q_dim, a.kv_dim, a.page_size, a.chunk, a.q_scale, G, cta, (uint32_t)L.qs, (uint32_t)L.kvnew,
            (uint32_t)L.pa);
    };

    auto accbuf = [&](int j) { return a.acc + (size_t)(j % 3) * a.acc_n; };
    const int npad_qkv = a.nt_qkv * DS_TN, npad_o = a.nt_o * DS_TN, npad_gu = a.nt_gu * DS_TN,
              npad_down = a.nt_down * DS_TN, npad_lm = a.nt_lm * DS_TN;
    const bool writer = cta == 0;
    const uint32_t pa_off = (uint32_t)L.pa, red_off = (uint32_t)L.red;
    const int rmax = G / a.nkv + 2;  // records per head: a head's units span at most this many CTAs

    // token of this step (embedding lookup, cpu.rs:485-498)
    int tok = a.tok_in >= 0 ? a.tok_in
                            : ((a.seq.prompt_len && pos < a.seq.prompt_len[0]) ? a.seq.prompt[pos] : a.seq.tok[0]);
    tok = min(max(tok, 0), a.V - 1);

    {
        const int rp = min(max(pos, 0), a.max_pos - 1);
        ds_prefetch_l2(a.embed + (size_t)tok * a.h, sizeof(float) * a.h, cta, G);
        ds_prefetch_l2(a.norm_in, sizeof(float) * a.h, cta, G);
        ds_prefetch_l2(a.rope_cos + (size_t)rp * (HD / 2), sizeof(float) * (HD / 2), cta, G);
        ds_prefetch_l2(a.rope_sin + (size_t)rp * (HD / 2), sizeof(float) * (HD / 2), cta, G);
    }
    mark(0);     // phase 0 starts with the kernel
    int xv = 0;  // index of the current residual version in a.x
    bool go = true;
    for (int l = 0; l < a.L; l++) {
        const DsLayer &ly = a.layers[l];
        const int j = 4 * l;  // GEMV index of this layer's QKV
        // ---- QKV: input = RMSNorm(x) (x = embedding, or x + down of the previous layer)
        if (go && l > 0) go = wait_all();
        if (go) {
            if (j >= 2) zero_acc(accbuf(j - 2), npad_gu);
            const float *nw = a.norm_in + (size_t)l * a.h;
            if (l == 0) {
                ds_in_rows<DS_QMAX_H>(a.embed + (size_t)tok * a.h, true, nw, a.h, a.ks_h, a.eps,
                                      writer ? a.x : nullptr, pa_off);
                xv = 0;
            } else if constexpr (TP) {
                const unsigned e = a.epoch0 + 2 * l;  // the down exchange of layer l - 1
                tp_push(accbuf(j - 1), gemv_factor(sh.shift, a.layers[l - 1].scale[3], sh.rstd), e);
                ds_in_resid_tp<DS_QMAX_H>(a.x + (size_t)xv * a.h, tp_cells(e), a.tp, tp_ld, e, nw, a.h, a.ks_h, a.eps,
                                          writer ? a.x + (size_t)(xv ^ 1) * a.h : nullptr,
                                          (writer && a.trace) ? a.trace + (size_t)(l - 1) * a.h : nullptr, pa_off);
                xv ^= 1;
            } else {
                ds_in_resid<DS_QMAX_H>(a.x + (size_t)xv * a.h, accbuf(j - 1), a.layers[l - 1].scale[3], sh.shift,
                                       sh.rstd, nw, a.h, a.ks_h, a.eps, writer ? a.x + (size_t)(xv ^ 1) * a.h : nullptr,
                                       (writer && a.trace) ? a.trace + (size_t)(l - 1) * a.h : nullptr, pa_off);
                xv ^= 1;
            }
            mark(1);
            it = ds_gemv(it, nst, bars, a.ks_h, a.nt_qkv, accbuf(j), G, cta, pa_off, red_off, ready_slot());
        }
        arrive();
        // ---- attention
        if (go) go = wait_all();
        if (go) {
            mark(1);
            attention(l);
        }
        arrive();
        // ---- O: input = combined attention output
        ds_prefetch_l2(a.norm_post + (size_t)l * a.h, sizeof(float) * a.h, cta, G);
        if (go) go = wait_all();
        if (go) {
            if (l > 0) zero_acc(accbuf(j - 1), npad_down);
            if (a.q_dim <= 4 * DS_CONSUMERS * 4)
                ds_in_att<HD, REP, 4>(a.part, (unsigned)att_U, nch, G, a.nh, a.q_dim, a.ks_q, rmax, pa_off);
            else
                ds_in_att<HD, REP, DS_QMAX_H>(a.part, (unsigned)att_U, nch, G, a.nh, a.q_dim, a.ks_q, rmax, pa_off);
            mark(1);
            it = ds_gemv(it, nst, bars, a.ks_q, a.nt_o, accbuf(j + 1), G, cta, pa_off, red_off, ready_slot());
        }
        arrive();
        // ---- gate/up: input = RMSNorm(x + o)
        if (go) go = wait_all();
        if (go) {
            zero_acc(accbuf(j), npad_qkv);
            if constexpr (TP) {
                const unsigned e = a.epoch0 + 2 * l + 1;  // the o exchange of layer l
                tp_push(accbuf(j + 1), gemv_factor(sh.shift, ly.scale[1], sh.rstd), e);
                ds_in_resid_tp<DS_QMAX_H>(a.x + (size_t)xv * a.h, tp_cells(e), a.tp, tp_ld, e,
                                          a.norm_post + (size_t)l * a.h, a.h, a.ks_h, a.eps,
                                          writer ? a.x + (size_t)(xv ^ 1) * a.h : nullptr, nullptr, pa_off);
            } else {
                ds_in_resid<DS_QMAX_H>(a.x + (size_t)xv * a.h, accbuf(j + 1), ly.scale[1], sh.shift, sh.rstd,
                                       a.norm_post + (size_t)l * a.h, a.h, a.ks_h, a.eps,
                                       writer ? a.x + (size_t)(xv ^ 1) * a.h : nullptr, nullptr, pa_off);
            }
            xv ^= 1;
            mark(1);
            it = ds_gemv(it, nst, bars, a.ks_h, a.nt_gu, accbuf(j + 2), G, cta, pa_off, red_off, ready_slot());
        }
        arrive();
        // ---- SwiGLU (llama.rs:490-500), this CTA's share of the F outputs
        if (go) go = wait_all();
        if (go) {
            mark(1);
            const long long *gu = accbuf(j + 2);
            const int f0 = (int)((long long)a.F * cta / G), f1 = (int)((long long)a.F * (cta + 1) / G);
            const double fg = gemv_factor(sh.shift, ly.scale[2], sh.rstd), fu = gemv_factor(sh.shift, ly.scale_up, sh.rstd);
            for (int f = f0 + tid; f < f1; f += DS_CONSUMERS) {
                const int col = (f >> 4) * 32 + (f & 15);
                const long long tg = __ldcg(gu + col), tu = __ldcg(gu + col + 16);
                const float yg = gemv_out(tg, fg);
                const float yu = gemv_out(tu, fu);
                a.act[f] = __fmul_rn(silu_f64(yg), yu);
            }
        }
        arrive();
        // ---- down: input = SwiGLU output
        ds_prefetch_l2(l + 1 < a.L ? a.norm_in + (size_t)(l + 1) * a.h : a.norm_final, sizeof(float) * a.h, cta, G);
        if (go) go = wait_all();
        if (go) {
            zero_acc(accbuf(j + 1), npad_o);
            ds_in_rows<DS_QMAX_F>(a.act, false, nullptr, a.F, a.ks_f, a.eps, nullptr, pa_off);
            mark(1);
            it = ds_gemv(it, nst, bars, a.ks_f, a.nt_down, accbuf(j + 3), G, cta, pa_off, red_off, ready_slot());
        }
        arrive();
    }
    const int jl = 4 * a.L;  // GEMV index of the lm_head
    // ---- lm_head: input = RMSNorm(x + down)
    if (go) go = wait_all();
    if (go) {
        zero_acc(accbuf(jl - 2), npad_gu);
        if constexpr (TP) {
            const unsigned e = a.epoch0 + 2 * a.L;  // the down exchange of the last layer
            tp_push(accbuf(jl - 1), gemv_factor(sh.shift, a.layers[a.L - 1].scale[3], sh.rstd), e);
            ds_in_resid_tp<DS_QMAX_H>(a.x + (size_t)xv * a.h, tp_cells(e), a.tp, tp_ld, e, a.norm_final, a.h,
                                      a.ks_h, a.eps, writer ? a.x + (size_t)(xv ^ 1) * a.h : nullptr,
                                      (writer && a.trace) ? a.trace + (size_t)(a.L - 1) * a.h : nullptr, pa_off);
        } else {
            ds_in_resid<DS_QMAX_H>(a.x + (size_t)xv * a.h, accbuf(jl - 1), a.layers[a.L - 1].scale[3], sh.shift,
                                   sh.rstd, a.norm_final, a.h, a.ks_h, a.eps,
                                   writer ? a.x + (size_t)(xv ^ 1) * a.h : nullptr,
                                   (writer && a.trace) ? a.trace + (size_t)(a.L - 1) * a.h : nullptr, pa_off);
        }
        mark(1);
        it = ds_gemv(it, nst, bars, a.ks_h, a.nt_lm, accbuf(jl), G, cta, pa_off, red_off, ready_slot());
    }
    arrive();
    // ---- logits and this CTA's argmax candidate (ties -> larger index,
    // generate.rs:167-173); the buffers still holding sums are cleared.
    if (go) go = wait_all();
    if (go) {
        long long *lm = accbuf(jl);
        const int n0 = (int)((long long)npad_lm * cta / G), n1 = (int)((long long)npad_lm * (cta + 1) / G);
        float best = -INFINITY;
        int bi = -1;
        const double fl = gemv_factor(sh.shift, a.lm_scale, sh.rstd);
        for (int n = n0 + tid; n < n1; n += DS_CONSUMERS) {
            const long long t = __ldcg(lm + n);
            lm[n] = 0;
            if (n < a.V_lm) {
                const float y = gemv_out(t, fl);
                a.logits[n] = y;
                if (bi < 0 || y >= best) best = y, bi = n;
            }
        }
        for (int off = 16; off > 0; off >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, off);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
            if (oi >= 0 && (bi < 0 || ov > best || (ov == best && oi > bi))) best = ov, bi = oi;
        }
        if (lane == 0) sh.cand_v[warp] = best, sh.cand_i[warp] = bi;
        zero_acc(accbuf(jl - 1), npad_down);
        ds_sync();
        if (tid == 0) {
            for (int w = 1; w < 8; w++) {
                const float ov = sh.cand_v[w];
                const int oi = sh.cand_i[w];
                if (oi >= 0 && (bi < 0 || ov > best || (ov == best && oi > bi))) best = ov, bi = oi;
            }
            a.cand_val[cta] = best;
            a.cand_idx[cta] = bi;
        }
    }
    // ---- exit: the last CTA picks the token, advances the sequence state
    // and resets the phase counters for the next step.
    ds_sync();
    if (tid == 0) {
        __threadfence();
        const unsigned prev = atomicAdd(a.sync + 1, 1u);
        sh.last = prev == (unsigned)G - 1;
    }
    ds_sync();
    if (sh.last && tid == 0) {
        __threadfence();
        if (a.greedy && !ld_acquire(abort_flag)) {
            float best = -INFINITY;
            int bi = -1;
            for (int c = 0; c < G; c++) {
                const float ov = __ldcg(a.cand_val + c);
                const int oi = __ldcg(a.cand_idx + c);
                if (oi >= 0 && (bi < 0 || ov > best || (ov == best && oi > bi))) best = ov, bi = oi;
            }
            bool ok = true;
            if constexpr (TP) {
                ok = ds_tp_argmax(a, best, bi);
                if (!ok) atomicExch(abort_flag, 1u);
            }
            if (ok) {
                const int next = bi < 0 ? 0 : bi;
                const SeqState &s = a.seq;
                const int plen = (a.pos_in < 0 && s.prompt_len) ? s.prompt_len[0] : 0;
                s.last[0] = next;
                if (pos >= plen - 1) {  // generate.rs:72-75: sample after the last prompt token
                    const int gcount = s.ngen[0];
                    if (gcount < s.max_gen) s.out[gcount] = next;
                    s.ngen[0] = gcount + 1;
                }
                s.tok[0] = next;
                s.pos[0] = pos + 1;
            }
        }
        a.sync[0] = 0;
        a.sync[1] = 0;
    }
}

template <int HD, int REP, typename KV, bool TP>
inline int ds_limit_k(int *limit) {
    static int lim[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!lim[dev & 63]) SB_TRY(allow_max_dynamic_smem(decode_step_kernel<HD, REP, KV, TP>, &lim[dev & 63]));
    *limit = lim[dev & 63];
    return SB_OK;
}
// Dynamic shared memory the step kernels of this shape may use (the single-GPU
// and tensor-parallel variants declare the same static shared memory).
template <int HD, int REP, typename KV>
inline int ds_limit(int *limit) {
    int l1 = 0, l2 = 0;
    SB_TRY((ds_limit_k<HD, REP, KV, false>(&l1)));
    SB_TRY((ds_limit_k<HD, REP, KV, true>(&l2)));
    *limit = std::min(l1, l2);
    return SB_OK;
}

template <int HD, typename KV>
inline int ds_limit_rep(int rep, int *limit) {
    switch (rep) {
    case 1: return ds_limit<HD, 1, KV>(limit);
    case 2: return ds_limit<HD, 2, KV>(limit);
    case 4: return ds_limit<HD, 4, KV>(limit);
    case 8: return ds_limit<HD, 8, KV>(limit);
    default: return set_error(SB_ERR_UNSUPPORTED, "decode step: GQA ratio %d", rep);
    }
}

template <int HD, int REP, typename KV>
inline int ds_inst(const DsArgs &a, cudaStream_t st) {
    auto kern = a.tp > 1 ? decode_step_kernel<HD, REP, KV, true> : decode_step_kernel<HD, REP, KV, false>;
    int limit = 0;
    const int lrc = ds_limit<HD, REP, KV>(&limit);
    SB_TRY(lrc);
    const int ksmax = std::max(std::max(a.ks_h, a.ks_q), a.ks_f);
    const size_t smem = ds_layout(a.nst, ksmax, REP, HD, a.chunk, a.mtab_bytes).total;
    SB_CHECK(smem <= (size_t)limit, SB_ERR_SHAPE, "decode step: %zu B of shared memory (limit %d)", smem, limit);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ds_grid());
    cfg.blockDim = dim3(DS_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // all CTAs resident at once, or the launch fails
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    SB_CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, a));
    return SB_OK;
}

template <int HD, typename KV>
inline int ds_rep(const DsArgs &a, int rep, cudaStream_t st) {
    switch (rep) {
    case 1: return ds_inst<HD, 1, KV>(a, st);
    case 2: return ds_inst<HD, 2, KV>(a, st);
    case 4: return ds_inst<HD, 4, KV>(a, st);
    case 8: return ds_inst<HD, 8, KV>(a, st);
    default: return set_error(SB_ERR_UNSUPPORTED, "decode step: GQA ratio %d", rep);
    }
}

}  // namespace
}  // namespace sb
