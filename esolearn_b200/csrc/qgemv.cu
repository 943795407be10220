// Dequant-fused int8 GEMV for decode (M <= 4 rows): the B200 replacement of
// matmul_i8_f32 (backend/mod.rs:521-533, CPU cpu.rs:1129-1160) on every
// projection of the Llama decode step.
//
// Arithmetic.  Each CTA turns its activation rows into exact 23-bit fixed
// point, a[k] * 2^s = A0 + 2^8 A1 + 2^16 A2 (bytes A0, A1 unsigned, A2
// signed), with one power-of-two exponent s per row.  The int8 weights are
// then multiplied against the three byte planes with dp4a: every product
// and partial sum is an exact integer, so the result only depends on the
// activations' fixed-point rounding (|err| <= 2^-23 * max|a| per element),
// never on summation order.  The weights are never dequantized: the
// per-tensor scale (and the fused RMSNorm factor) multiplies the exact
// integer dot product once, in f64, in the epilogue.  Grouped scales (32 or
// 64 rows) are applied per group, in f64.
//
// Bandwidth.  One CTA owns one TN-column tile over all of K.  Tile widths
// are chosen so that every tile is resident in a single wave with equal
// work, each thread keeps QG_DEPTH 16-byte weight loads in flight (the first
// batch is issued before the grid-dependency wait, overlapping the previous
// kernel's tail), and weight loads bypass L1.
//
// RMSNorm fusion (rmsnorm, cpu.rs:574-599): with norm_w set, the planes
// encode x[k]*w[k] and each CTA computes rstd = 1/sqrt(mean(x^2)+eps) of the
// whole row in f64; y is multiplied by rstd in the epilogue.
#include "qgemv.cuh"

#include <algorithm>

namespace sb {

constexpr int QG_DEPTH = 8;

struct QGSmem {
    // Offsets inside the dynamic shared memory block.
    size_t planes, red, ys, rowinfo, total;
};

__host__ __device__ inline QGSmem qg_layout(int M, int KS, int TN) {
    QGSmem L;
    L.planes = 0;
    L.red = (size_t)M * 3 * KS * 16;
    L.ys = L.red + (size_t)M * QG_THREADS * 8;
    L.rowinfo = L.ys + (size_t)M * TN * 4;
    L.rowinfo = (L.rowinfo + 15) & ~(size_t)15;
    // rowinfo: rstd[M] (double), shift[M] (int, stored as double), prologue
    // reduction scratch [8 warps][M][2] doubles.
    L.total = L.rowinfo + (size_t)M * 16 + (size_t)8 * M * 2 * 8;
    return L;
}

size_t qgemv_smem_bytes(int M, int KS, int TN) { return qg_layout(M, KS, TN).total; }

template <int M>
__device__ __forceinline__ void load_quad(const QGemvArgs &a, int m, int q, float v[4]) {
    const int K = a.w.K;
    const int k0 = q * 4;
    if (m >= a.M || k0 >= K) {
        v[0] = v[1] = v[2] = v[3] = 0.0f;
        return;
    }
    if (a.x_bf16) {
        const __nv_bfloat16 *xr = reinterpret_cast<const __nv_bfloat16 *>(a.x) + (size_t)m * a.ldx;
#pragma unroll
        for (int i = 0; i < 4; i++) v[i] = (k0 + i < K) ? __bfloat162float(xr[k0 + i]) : 0.0f;
    } else {
        const float *xr = reinterpret_cast<const float *>(a.x) + (size_t)m * a.ldx;
        if (k0 + 4 <= K && ((reinterpret_cast<uintptr_t>(xr + k0) & 15) == 0)) {
            float4 t = *reinterpret_cast<const float4 *>(xr + k0);
            v[0] = t.x, v[1] = t.y, v[2] = t.z, v[3] = t.w;
        } else {
#pragma unroll
            for (int i = 0; i < 4; i++) v[i] = (k0 + i < K) ? xr[k0 + i] : 0.0f;
        }
    }
}

// Builds the fixed-point byte planes of the M activation rows in shared
// memory and the per-row rstd / exponent.
template <int M>
__device__ void qg_prologue(const QGemvArgs &a, uint8_t *smem, const QGSmem &L) {
    const int KS = a.w.KS, K = a.w.K;
    const int nq = KS * 4;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    uint32_t *planes = reinterpret_cast<uint32_t *>(smem + L.planes);
    double *rstd = reinterpret_cast<double *>(smem + L.rowinfo);
    int *shift = reinterpret_cast<int *>(smem + L.rowinfo + (size_t)M * 8);
    double *scratch = reinterpret_cast<double *>(smem + L.rowinfo + (size_t)M * 16);

    float ssq[M], amx[M];
#pragma unroll
    for (int m = 0; m < M; m++) ssq[m] = 0.0f, amx[m] = 0.0f;
    for (int q = tid; q < nq; q += QG_THREADS) {
        float nw[4] = {1.0f, 1.0f, 1.0f, 1.0f};
        if (a.norm_w) {
#pragma unroll
            for (int i = 0; i < 4; i++) nw[i] = (q * 4 + i < K) ? __ldg(a.norm_w + q * 4 + i) : 0.0f;
        }
#pragma unroll
        for (int m = 0; m < M; m++) {
            float v[4];
            load_quad<M>(a, m, q, v);
#pragma unroll
            for (int i = 0; i < 4; i++) {
                ssq[m] = fmaf(v[i], v[i], ssq[m]);
                amx[m] = fmaxf(amx[m], fabsf(__fmul_rn(v[i], nw[i])));
            }
        }
    }
#pragma unroll
    for (int m = 0; m < M; m++) {
        const double s = warp_sum_d((double)ssq[m]);
        const float x = warp_max_f(amx[m]);
        if (lane == 0) {
            scratch[(warp * M + m) * 2 + 0] = s;
            scratch[(warp * M + m) * 2 + 1] = (double)x;
        }
    }
    __syncthreads();
    if (tid < M) {
        const int m = tid;
        double s = 0.0, x = 0.0;
        for (int w = 0; w < QG_THREADS / 32; w++) {
            s += scratch[(w * M + m) * 2 + 0];
            x = fmax(x, scratch[(w * M + m) * 2 + 1]);
        }
        // rmsnorm (cpu.rs:582-588): mean of squares, rstd = 1/sqrt(mean+eps), f64.
        rstd[m] = a.norm_w ? 1.0 / sqrt(s / (double)K + (double)a.eps) : 1.0;
        int e = 0;
        if (x > 0.0) frexp(x, &e);  // x = f * 2^e, f in [0.5, 1)
        int sh = (x > 0.0) ? 22 - e : 0;  // |a * 2^sh| < 2^22
        shift[m] = sh < -126 ? -126 : (sh > 126 ? 126 : sh);
    }
    __syncthreads();
    for (int q = tid; q < nq; q += QG_THREADS) {
        float nw[4] = {1.0f, 1.0f, 1.0f, 1.0f};
        if (a.norm_w) {
#pragma unroll
            for (int i = 0; i < 4; i++) nw[i] = (q * 4 + i < K) ? __ldg(a.norm_w + q * 4 + i) : 0.0f;
        }
#pragma unroll
        for (int m = 0; m < M; m++) {
            float v[4];
            load_quad<M>(a, m, q, v);
            const float sc = __int_as_float((shift[m] + 127) << 23);  // 2^shift, exact
            uint32_t w0 = 0, w1 = 0, w2 = 0;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                // round-to-nearest-even to an integer: |t| < 2^22, so t + 1.5*2^23
                // lands in [2^23, 2^24) where the float ulp is 1.
                const float t = __fmul_rn(__fmul_rn(v[i], nw[i]), sc);
                const int A = __float_as_int(__fadd_rn(t, 12582912.0f)) - 0x4B400000;
                w0 |= (uint32_t)(A & 0xff) << (8 * i);
                w1 |= (uint32_t)((A >> 8) & 0xff) << (8 * i);
                w2 |= (uint32_t)((A >> 16) & 0xff) << (8 * i);
            }
            planes[(size_t)(m * 3 + 0) * nq + q] = w0;
            planes[(size_t)(m * 3 + 1) * nq + q] = w1;
            planes[(size_t)(m * 3 + 2) * nq + q] = w2;
        }
    }
}

template <int M>
__device__ __forceinline__ void qg_mac(const uint4 &wv, const uint4 *planes4, int KS, int ks,
                                       int (&acc0)[M], int (&acc1)[M], int (&acc2)[M]) {
#pragma unroll
    for (int m = 0; m < M; m++) {
        const uint4 p0 = planes4[(size_t)(m * 3 + 0) * KS + ks];
        const uint4 p1 = planes4[(size_t)(m * 3 + 1) * KS + ks];
        const uint4 p2 = planes4[(size_t)(m * 3 + 2) * KS + ks];
        acc0[m] = dp4a_su(wv.x, p0.x, acc0[m]);
        acc0[m] = dp4a_su(wv.y, p0.y, acc0[m]);
        acc0[m] = dp4a_su(wv.z, p0.z, acc0[m]);
        acc0[m] = dp4a_su(wv.w, p0.w, acc0[m]);
        acc1[m] = dp4a_su(wv.x, p1.x, acc1[m]);
        acc1[m] = dp4a_su(wv.y, p1.y, acc1[m]);
        acc1[m] = dp4a_su(wv.z, p1.z, acc1[m]);
        acc1[m] = dp4a_su(wv.w, p1.w, acc1[m]);
        acc2[m] = dp4a_ss(wv.x, p2.x, acc2[m]);
        acc2[m] = dp4a_ss(wv.y, p2.y, acc2[m]);
        acc2[m] = dp4a_ss(wv.z, p2.z, acc2[m]);
        acc2[m] = dp4a_ss(wv.w, p2.w, acc2[m]);
    }
}

__device__ __forceinline__ long long combine_planes(int a0, int a1, int a2) {
    return (long long)a0 + ((long long)a1 << 8) + ((long long)a2 << 16);
}

template <int M, int EPI>
__device__ void qg_epilogue(const QGemvArgs &a, const float *ys) {
    const int TN = a.w.TN, tile = blockIdx.x, tid = threadIdx.x;
    for (int it = tid; it < M * TN; it += QG_THREADS) {
        const int m = it / TN, c = it - m * TN;
        if (m >= a.M) continue;
        const int n = tile * TN + c;
        const float y = ys[m * TN + c];
        if (EPI == QEPI_STORE || EPI == QEPI_LOGITS) {
            if (n < a.w.N) a.out[(size_t)m * a.ldo + n] = y;
        } else if (EPI == QEPI_BIAS) {
            if (n < a.w.N) a.out[(size_t)m * a.ldo + n] = __fadd_rn(y, a.bias[n]);
        } else if (EPI == QEPI_RESID) {
            if (n < a.w.N) {
                float *o = a.out + (size_t)m * a.ldo + n;
                *o = __fadd_rn(*o, y);
            }
        } else if (EPI == QEPI_SWIGLU) {
            const int within = n & 31;
            if (within < 16) {
                const int j = (n >> 5) * 16 + within;
                if (j < a.F) {
                    const float u = ys[m * TN + c + 16];
                    a.out[(size_t)m * a.ldo + j] = __fmul_rn(silu_f64(y), u);
                }
            }
        } else if (EPI == QEPI_QKV) {
            if (n >= a.w.N) continue;
            const int pos = a.pos[m];
            if (pos < 0 || pos >= a.max_pos) continue;  // beyond the cache: nothing to write
            const int qk = a.q_dim + a.kv_dim;
            float val = y;
            if (n < qk) {
                // rope_with_freqs_preloaded (cpu.rs:650-661) with the
                // host-computed f32 cos/sin of pos*freq.
                const int nn = n < a.q_dim ? n : n - a.q_dim;
                const int d = nn % a.hd, i = d >> 1;
                const float partner = ys[m * TN + (c ^ 1)];
                const float cs = a.rope_cos[(size_t)pos * (a.hd / 2) + i];
                const float sn = a.rope_sin[(size_t)pos * (a.hd / 2) + i];
                if (d & 1)
                    val = __fadd_rn(__fmul_rn(partner, sn), __fmul_rn(y, cs));
                else
                    val = __fsub_rn(__fmul_rn(y, cs), __fmul_rn(partner, sn));
            }
            if (n < a.q_dim) {
                a.q_out[(size_t)m * a.q_dim + n] = __fmul_rn(val, a.q_scale);
            } else {
                const bool is_k = n < qk;
                const int nn = is_k ? n - a.q_dim : n - qk;
                const int kh = nn / a.hd, d = nn - kh * a.hd;
                const int page = a.page_table[(size_t)m * a.max_pages + pos / a.page_size];
                const int slot = pos % a.page_size;
                const size_t idx = (((size_t)page * a.n_kv + kh) * a.page_size + slot) * a.hd + d;
                void *cache = is_k ? a.kcache : a.vcache;
                if (a.kv_f32)
                    reinterpret_cast<float *>(cache)[idx] = val;
                else
                    reinterpret_cast<__nv_bfloat16 *>(cache)[idx] = __float2bfloat16_rn(val);
            }
        }
    }
    if (EPI == QEPI_LOGITS) {
        // Per-tile argmax candidate; ties resolve to the larger index.
        const int warp = tid >> 5, lane = tid & 31;
        if (warp < M && warp < a.M) {
            const int m = warp;
            float best = -INFINITY;
            int bi = -1;
            for (int c = lane; c < TN; c += 32) {
                const int n = tile * TN + c;
                if (n < a.w.N) {
                    const float v = ys[m * TN + c];
                    if (bi < 0 || v >= best) best = v, bi = n;
                }
            }
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, best, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (oi >= 0 && (bi < 0 || ov > best || (ov == best && oi > bi))) best = ov, bi = oi;
            }
            if (lane == 0) {
                a.cand_val[(size_t)m * a.w.ntiles + tile] = best;
                a.cand_idx[(size_t)m * a.w.ntiles + tile] = bi;
            }
        }
    }
}

template <int M, int EPI, bool GROUPED>
__global__ void __launch_bounds__(QG_THREADS, 2) qgemv_kernel(const QGemvArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int KS = a.w.KS, TN = a.w.TN;
    const QGSmem L = qg_layout(M, KS, TN);
    const int tid = threadIdx.x;
    const int nkg = QG_THREADS / TN;
    const int col = tid % TN, kg = tid / TN;
    const int R = GROUPED ? a.w.group / 16 : 1;  // k-steps per scale group
    const int nruns = KS / R;
    const int myruns = nruns > kg ? (nruns - kg + nkg - 1) / nkg : 0;
    const int nsteps = myruns * R;
    const uint4 *wp = a.w.w + (size_t)blockIdx.x * KS * TN + col;
    auto step_ks = [&](int i) { return GROUPED ? (kg + (i / R) * nkg) * R + (i % R) : kg + i * nkg; };

    // Weight loads do not depend on earlier kernels: start them before the
    // grid-dependency wait.
    uint4 wb[QG_DEPTH];
#pragma unroll
    for (int d = 0; d < QG_DEPTH; d++)
        if (d < nsteps) wb[d] = ldg_stream(wp + (size_t)step_ks(d) * TN);
    pdl_launch_dependents();
    pdl_wait();

    qg_prologue<M>(a, smem, L);
    __syncthreads();

    const uint4 *planes4 = reinterpret_cast<const uint4 *>(smem + L.planes);
    int acc0[M], acc1[M], acc2[M];
    double accd[M];
#pragma unroll
    for (int m = 0; m < M; m++) acc0[m] = acc1[m] = acc2[m] = 0, accd[m] = 0.0;
    const int NG = GROUPED ? KS / R : 0;
    const float *gs = GROUPED ? a.w.gscale + (size_t)blockIdx.x * NG * TN + col : nullptr;

    for (int base = 0; base < nsteps; base += QG_DEPTH) {
#pragma unroll
        for (int d = 0; d < QG_DEPTH; d++) {
            const int i = base + d;
            if (i < nsteps) {
                const int ks = step_ks(i);
                const uint4 wv = wb[d];
                if (i + QG_DEPTH < nsteps) wb[d] = ldg_stream(wp + (size_t)step_ks(i + QG_DEPTH) * TN);
                qg_mac<M>(wv, planes4, KS, ks, acc0, acc1, acc2);
                if (GROUPED && (i % R) == R - 1) {
                    const double g = (double)__ldg(gs + (size_t)(ks / R) * TN);
#pragma unroll
                    for (int m = 0; m < M; m++) {
                        accd[m] += (double)combine_planes(acc0[m], acc1[m], acc2[m]) * g;
                        acc0[m] = acc1[m] = acc2[m] = 0;
                    }
                }
            }
        }
    }

    // Reduce the nkg partial sums of every column in a fixed order.
    const double *rstd = reinterpret_cast<const double *>(smem + L.rowinfo);
    const int *shift = reinterpret_cast<const int *>(smem + L.rowinfo + (size_t)M * 8);
    float *ys = reinterpret_cast<float *>(smem + L.ys);
    if (GROUPED) {
        double *red = reinterpret_cast<double *>(smem + L.red);
#pragma unroll
        for (int m = 0; m < M; m++) red[m * QG_THREADS + tid] = accd[m];
        __syncthreads();
        if (tid < TN) {
#pragma unroll
            for (int m = 0; m < M; m++) {
                double s = 0.0;
                for (int g = 0; g < nkg; g++) s += red[m * QG_THREADS + g * TN + tid];
                ys[m * TN + tid] = (float)(ldexp(s, -shift[m]) * rstd[m]);
            }
        }
    } else {
        long long *red = reinterpret_cast<long long *>(smem + L.red);
#pragma unroll
        for (int m = 0; m < M; m++) red[m * QG_THREADS + tid] = combine_planes(acc0[m], acc1[m], acc2[m]);
        __syncthreads();
        if (tid < TN) {
#pragma unroll
            for (int m = 0; m < M; m++) {
                long long s = 0;
                for (int g = 0; g < nkg; g++) s += red[m * QG_THREADS + g * TN + tid];
                const float sc = (EPI == QEPI_SWIGLU && (tid & 31) >= 16) ? a.w.scale_up : a.w.scale;
                ys[m * TN + tid] = (float)(ldexp((double)s, -shift[m]) * (double)sc * rstd[m]);
            }
        }
    }
    __syncthreads();
    qg_epilogue<M, EPI>(a, ys);
}

// ---------------------------------------------------------------------------
// host side

size_t qweight_bytes(int K, int N, int TN) {
    const int KS = ceil_div(K, 16);
    const int ntiles = ceil_div(N, TN);
    return (size_t)ntiles * KS * TN * 16;
}

size_t qweight_scale_count(int K, int N, int TN, int group) {
    if (group <= 0) return 1;
    const int KS = ceil_div(K, 16);
    const int NG = KS / (group / 16);
    return (size_t)ceil_div(N, TN) * NG * TN;
}

int qgemv_pick_tn(int N, int K, int min_tn) {
    // Widest parallelism that still fits one resident wave: the smallest
    // tile width whose tile count fits in (#SMs x CTAs per SM).
    const DeviceProps &dp = device_props();
    const int KS = ceil_div(K, 16);
    int per_sm = 2;
    const size_t smem = qgemv_smem_bytes(1, KS, 64);
    if (smem * 3 <= 200 * 1024) per_sm = 3;
    const int slots = dp.sm_count * per_sm;
    const int cands[5] = {16, 32, 64, 128, 256};
    for (int i = 0; i < 5; i++) {
        const int tn = cands[i];
        if (tn < min_tn) continue;
        if (ceil_div(N, tn) <= slots) return tn;
    }
    return 256;
}

template <int M, int EPI, bool GROUPED>
static int launch_inst(const QGemvArgs &a, cudaStream_t st, bool pdl) {
    const size_t smem = qgemv_smem_bytes(M, a.w.KS, a.w.TN);
    auto kern = qgemv_kernel<M, EPI, GROUPED>;
    static int limit[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!limit[dev & 63]) SB_TRY(allow_max_dynamic_smem(kern, &limit[dev & 63]));
    SB_CHECK(smem <= (size_t)limit[dev & 63], SB_ERR_SHAPE,
             "qgemv: K=%d with M=%d needs %zu B of shared memory (max %d)", a.w.K, M, smem, limit[dev & 63]);
    SB_CUDA_TRY(launch(kern, dim3(a.w.ntiles), dim3(QG_THREADS), smem, st, pdl, a));
    return SB_OK;
}

template <int EPI, bool GROUPED>
static int dispatch_m(const QGemvArgs &a, cudaStream_t st, bool pdl) {
    switch (a.M) {
    case 1: return launch_inst<1, EPI, GROUPED>(a, st, pdl);
    case 2: return launch_inst<2, EPI, GROUPED>(a, st, pdl);
    case 3: return launch_inst<3, EPI, GROUPED>(a, st, pdl);
    case 4: return launch_inst<4, EPI, GROUPED>(a, st, pdl);
    default: return set_error(SB_ERR_SHAPE, "qgemv: M=%d outside 1..%d", a.M, QG_MAX_M);
    }
}

int qgemv_launch(int epi, const QGemvArgs &a, cudaStream_t st, bool pdl) {
    SB_CHECK(a.w.w != nullptr && a.x != nullptr, SB_ERR_ARG, "qgemv: null weight or input");
    SB_CHECK(a.w.TN >= 16 && a.w.TN <= 256 && (QG_THREADS % a.w.TN) == 0, SB_ERR_SHAPE,
             "qgemv: bad tile width %d", a.w.TN);
    const bool grouped = a.w.group > 0;
    if (grouped) {
        SB_CHECK(a.w.group == 32 || a.w.group == 64, SB_ERR_SHAPE, "qgemv: group %d not 32/64", a.w.group);
        SB_CHECK(a.w.gscale != nullptr, SB_ERR_ARG, "qgemv: grouped weight without scales");
        switch (epi) {
        case QEPI_STORE: return dispatch_m<QEPI_STORE, true>(a, st, pdl);
        case QEPI_BIAS: return dispatch_m<QEPI_BIAS, true>(a, st, pdl);
        default: return set_error(SB_ERR_UNSUPPORTED, "qgemv: epilogue %d with grouped scales", epi);
        }
    }
    switch (epi) {
    case QEPI_STORE: return dispatch_m<QEPI_STORE, false>(a, st, pdl);
    case QEPI_RESID: return dispatch_m<QEPI_RESID, false>(a, st, pdl);
    case QEPI_SWIGLU:
        SB_CHECK(a.w.TN >= 32, SB_ERR_SHAPE, "qgemv: SwiGLU needs TN >= 32");
        return dispatch_m<QEPI_SWIGLU, false>(a, st, pdl);
    case QEPI_QKV: return dispatch_m<QEPI_QKV, false>(a, st, pdl);
    case QEPI_LOGITS: return dispatch_m<QEPI_LOGITS, false>(a, st, pdl);
    case QEPI_BIAS: return dispatch_m<QEPI_BIAS, false>(a, st, pdl);
    default: return set_error(SB_ERR_ARG, "qgemv: unknown epilogue %d", epi);
    }
}

// ---- packing ---------------------------------------------------------------
__global__ void qweight_pack_kernel(const int8_t *__restrict__ src, int K, int N, int TN, int KS,
                                    int pair_F, int src_tr, uint4 *__restrict__ dst, size_t total16) {
    // One thread per 16-byte unit of the packed layout.
    for (size_t u = blockIdx.x * (size_t)blockDim.x + threadIdx.x; u < total16;
         u += (size_t)gridDim.x * blockDim.x) {
        const int c = (int)(u % TN);
        const size_t r = u / TN;
        const int ks = (int)(r % KS);
        const int tile = (int)(r / KS);
        const int n = tile * TN + c;
        uint32_t words[4] = {0, 0, 0, 0};
        int srcN = N, sn = n;
        bool valid = n < N;
        if (pair_F > 0) {
            // packed column n -> (gate|up, feature j); the source is gate [K,F] then up [K,F].
            const int within = n & 31, j = (n >> 5) * 16 + (within & 15);
            valid = j < pair_F;
            srcN = pair_F;
            sn = j;
        }
        if (valid) {
            const int8_t *base = src;
            if (pair_F > 0 && (n & 31) >= 16) base = src + (size_t)K * pair_F;
#pragma unroll
            for (int j = 0; j < 16; j++) {
                const int k = ks * 16 + j;
                const size_t at = src_tr ? (size_t)sn * K + k : (size_t)k * srcN + sn;
                const uint8_t b = (k < K) ? (uint8_t)base[at] : 0;
                words[j >> 2] |= (uint32_t)b << (8 * (j & 3));
            }
        }
        dst[u] = make_uint4(words[0], words[1], words[2], words[3]);
    }
}

int qweight_pack(const int8_t *src, int K, int N, int TN, int pair_F, int src_tr, uint4 *dst, cudaStream_t st) {
    const int KS = ceil_div(K, 16);
    const size_t total16 = qweight_bytes(K, N, TN) / 16;
    const int blocks = (int)std::min<size_t>((total16 + 255) / 256, (size_t)device_props().sm_count * 16);
    qweight_pack_kernel<<<blocks, 256, 0, st>>>(src, K, N, TN, KS, pair_F, src_tr, dst, total16);
    SB_CUDA_TRY(cudaGetLastError());
    return SB_OK;
}

__global__ void qweight_unpack_kernel(const uint4 *__restrict__ src, int K, int N, int TN, int KS, int pair_F,
                                      int8_t *__restrict__ dst, size_t total16) {
    for (size_t u = blockIdx.x * (size_t)blockDim.x + threadIdx.x; u < total16;
         u += (size_t)gridDim.x * blockDim.x) {
        const int c = (int)(u % TN);
        const size_t r = u / TN;
        const int ks = (int)(r % KS);
        const int tile = (int)(r / KS);
        const int n = tile * TN + c;
        int dstN = N, dn = n;
        bool valid = n < N;
        int8_t *base = dst;
        if (pair_F > 0) {
            const int within = n & 31, j = (n >> 5) * 16 + (within & 15);
            valid = j < pair_F;
            dstN = pair_F;
            dn = j;
            if (within >= 16) base = dst + (size_t)K * pair_F;
        }
        if (!valid) continue;
        const uint4 v = src[u];
        const uint32_t words[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 16; j++) {
            const int k = ks * 16 + j;
            if (k < K) base[(size_t)k * dstN + dn] = (int8_t)((words[j >> 2] >> (8 * (j & 3))) & 0xff);
        }
    }
}

int qweight_unpack(const uint4 *src, int K, int N, int TN, int pair_F, int8_t *dst, cudaStream_t st) {
    const int KS = ceil_div(K, 16);
    const size_t total16 = qweight_bytes(K, N, TN) / 16;
    const int blocks = (int)std::min<size_t>((total16 + 255) / 256, (size_t)device_props().sm_count * 16);
    qweight_unpack_kernel<<<blocks, 256, 0, st>>>(src, K, N, TN, KS, pair_F, dst, total16);
    SB_CUDA_TRY(cudaGetLastError());
    return SB_OK;
}

__global__ void qscale_pack_kernel(const float *__restrict__ src, int N, int TN, int NG, float *dst,
                                   size_t total) {
    for (size_t u = blockIdx.x * (size_t)blockDim.x + threadIdx.x; u < total;
         u += (size_t)gridDim.x * blockDim.x) {
        const int c = (int)(u % TN);
        const size_t r = u / TN;
        const int g = (int)(r % NG);
        const int tile = (int)(r / NG);
        const int n = tile * TN + c;
        dst[u] = n < N ? src[(size_t)g * N + n] : 0.0f;
    }
}

int qscale_pack(const float *src, int K, int N, int TN, int group, float *dst, cudaStream_t st) {
    const int KS = ceil_div(K, 16);
    const int NG = KS / (group / 16);
    const size_t total = qweight_scale_count(K, N, TN, group);
    const int blocks = (int)std::min<size_t>((total + 255) / 256, 4096);
    qscale_pack_kernel<<<blocks, 256, 0, st>>>(src, N, TN, NG, dst, total);
    SB_CUDA_TRY(cudaGetLastError());
    return SB_OK;
}

}  // namespace sb
