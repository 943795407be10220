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
// Data movement.  One CTA owns one TN-column tile over all of K; its weights
// are one contiguous slab of the packed layout.  A producer warp streams the
// slab with 1-D TMA bulk copies (cp.async.bulk, no multicast) through a ring
// of QG_NST x 16 KB shared-memory stages guarded by mbarriers; the first
// ring fill is requested before the grid-dependency wait, so under
// programmatic dependent launch the weight stream starts while the previous
// kernel drains.  Right after the wait the same warp fetches the activation
// rows with one bulk copy each, so the consumers never issue scattered
// global loads for them.  Tile widths are chosen so that every tile is
// resident in one wave with equal work.  Eight consumer warps read the
// stage from shared memory: each thread owns 4 columns of one k-step per
// stage, so the three activation-plane loads serve 4 weight vectors.
//
// RMSNorm fusion (rmsnorm, cpu.rs:574-599): with norm_w set, the planes
// encode x[k]*w[k] and each CTA computes rstd = 1/sqrt(mean(x^2)+eps) of the
// whole row; y is multiplied by rstd in the epilogue.  The norm weights are
// read before the dependency wait (they never change).
//
// Every mbarrier wait is bounded (2 s of %globaltimer); a wait that runs out
// sets qg_error_flag and the kernel writes nothing instead of hanging.
#include "qgemv.cuh"
#include "pipeline.cuh"

#include <algorithm>

namespace sb {

constexpr int QG_CONSUMERS = 256;  // 8 consumer warps
constexpr int QG_STAGE = 16384;    // bytes per ring stage
constexpr int QG_NST = 4;          // ring stages
constexpr int QG_CPT = 4;          // columns per consumer thread

__device__ unsigned qg_error_flag = 0;

__device__ __forceinline__ void consumer_sync() { named_sync<QG_CONSUMERS>(); }  // 1: a bounded wait ran out

// Epilogues whose input is RMSNorm-fused (QKV, SwiGLU, logits).
__host__ __device__ constexpr bool epi_has_norm(int epi) {
    return epi == QEPI_QKV || epi == QEPI_SWIGLU || epi == QEPI_LOGITS;
}

// Activation quads each consumer thread holds per prologue batch (fewer with
// a fused norm, whose weights take registers too).
__host__ __device__ constexpr int qg_quads_per_thread(int M, bool norm) {
    return (M == 1 ? 6 : (M == 2 ? 4 : (M == 3 ? 2 : 1))) * (norm ? 1 : 2);
}
// Whole rows fit one register batch: the only case in which the producer
// copies the f32 rows into shared memory (the planes then overwrite them).
__host__ __device__ constexpr bool qg_row_in_smem(int M, int KS, bool norm) {
    return KS * 4 <= qg_quads_per_thread(M, norm) * QG_CONSUMERS;
}

struct QGSmem {
    // Offsets inside the dynamic shared memory block.  `xp` holds the byte
    // planes (plane (m,p) at (3m+p)*16*KS bytes); when the rows come in by
    // bulk copy it first receives them (row m at m*64*KS bytes).  The column
    // partial sums reuse the ring once its last stage is consumed.
    size_t ring, xp, ys, pre, rowinfo, bars, total;
};

__host__ __device__ inline QGSmem qg_layout(int M, int KS, int TN, bool norm) {
    QGSmem L;
    L.ring = 0;
    L.xp = (size_t)QG_NST * QG_STAGE;
    L.ys = L.xp + (size_t)M * (qg_row_in_smem(M, KS, norm) ? 64 : 48) * KS;
    L.pre = L.ys + (size_t)M * TN * 4;  // residual tile preloaded for the RESID epilogue
    L.rowinfo = (L.pre + (size_t)M * TN * 4 + 15) & ~(size_t)15;
    // rowinfo: rstd[M] (double), shift[M] (int), reduction scratch [8][M][2] doubles
    L.bars = L.rowinfo + (size_t)M * 16 + (size_t)8 * M * 2 * 8;
    L.total = L.bars + (2 * QG_NST + 1) * 8;  // full[], empty[], x
    return L;
}

size_t qgemv_smem_bytes(int M, int KS, int TN, bool norm) { return qg_layout(M, KS, TN, norm).total; }

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
            const float4 t = __ldg(reinterpret_cast<const float4 *>(xr + k0));
            v[0] = t.x, v[1] = t.y, v[2] = t.z, v[3] = t.w;
        } else {
#pragma unroll
            for (int i = 0; i < 4; i++) v[i] = (k0 + i < K) ? __ldg(xr + k0 + i) : 0.0f;
        }
    }
}

__device__ __forceinline__ void load_norm_quad(const QGemvArgs &a, int q, float nw[4]) {
    const int K = a.w.K, k0 = q * 4;
    if (!a.norm_w) {
        nw[0] = nw[1] = nw[2] = nw[3] = 1.0f;
        return;
    }
    if (k0 + 4 <= K && ((reinterpret_cast<uintptr_t>(a.norm_w + k0) & 15) == 0)) {
        const float4 t = __ldg(reinterpret_cast<const float4 *>(a.norm_w + k0));
        nw[0] = t.x, nw[1] = t.y, nw[2] = t.z, nw[3] = t.w;
    } else {
#pragma unroll
        for (int i = 0; i < 4; i++) nw[i] = (k0 + i < K) ? __ldg(a.norm_w + k0 + i) : 0.0f;
    }
}


// Quads (4 elements) of one activation row that each consumer thread keeps
// in registers.  Without a fused norm the norm-weight registers hold
// activations instead.
template <int M, bool NORM>
struct QgPro {
    static constexpr int QB = qg_quads_per_thread(M, NORM);
    float4 nv[NORM ? QB : 1];  // norm weights (loaded before the dependency wait)
    float4 xv[M][QB];          // activations of the current batch
};

__device__ __forceinline__ float4 f4_zero() { return make_float4(0.0f, 0.0f, 0.0f, 0.0f); }

template <int M, bool NORM>
__device__ __forceinline__ void pro_load_norm(const QGemvArgs &a, int q0, QgPro<M, NORM> &P) {
    if (!NORM) return;
    const int K = a.w.K, nq = a.w.KS * 4;
#pragma unroll
    for (int j = 0; j < QgPro<M, NORM>::QB; j++) {
        const int q = q0 + j * QG_CONSUMERS;
        float nw[4] = {1.0f, 1.0f, 1.0f, 1.0f};
        if (q < nq) load_norm_quad(a, q, nw);
        P.nv[NORM ? j : 0] = (q < nq && q * 4 < K) ? make_float4(nw[0], nw[1], nw[2], nw[3]) : f4_zero();
    }
}

// Activations from global memory (general path) or from the rows the
// producer copied into shared memory (xs != nullptr, one batch only).
template <int M, bool NORM>
__device__ __forceinline__ void pro_load_x(const QGemvArgs &a, int q0, QgPro<M, NORM> &P, const float *xs, int KS) {
    const int nq = KS * 4, K = a.w.K;
#pragma unroll
    for (int j = 0; j < QgPro<M, NORM>::QB; j++) {
        const int q = q0 + j * QG_CONSUMERS;
#pragma unroll
        for (int m = 0; m < M; m++) {
            float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            if (q < nq) {
                if (xs) {
                    if (m < a.M && q * 4 < K) {  // rows are K floats (K % 4 == 0 on this path)
                        const float4 t = reinterpret_cast<const float4 *>(xs + (size_t)m * 16 * KS)[q];
                        v[0] = t.x, v[1] = t.y, v[2] = t.z, v[3] = t.w;
                    }
                } else {
                    load_quad<M>(a, m, q, v);
                }
            }
            P.xv[m][j] = make_float4(v[0], v[1], v[2], v[3]);
        }
    }
}

// Builds the fixed-point byte planes of the M activation rows in shared
// memory and the per-row rstd / exponent.  Consumer threads only.  P holds
// the norm weights of the first batch, loaded before the dependency wait.
template <int M, bool NORM>
__device__ void qg_prologue(const QGemvArgs &a, uint8_t *smem, const QGSmem &L, QgPro<M, NORM> &P, const float *xs) {
    constexpr int QB = QgPro<M, NORM>::QB;
    const int KS = a.w.KS, K = a.w.K;
    const int nq = KS * 4;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const bool one_batch = nq <= QB * QG_CONSUMERS;
    uint32_t *planes = reinterpret_cast<uint32_t *>(smem + L.xp);
    double *rstd = reinterpret_cast<double *>(smem + L.rowinfo);
    int *shift = reinterpret_cast<int *>(smem + L.rowinfo + (size_t)M * 8);
    double *scratch = reinterpret_cast<double *>(smem + L.rowinfo + (size_t)M * 16);

    // pass 1: sum of squares and max |x*w| per row, QB quads per load batch
    float ssq[M], amx[M];
#pragma unroll
    for (int m = 0; m < M; m++) ssq[m] = 0.0f, amx[m] = 0.0f;
    for (int q0 = tid; q0 < nq; q0 += QB * QG_CONSUMERS) {
        if (q0 != tid) pro_load_norm<M, NORM>(a, q0, P);
        pro_load_x<M, NORM>(a, q0, P, xs, KS);
#pragma unroll
        for (int j = 0; j < QB; j++)
#pragma unroll
            for (int m = 0; m < M; m++) {
                const float4 x = P.xv[m][j];
                const float4 w = NORM ? P.nv[NORM ? j : 0] : make_float4(1.f, 1.f, 1.f, 1.f);
                ssq[m] = fmaf(x.x, x.x, fmaf(x.y, x.y, fmaf(x.z, x.z, fmaf(x.w, x.w, ssq[m]))));
                amx[m] = fmaxf(amx[m], fmaxf(fmaxf(fabsf(__fmul_rn(x.x, w.x)), fabsf(__fmul_rn(x.y, w.y))),
                                             fmaxf(fabsf(__fmul_rn(x.z, w.z)), fabsf(__fmul_rn(x.w, w.w)))));
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
    consumer_sync();  // also: every thread has read its x from shared memory
    if (tid < M) {
        const int m = tid;
        double s = 0.0, x = 0.0;
        for (int w = 0; w < QG_CONSUMERS / 32; w++) {
            s += scratch[(w * M + m) * 2 + 0];
            x = fmax(x, scratch[(w * M + m) * 2 + 1]);
        }
        // rmsnorm (cpu.rs:582-588): mean of squares, rstd = 1/sqrt(mean+eps), f64.
        rstd[m] = NORM ? 1.0 / sqrt(s / (double)K + (double)a.eps) : 1.0;
        int e = 0;
        if (x > 0.0) frexp(x, &e);        // x = f * 2^e, f in [0.5, 1)
        int sh = (x > 0.0) ? 22 - e : 0;  // |a * 2^sh| < 2^22
        shift[m] = sh < -126 ? -126 : (sh > 126 ? 126 : sh);
    }
    consumer_sync();
    // pass 2: quantize to three byte planes (registers still hold a single batch)
    for (int q0 = tid; q0 < nq; q0 += QB * QG_CONSUMERS) {
        if (!one_batch) {
            pro_load_norm<M, NORM>(a, q0, P);
            pro_load_x<M, NORM>(a, q0, P, nullptr, KS);
        }
#pragma unroll
        for (int j = 0; j < QB; j++) {
            const int q = q0 + j * QG_CONSUMERS;
            if (q >= nq) continue;
#pragma unroll
            for (int m = 0; m < M; m++) {
                const float sc = __int_as_float((shift[m] + 127) << 23);  // 2^shift, exact
                const float xs4[4] = {P.xv[m][j].x, P.xv[m][j].y, P.xv[m][j].z, P.xv[m][j].w};
                const float4 wv = NORM ? P.nv[NORM ? j : 0] : make_float4(1.f, 1.f, 1.f, 1.f);
                const float ws[4] = {wv.x, wv.y, wv.z, wv.w};
                uint32_t w0 = 0, w1 = 0, w2 = 0;
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    // round-to-nearest-even to an integer: |t| < 2^22, so t + 1.5*2^23
                    // lands in [2^23, 2^24) where the float ulp is 1.
                    const float t = __fmul_rn(__fmul_rn(xs4[i], ws[i]), sc);
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
}

template <int M, int EPI>
__device__ void qg_epilogue(const QGemvArgs &a, const float *ys, int tile, const float *pre) {
    const int TN = a.w.TN, tid = threadIdx.x;
    for (int it = tid; it < M * TN; it += QG_CONSUMERS) {
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
                *o = __fadd_rn(pre ? pre[m * TN + c] : *o, y);
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


// Reduce the CTA's partial sums of one tile (stages [first, first+n) of it),
// then either finish the tile (epilogue) or, when other CTAs hold the rest of
// its K range, add the exact int64 partial to the tile accumulator; the CTA
// that completes the tile's stage count runs the epilogue.  Every consumer
// thread calls this at the same points (it contains consumer barriers).

template <int M, int EPI, bool GROUPED>
__global__ void __launch_bounds__(QG_THREADS, M <= 2 ? 2 : 1) qgemv_kernel(const QGemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int KS = a.w.KS, TN = a.w.TN, K = a.w.K;
    constexpr bool NORM = epi_has_norm(EPI);
    const QGSmem L = qg_layout(M, KS, TN, NORM);
    const int tid = threadIdx.x;
    const int tile = blockIdx.x;
    const int TPK = TN / QG_CPT;              // threads per k-step
    const int KPS = QG_STAGE / (TN * 16);     // k-steps per stage (= QG_CONSUMERS / TPK)
    const int nstages = (KS + KPS - 1) / KPS;
    const size_t slab_bytes = (size_t)KS * TN * 16;
    const uint8_t *slab = reinterpret_cast<const uint8_t *>(a.w.w + (size_t)tile * KS * TN);
    const uint32_t bars = smem_u32(smem + L.bars);  // full[QG_NST], empty[QG_NST], x
    const uint32_t xbar = bars + 8 * (2 * QG_NST);
    const uint32_t ring = smem_u32(smem + L.ring);
    // The activation rows come in by TMA when they are f32 rows of a whole
    // number of 16-byte chunks and fit one register batch of the prologue.
    const bool xtma = !a.x_bf16 && (K & 3) == 0 && (a.ldx & 3) == 0 &&
                      ((reinterpret_cast<uintptr_t>(a.x) & 15) == 0) &&
                      qg_row_in_smem(M, KS, NORM);
    __shared__ int s_failed;

    if (tid == 0) {
        for (int i = 0; i < QG_NST; i++) {
            mbar_init(bars + 8 * i, 1);                            // full: producer arrival + tx bytes
            mbar_init(bars + 8 * (QG_NST + i), QG_CONSUMERS / 32);  // empty: one arrival per consumer warp
        }
        mbar_init(xbar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        s_failed = 0;
    }
    __syncthreads();
    pdl_launch_dependents();

    if (tid >= QG_CONSUMERS) {
        // ---- producer warp
        if (tid == QG_CONSUMERS) {
            const int first = min(nstages, QG_NST);
            for (int s = 0; s < first; s++) {  // weights never change: before the dependency wait
                const uint32_t bytes = (uint32_t)min((size_t)QG_STAGE, slab_bytes - (size_t)s * QG_STAGE);
                mbar_expect_tx(bars + 8 * s, bytes);
                tma_load_1d(ring + s * QG_STAGE, slab + (size_t)s * QG_STAGE, bytes, bars + 8 * s);
            }
            pdl_wait();
            if (xtma) {
                const uint32_t row = (uint32_t)K * 4;
                mbar_expect_tx(xbar, row * (uint32_t)a.M);
                for (int m = 0; m < a.M; m++)
                    tma_load_1d(smem_u32(smem + L.xp + (size_t)m * 64 * KS),
                                reinterpret_cast<const float *>(a.x) + (size_t)m * a.ldx, row, xbar);
            }
            for (int s = QG_NST; s < nstages; s++) {
                const int slot = s % QG_NST;
                if (!mbar_wait(bars + 8 * (QG_NST + slot), ((s / QG_NST) - 1) & 1)) {
                    atomicOr(&qg_error_flag, 1u);
                    break;
                }
                const uint32_t bytes = (uint32_t)min((size_t)QG_STAGE, slab_bytes - (size_t)s * QG_STAGE);
                mbar_expect_tx(bars + 8 * slot, bytes);
                tma_load_1d(ring + slot * QG_STAGE, slab + (size_t)s * QG_STAGE, bytes, bars + 8 * slot);
            }
        }
        return;
    }

    // ---- consumer warps
    QgPro<M, NORM> pro;
    pro_load_norm<M, NORM>(a, tid, pro);  // norm weights never change: load before the wait
    pdl_wait();
    // RESID: read the residual tile now, so the epilogue does not wait for it.
    float *pre = nullptr;
    if (EPI == QEPI_RESID) {
        pre = reinterpret_cast<float *>(smem + L.pre);
        for (int it = tid; it < M * TN; it += QG_CONSUMERS) {
            const int m = it / TN, n = tile * TN + (it - m * TN);
            pre[it] = (m < a.M && n < a.w.N) ? a.out[(size_t)m * a.ldo + n] : 0.0f;
        }
    }
    // A timed-out wait stops all further waiting and computing, but every
    // thread still makes the same consumer-barrier calls so none blocks.
    bool failed = false;
    if (xtma && !mbar_wait(xbar, 0)) {
        atomicOr(&qg_error_flag, 1u);
        s_failed = 1;
        failed = true;
    }
    qg_prologue<M, NORM>(a, smem, L, pro, xtma ? reinterpret_cast<const float *>(smem + L.xp) : nullptr);
    consumer_sync();

    const uint4 *planes4 = reinterpret_cast<const uint4 *>(smem + L.xp);
    const uint4 *ring4 = reinterpret_cast<const uint4 *>(smem + L.ring);
    const int ksl = tid / TPK, c0 = tid % TPK;
    const int lane = tid & 31, warp = tid >> 5;
    int acc[M][QG_CPT][3];
    double accd[M][QG_CPT];
#pragma unroll
    for (int m = 0; m < M; m++)
#pragma unroll
        for (int j = 0; j < QG_CPT; j++) acc[m][j][0] = acc[m][j][1] = acc[m][j][2] = 0, accd[m][j] = 0.0;
    const int R = GROUPED ? a.w.group / 16 : 1;
    const int NG = GROUPED ? KS / R : 0;
    const float *gs = GROUPED ? a.w.gscale + (size_t)tile * NG * TN + c0 : nullptr;

    int slot = 0, phase = 0;
    for (int s = 0; s < nstages; s++) {
        if (!failed && !mbar_wait(bars + 8 * slot, phase)) {
            atomicOr(&qg_error_flag, 1u);
            s_failed = 1;
            failed = true;
        }
        const int ks = s * KPS + ksl;
        if (!failed && ks < KS) {
            const uint4 *wst = ring4 + (size_t)slot * (QG_STAGE / 16) + ksl * TN + c0;
            uint4 w[QG_CPT];
#pragma unroll
            for (int j = 0; j < QG_CPT; j++) w[j] = wst[j * TPK];
#pragma unroll
            for (int m = 0; m < M; m++) {
                const uint4 p0 = planes4[(size_t)(m * 3 + 0) * KS + ks];
                const uint4 p1 = planes4[(size_t)(m * 3 + 1) * KS + ks];
                const uint4 p2 = planes4[(size_t)(m * 3 + 2) * KS + ks];
#pragma unroll
                for (int j = 0; j < QG_CPT; j++) dot16(w[j], p0, p1, p2, acc[m][j][0], acc[m][j][1], acc[m][j][2]);
            }
            if (GROUPED) {
#pragma unroll
                for (int j = 0; j < QG_CPT; j++) {
                    const double g = (double)__ldg(gs + (size_t)(ks / R) * TN + j * TPK);
#pragma unroll
                    for (int m = 0; m < M; m++) {
                        accd[m][j] += (double)combine_planes(acc[m][j][0], acc[m][j][1], acc[m][j][2]) * g;
                        acc[m][j][0] = acc[m][j][1] = acc[m][j][2] = 0;
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0 && !failed) mbar_arrive(bars + 8 * (QG_NST + slot));
        if (++slot == QG_NST) slot = 0, phase ^= 1;
    }

    // Reduce the partial sums of every column in a fixed order: across the
    // lanes of a warp that share columns (shuffles), then across warps
    // through shared memory (the ring, whose last stage has been consumed).
    consumer_sync();
    const double *rstd = reinterpret_cast<const double *>(smem + L.rowinfo);
    const int *shift = reinterpret_cast<const int *>(smem + L.rowinfo + (size_t)M * 8);
    float *ys = reinterpret_cast<float *>(smem + L.ys);
    const int wpk = TPK >= 32 ? TPK / 32 : 1;       // warps spanning one k-step
    const int ngroups = (QG_CONSUMERS / 32) / wpk;   // warp groups holding the same columns
    const int wgrp = warp / wpk;
    if (GROUPED) {
        double *red = reinterpret_cast<double *>(smem + L.ring);
#pragma unroll
        for (int m = 0; m < M; m++)
#pragma unroll
            for (int j = 0; j < QG_CPT; j++) {
                double v = accd[m][j];
                for (int o = TPK; o < 32; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                if (lane < TPK || TPK >= 32) red[((size_t)m * ngroups + wgrp) * TN + c0 + j * TPK] = v;
            }
        consumer_sync();
        if (tid < TN) {
#pragma unroll
            for (int m = 0; m < M; m++) {
                double t = 0.0;
                for (int g = 0; g < ngroups; g++) t += red[((size_t)m * ngroups + g) * TN + tid];
                ys[m * TN + tid] = (float)(t * pow2_neg(shift[m]) * rstd[m]);
            }
        }
    } else {
        long long *red = reinterpret_cast<long long *>(smem + L.ring);
#pragma unroll
        for (int m = 0; m < M; m++)
#pragma unroll
            for (int j = 0; j < QG_CPT; j++) {
                long long v = combine_planes(acc[m][j][0], acc[m][j][1], acc[m][j][2]);
                for (int o = TPK; o < 32; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                if (lane < TPK || TPK >= 32) red[((size_t)m * ngroups + wgrp) * TN + c0 + j * TPK] = v;
            }
        consumer_sync();
        if (tid < TN) {
#pragma unroll
            for (int m = 0; m < M; m++) {
                long long t = 0;
                for (int g = 0; g < ngroups; g++) t += red[((size_t)m * ngroups + g) * TN + tid];
                const float sc = (EPI == QEPI_SWIGLU && (tid & 31) >= 16) ? a.w.scale_up : a.w.scale;
                ys[m * TN + tid] = gemv_out(t, gemv_factor(shift[m], sc, rstd[m]));
            }
        }
    }
    consumer_sync();
    if (s_failed) return;  // a bounded wait ran out: qg_error_flag is set, nothing is written
    qg_epilogue<M, EPI>(a, ys, tile, pre);
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
    const size_t smem = qgemv_smem_bytes(1, KS, 64, false) + 1024;
    int per_sm = (int)std::min<size_t>(2, (size_t)dp.max_smem_optin / smem);
    per_sm = std::max(per_sm, 1);
    const int slots = dp.sm_count * per_sm;
    const int cands[5] = {16, 32, 64, 128, 256};
    for (int i = 0; i < 5; i++) {
        const int tn = cands[i];
        if (tn < min_tn) continue;
        if (ceil_div(N, tn) <= slots) return tn;
    }
    return 256;
}

int qgemv_error_peek(unsigned *host, cudaStream_t st) {
    SB_CUDA_TRY(cudaMemcpyFromSymbolAsync(host, qg_error_flag, sizeof(unsigned), 0, cudaMemcpyDeviceToHost, st));
    return SB_OK;
}

int qgemv_check_error() {
    unsigned f = 0;
    SB_CUDA_TRY(cudaMemcpyFromSymbol(&f, qg_error_flag, sizeof f));
    if (f) {
        const unsigned zero = 0;
        cudaMemcpyToSymbol(qg_error_flag, &zero, sizeof zero);
        return set_error(SB_ERR_TIMEOUT, "qgemv: a bounded shared-memory pipeline wait timed out");
    }
    return SB_OK;
}

template <int M, int EPI, bool GROUPED>
static int launch_inst(const QGemvArgs &a, cudaStream_t st, bool pdl) {
    const size_t smem = qgemv_smem_bytes(M, a.w.KS, a.w.TN, epi_has_norm(EPI));
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
    SB_CHECK(a.w.TN >= 16 && a.w.TN <= 256 && (a.w.TN & (a.w.TN - 1)) == 0, SB_ERR_SHAPE,
             "qgemv: bad tile width %d", a.w.TN);
    SB_CHECK(a.norm_w == nullptr || epi_has_norm(epi), SB_ERR_ARG, "qgemv: epilogue %d takes no fused RMSNorm", epi);
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
