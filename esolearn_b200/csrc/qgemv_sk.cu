// Split-K GEMV for 1-4 rows of a per-tensor int8 weight with 128-column
// tiles (the op-level matmul_i8_f32, store or bias epilogue).  With one CTA
// per tile, as qgemv_kernel runs it, a 4096-column weight has 32 CTAs on
// 148 SMs and the call is bound by one CTA streaming a whole tile.  Here
// CTA (tile, split) takes a run of k-steps of one tile:
//   1. every CTA reads its rows in full and derives the row exponent the
//      GEMV uses (max |x| -> 2^shift, |x * 2^shift| < 2^22), so all splits
//      share one fixed-point scale;
//   2. it quantizes its own k-steps into the three byte planes (A0, A1
//      unsigned, A2 signed, a = A0 + 2^8 A1 + 2^16 A2) in shared memory;
//   3. its 256 threads stream the tile's weights for those k-steps (column
//      tid % 128, alternate k-steps per half) and multiply them against the
//      planes with dp4a (exact int32);
//   4. the exact column sums go into an int64 workspace with atomics
//      (integer addition: the result does not depend on the order);
//   5. the last split of a tile to finish (arrival counter) scales the sums
//      once in f64, stores the row (plus bias), and clears the workspace.
// So the output equals the one-CTA-per-tile GEMV's bit for bit.
#include "pipeline.cuh"
#include "qgemv.cuh"

#include <algorithm>

namespace sb {

namespace {

constexpr int SK_THREADS = 256;
constexpr int SK_TN = 128;
constexpr int SK_MAX_KSP = 64;  // k-steps of 16 per split, at most

template <int M, int EPI>
__global__ void __launch_bounds__(SK_THREADS) qsk_kernel(const QGemvArgs a, long long *__restrict__ sums,
                                                         unsigned *__restrict__ counters, int kps) {
    __shared__ uint4 planes[M][3][SK_MAX_KSP];
    __shared__ float s_red[SK_THREADS / 32][M];
    __shared__ int s_shift[M];
    __shared__ long long s_part[M][SK_TN];
    __shared__ int s_last;
    const int tile = blockIdx.x, sp = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int K = a.w.K, KS = a.w.KS, N = a.w.N;
    const int ks0 = sp * kps, ks1 = min(KS, ks0 + kps), nks = ks1 - ks0;
    const int ld = a.w.ntiles * SK_TN;

    // 1. max |x| of every row over all of K
    float amx[M];
#pragma unroll
    for (int m = 0; m < M; m++) amx[m] = 0.f;
    if (a.x_bf16) {
        const __nv_bfloat16 *x = reinterpret_cast<const __nv_bfloat16 *>(a.x);
        const bool vec = ((reinterpret_cast<uintptr_t>(x) | ((size_t)a.ldx * 2)) & 15) == 0 && K % 8 == 0;
#pragma unroll
        for (int m = 0; m < M; m++) {
            const __nv_bfloat16 *r = x + (size_t)m * a.ldx;
            if (vec) {
                for (int i = tid; i < K / 8; i += SK_THREADS) {
                    const uint4 u = __ldg(reinterpret_cast<const uint4 *>(r) + i);
                    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
                    for (int j = 0; j < 4; j++)
                        amx[m] = fmaxf(amx[m], fmaxf(fabsf(__uint_as_float(w[j] << 16)),
                                                     fabsf(__uint_as_float(w[j] & 0xffff0000u))));
                }
            } else {
                for (int i = tid; i < K; i += SK_THREADS) amx[m] = fmaxf(amx[m], fabsf(__bfloat162float(r[i])));
            }
        }
    } else {
        const float *x = reinterpret_cast<const float *>(a.x);
        const bool vec = ((reinterpret_cast<uintptr_t>(x) | ((size_t)a.ldx * 4)) & 15) == 0 && K % 4 == 0;
#pragma unroll
        for (int m = 0; m < M; m++) {
            const float *r = x + (size_t)m * a.ldx;
            if (vec) {
                for (int i = tid; i < K / 4; i += SK_THREADS) {
                    const float4 f = __ldg(reinterpret_cast<const float4 *>(r) + i);
                    amx[m] = fmaxf(amx[m], fmaxf(fmaxf(fabsf(f.x), fabsf(f.y)), fmaxf(fabsf(f.z), fabsf(f.w))));
                }
            } else {
                for (int i = tid; i < K; i += SK_THREADS) amx[m] = fmaxf(amx[m], fabsf(r[i]));
            }
        }
    }
#pragma unroll
    for (int m = 0; m < M; m++) {
        const float v = warp_max_f(amx[m]);
        if (lane == 0) s_red[warp][m] = v;
    }
    __syncthreads();
    if (tid < M) {
        float x = 0.f;
        for (int w = 0; w < SK_THREADS / 32; w++) x = fmaxf(x, s_red[w][tid]);
        int e = 0;
        if (x > 0.f) frexp((double)x, &e);  // x = f * 2^e, f in [0.5, 1)
        const int sh = (x > 0.f) ? 22 - e : 0;  // |a * 2^sh| < 2^22
        s_shift[tid] = sh < -126 ? -126 : (sh > 126 ? 126 : sh);
    }
    __syncthreads();

    // 2. this split's k-steps as byte planes
    for (int idx = tid; idx < M * nks; idx += SK_THREADS) {
        const int m = idx / nks, j = idx - m * nks, k0 = (ks0 + j) * 16;
        const float sc = __int_as_float((s_shift[m] + 127) << 23);  // 2^shift, exact
        uint32_t w0[4] = {0, 0, 0, 0}, w1[4] = {0, 0, 0, 0}, w2[4] = {0, 0, 0, 0};
#pragma unroll
        for (int i = 0; i < 16; i++) {
            const int k = k0 + i;
            float v = 0.f;
            if (k < K)
                v = a.x_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(a.x)[(size_t)m * a.ldx + k])
                             : reinterpret_cast<const float *>(a.x)[(size_t)m * a.ldx + k];
            // round to nearest even: |t| < 2^22, so t + 1.5 * 2^23 lands where the ulp is 1
            const int A = __float_as_int(__fadd_rn(__fmul_rn(v, sc), 12582912.0f)) - 0x4B400000;
            w0[i >> 2] |= (uint32_t)(A & 0xff) << (8 * (i & 3));
            w1[i >> 2] |= (uint32_t)((A >> 8) & 0xff) << (8 * (i & 3));
            w2[i >> 2] |= (uint32_t)((A >> 16) & 0xff) << (8 * (i & 3));
        }
        planes[m][0][j] = make_uint4(w0[0], w0[1], w0[2], w0[3]);
        planes[m][1][j] = make_uint4(w1[0], w1[1], w1[2], w1[3]);
        planes[m][2][j] = make_uint4(w2[0], w2[1], w2[2], w2[3]);
    }
    __syncthreads();

    // 3. weights x planes: column c, k-steps ks0 + g, ks0 + g + 2, ...
    const int c = tid & (SK_TN - 1), g = tid >> 7;
    int acc[M][3];
#pragma unroll
    for (int m = 0; m < M; m++) acc[m][0] = acc[m][1] = acc[m][2] = 0;
    const uint4 *wt = reinterpret_cast<const uint4 *>(a.w.w) + ((size_t)tile * KS + ks0) * SK_TN + c;
    int j = g;
    for (; j + 6 < nks; j += 8) {
        uint4 w[4];
#pragma unroll
        for (int u = 0; u < 4; u++) w[u] = ldg_stream(wt + (size_t)(j + 2 * u) * SK_TN);
#pragma unroll
        for (int u = 0; u < 4; u++)
#pragma unroll
            for (int m = 0; m < M; m++)
                dot16(w[u], planes[m][0][j + 2 * u], planes[m][1][j + 2 * u], planes[m][2][j + 2 * u], acc[m][0],
                      acc[m][1], acc[m][2]);
    }
    for (; j < nks; j += 2) {
        const uint4 w = ldg_stream(wt + (size_t)j * SK_TN);
#pragma unroll
        for (int m = 0; m < M; m++)
            dot16(w, planes[m][0][j], planes[m][1][j], planes[m][2][j], acc[m][0], acc[m][1], acc[m][2]);
    }

    // 4. the two halves' sums, then int64 atomics into the workspace
    if (g == 1)
#pragma unroll
        for (int m = 0; m < M; m++) s_part[m][c] = combine_planes(acc[m][0], acc[m][1], acc[m][2]);
    __syncthreads();
    if (g == 0)
#pragma unroll
        for (int m = 0; m < M; m++) {
            const long long s = s_part[m][c] + combine_planes(acc[m][0], acc[m][1], acc[m][2]);
            if (s != 0)
                atomicAdd(reinterpret_cast<unsigned long long *>(sums + (size_t)m * ld + tile * SK_TN + c),
                          (unsigned long long)s);
        }

    // 5. the tile's last split scales, stores and clears
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const unsigned prev = atomicAdd(counters + tile, 1u);
        s_last = prev == gridDim.y - 1;
        if (s_last) counters[tile] = 0u;  // ready for the next call
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int idx = tid; idx < M * SK_TN; idx += SK_THREADS) {
        const int m = idx / SK_TN, cc = idx - m * SK_TN, n = tile * SK_TN + cc;
        long long *p = sums + (size_t)m * ld + n;
        const long long t = __ldcg(p);
        *p = 0;
        if (n < N) {
            const float y = gemv_out(t, gemv_factor(s_shift[m], a.w.scale, 1.0));
            a.out[(size_t)m * a.ldo + n] = EPI == QEPI_BIAS ? __fadd_rn(y, a.bias[n]) : y;
        }
    }
}

template <int EPI>
int qsk_dispatch(const QGemvArgs &a, long long *sums, unsigned *counters, int kps, int S, cudaStream_t st) {
    const dim3 grid(a.w.ntiles, S);
    switch (a.M) {
    case 1: qsk_kernel<1, EPI><<<grid, SK_THREADS, 0, st>>>(a, sums, counters, kps); break;
    case 2: qsk_kernel<2, EPI><<<grid, SK_THREADS, 0, st>>>(a, sums, counters, kps); break;
    case 3: qsk_kernel<3, EPI><<<grid, SK_THREADS, 0, st>>>(a, sums, counters, kps); break;
    case 4: qsk_kernel<4, EPI><<<grid, SK_THREADS, 0, st>>>(a, sums, counters, kps); break;
    default: return set_error(SB_ERR_SHAPE, "qgemv (split-K): M=%d outside 1..%d", a.M, QG_MAX_M);
    }
    SB_CUDA_TRY(cudaGetLastError());
    return SB_OK;
}

// k-steps per split: about two CTAs per SM over the whole grid, at least 8
// (one 16 KB unit of a tile) and at most SK_MAX_KSP.
int qsk_kps(const QWeightDesc &w) {
    const int want = ceil_div(w.KS * w.ntiles, 2 * device_props().sm_count);
    return std::max(8, std::min(SK_MAX_KSP, want));
}

}  // namespace

bool qgemv_splitk_wanted(const QWeightDesc &w, int M) {
    return M >= 1 && M <= QG_MAX_M && w.TN == SK_TN && w.group == 0 && w.ntiles < device_props().sm_count &&
           ceil_div(w.KS, qsk_kps(w)) > 1;
}

size_t qgemv_splitk_ws_bytes(const QWeightDesc &w, int M) {
    return sizeof(long long) * (size_t)M * w.ntiles * SK_TN + sizeof(unsigned) * (size_t)w.ntiles;
}

int qgemv_splitk_launch(int epi, const QGemvArgs &a, void *ws, cudaStream_t st) {
    SB_CHECK(a.w.w && a.x && a.out && ws, SB_ERR_ARG, "qgemv (split-K): null argument");
    SB_CHECK(a.w.TN == SK_TN && a.w.group == 0 && a.norm_w == nullptr, SB_ERR_UNSUPPORTED,
             "qgemv (split-K): needs a per-tensor weight of 128-column tiles, no fused norm");
    SB_CHECK(epi == QEPI_STORE || (epi == QEPI_BIAS && a.bias), SB_ERR_ARG, "qgemv (split-K): epilogue %d", epi);
    const int kps = qsk_kps(a.w), S = ceil_div(a.w.KS, kps);
    long long *sums = static_cast<long long *>(ws);
    unsigned *counters = reinterpret_cast<unsigned *>(sums + (size_t)a.M * a.w.ntiles * SK_TN);
    return epi == QEPI_BIAS ? qsk_dispatch<QEPI_BIAS>(a, sums, counters, kps, S, st)
                            : qsk_dispatch<QEPI_STORE>(a, sums, counters, kps, S, st);
}

}  // namespace sb
