// Batched int8 linear on tcgen05 tensor cores: the batched-decode form of
// matmul_i8_f32 (backend/mod.rs:521-533, CPU cpu.rs:1129-1160) for 5-64 rows.
//
// Arithmetic.  Exactly the fixed point of the GEMV (qgemv.cu): each row is
// scaled by a power of two so |a * 2^s| < 2^22 and rounded to an integer A;
// here it is offset to U = A + 2^23 in [0, 2^24) and split into three
// UNSIGNED byte planes.  The tensor cores multiply the signed int8 weights
// (A operand, 128 output columns x K) with the unsigned planes plus one
// all-ones row (B operand, 3M+1 rows x K) into int32 accumulators in TMEM
// (tcgen05.mma kind::i8); |each accumulator| <= K * 127 * 255 < 2^31 for
// K <= 32768.  Per output column and row:
//   sum_k w a 2^s = D[plane0] + 2^8 D[plane1] + 2^16 D[plane2] - 2^23 D[ones]
// (B rows: the ones row first, then the three planes of each activation row)
// exactly, so results equal the GEMV path bit for bit whenever the row
// exponents agree.
//
// Data movement.  A producer thread streams 32 KB stages of the packed weight
// (the same tile-major 16 KB units as the persistent decode step, split evenly
// over the CTAs) together with the matching 16-k-chunk slice of the planes
// through a ring of shared-memory slots with 1-D TMA bulk copies.  The packed
// tile layout [k/16][128 columns][16 bytes] already is the K-major
// no-swizzle core-matrix layout the MMA reads (8 rows x 16 bytes per core
// matrix, 128 B between row groups, 2 KB between k chunks).  One thread
// issues the MMAs of a stage and commits them to the slot's "empty" barrier,
// so the tensor core releases the slot.  At the end of a tile segment four
// warps drain TMEM (tcgen05.ld, one output column per lane; two accumulator
// buffers, so the next segment's MMAs run meanwhile), recombine the planes
// and add the exact int64 column sums into global memory; a finish kernel
// applies the scale, rstd and epilogue and clears the sums.
//
// Every wait is bounded (2 s); a wait that runs out sets qgm_error_flag and
// the CTA stops issuing, waits for its tensor-core work and frees TMEM.
#include "qgemm.cuh"

#include <cooperative_groups.h>

#include <algorithm>

#include "pipeline.cuh"
#include "tcgen05.cuh"

namespace sb {
namespace cg = cooperative_groups;

namespace {

constexpr int QGM_TN = 128;
constexpr int QGM_UNIT_KS = 8;      // k-steps per 16 KB work unit (split granularity)
// A stage is two units (16 k-steps, 32 KB of weights) while the plane rows
// are few, one unit beyond QGM_UPS2_NP plane rows so the ring keeps 4+ slots.
constexpr int QGM_UPS2_NP = 112;
constexpr int QGM_THREADS = 192;    // warps 0-3 TMEM drain, 4 MMA, 5 producer
constexpr int QGM_MAX_NST = 6;

__device__ unsigned qgm_error_flag = 0;

__host__ __device__ inline int qgm_ups(int np) { return np <= QGM_UPS2_NP ? 2 : 1; }
__host__ __device__ inline int qgm_wbytes(int np) { return qgm_ups(np) * QGM_UNIT_KS * QGM_TN * 16; }
__host__ __device__ inline int qgm_slot_bytes(int np) { return qgm_wbytes(np) + qgm_ups(np) * QGM_UNIT_KS * np * 16; }

// kind::i8, signed A (weights), unsigned B (planes), s32 accumulate, both K-major.
__device__ __forceinline__ uint32_t qgm_idesc(int n) { return umma_idesc_i8(QGM_TN, n, 1, 0); }
// The CTA's stages: units of 8 k-steps of a 128-column tile, tile-major,
// CTA c takes [c*U/G, (c+1)*U/G), up to `ups` units of one tile per stage.
struct QgmWalk {
    int tile, ut, u, u1, upt, KS, ups;
    __device__ QgmWalk(int KS_, int ntiles, int G, int cta, int ups_) : KS(KS_), ups(ups_) {
        upt = (KS + QGM_UNIT_KS - 1) / QGM_UNIT_KS;
        const int U = ntiles * upt;
        u = (int)((long long)U * cta / G);
        u1 = (int)((long long)U * (cta + 1) / G);
        tile = u / upt;
        ut = u - tile * upt;
    }
    __device__ bool more() const { return u < u1; }
    // Next stage: tile, first k-step, k-steps, and whether it ends the CTA's
    // segment of that tile.
    __device__ void next(int &t, int &k0, int &nks, bool &seg_end) {
        const int n = (ups == 2 && ut + 1 < upt && u + 1 < u1) ? 2 : 1;
        t = tile;
        k0 = ut * QGM_UNIT_KS;
        nks = min(n * QGM_UNIT_KS, KS - k0);
        u += n;
        ut += n;
        if (ut >= upt) ut = 0, tile++;
        seg_end = (u >= u1) || (tile != t);
    }
};

// ---- kernel 0: activation rows -> fixed-point planes ----------------------------
// Plane rows of one 16-k chunk: row 0 is all ones, rows 1+3m .. 3+3m the three
// byte planes of activation row m, the rest zero padding.  Block m < M builds
// row m (RMSNorm-weighted when norm_w is set): every thread keeps up to
// QGM_PL_CHUNKS chunks of 16 values in registers, so the row is read once with
// independent 16-byte loads.  Blocks M.. write the ones row and the padding
// rows of 16 chunks each.
constexpr int QGM_PL_THREADS = 256;
constexpr int QGM_PL_CHUNKS = 8;  // 16-k chunks per thread: K <= 256 * 8 * 16 = 32768
static_assert(QGM_PL_THREADS == 256, "the padding blocks map 16 chunks x 16 rows onto the threads");

__device__ __forceinline__ void qgm_load16(const QGemvArgs &a, int m, int kc, bool vec, float v[16]) {
    const int K = a.w.K, k0 = kc * 16;
    if (a.x_bf16) {
        const __nv_bfloat16 *x = reinterpret_cast<const __nv_bfloat16 *>(a.x) + (size_t)m * a.ldx + k0;
        if (vec && k0 + 16 <= K) {
            const uint4 u0 = __ldg(reinterpret_cast<const uint4 *>(x)), u1 = __ldg(reinterpret_cast<const uint4 *>(x) + 1);
            const uint32_t w[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
            for (int i = 0; i < 8; i++) {
                v[2 * i] = __uint_as_float(w[i] << 16);
                v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
            }
        } else {
#pragma unroll
            for (int i = 0; i < 16; i++) v[i] = k0 + i < K ? __bfloat162float(x[i]) : 0.f;
        }
    } else {
        const float *x = reinterpret_cast<const float *>(a.x) + (size_t)m * a.ldx + k0;
        if (vec && k0 + 16 <= K) {
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float4 f = __ldg(reinterpret_cast<const float4 *>(x) + i);
                v[4 * i] = f.x, v[4 * i + 1] = f.y, v[4 * i + 2] = f.z, v[4 * i + 3] = f.w;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 16; i++) v[i] = k0 + i < K ? x[i] : 0.f;
        }
    }
}

__global__ void __launch_bounds__(QGM_PL_THREADS) qgm_planes_kernel(const QGemvArgs a, QGemmWs ws, int np) {
    pdl_launch_dependents();
    pdl_wait();
    const int K = a.w.K, KS = a.w.KS, M = a.M;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int m = blockIdx.x;
    if (m >= M) {
        // ones row and padding rows of 16 chunks per block: thread -> (chunk, padding row)
        const int npad = np - 3 * M;  // 1 ones row + 0..15 zero rows
        const int kc = (m - M) * 16 + (tid >> 4), j = tid & 15;
        if (kc < KS && j < npad) {
            const int r = j == 0 ? 0 : 3 * M + j;
            const uint32_t one = j == 0 ? 0x01010101u : 0u;
            reinterpret_cast<uint4 *>(ws.planes)[(size_t)kc * np + r] = make_uint4(one, one, one, one);
        }
        return;
    }
    const size_t esz = a.x_bf16 ? 2 : 4;
    const bool vec = ((reinterpret_cast<uintptr_t>(a.x) | ((size_t)a.ldx * esz)) & 15) == 0;
    const bool vecw = a.norm_w && (reinterpret_cast<uintptr_t>(a.norm_w) & 15) == 0;
    __shared__ double red_s[QGM_PL_THREADS / 32];
    __shared__ float red_m[QGM_PL_THREADS / 32];
    __shared__ int s_shift;
    float v[QGM_PL_CHUNKS][16];
    float ssq = 0.f, amx = 0.f;
#pragma unroll
    for (int j = 0; j < QGM_PL_CHUNKS; j++) {
        const int kc = tid + QGM_PL_THREADS * j;
        if (kc >= KS) continue;
        qgm_load16(a, m, kc, vec, v[j]);
#pragma unroll
        for (int i = 0; i < 16; i++) ssq = fmaf(v[j][i], v[j][i], ssq);
        if (a.norm_w) {
            float w[16];
            if (vecw && kc * 16 + 16 <= K) {
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const float4 f = __ldg(reinterpret_cast<const float4 *>(a.norm_w + kc * 16) + i);
                    w[4 * i] = f.x, w[4 * i + 1] = f.y, w[4 * i + 2] = f.z, w[4 * i + 3] = f.w;
                }
            } else {
#pragma unroll
                for (int i = 0; i < 16; i++) w[i] = kc * 16 + i < K ? __ldg(a.norm_w + kc * 16 + i) : 0.f;
            }
#pragma unroll
            for (int i = 0; i < 16; i++) v[j][i] = __fmul_rn(v[j][i], w[i]);
        }
#pragma unroll
        for (int i = 0; i < 16; i++) amx = fmaxf(amx, fabsf(v[j][i]));
    }
    const double s = warp_sum_d((double)ssq);
    const float mx = warp_max_f(amx);
    if (lane == 0) red_s[warp] = s, red_m[warp] = mx;
    __syncthreads();
    if (tid == 0) {
        double st = 0.0, mt = 0.0;
        for (int w = 0; w < QGM_PL_THREADS / 32; w++) st += red_s[w], mt = fmax(mt, (double)red_m[w]);
        // rmsnorm (cpu.rs:582-588): rstd = 1/sqrt(mean(x^2) + eps) in f64
        ws.rstd[m] = a.norm_w ? 1.0 / sqrt(st / (double)K + (double)a.eps) : 1.0;
        int e = 0;
        if (mt > 0.0) frexp(mt, &e);
        const int sh = (mt > 0.0) ? 22 - e : 0;  // |a * 2^sh| < 2^22
        s_shift = sh < -126 ? -126 : (sh > 126 ? 126 : sh);
        ws.shift[m] = s_shift;
    }
    __syncthreads();
    const float sc = __int_as_float((s_shift + 127) << 23);
    // U = A + 2^23 in [0, 2^24): three unsigned byte planes per 16-k chunk
#pragma unroll
    for (int j = 0; j < QGM_PL_CHUNKS; j++) {
        const int kc = tid + QGM_PL_THREADS * j;
        if (kc >= KS) continue;
        uint32_t w[3][4];
#pragma unroll
        for (int q = 0; q < 4; q++) {
            uint32_t b0 = 0, b1 = 0, b2 = 0;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float t = __fmul_rn(v[j][q * 4 + i], sc);
                const int A = __float_as_int(__fadd_rn(t, 12582912.0f)) - 0x4B400000;  // round to nearest even
                const uint32_t U = (uint32_t)(A + (1 << 23));
                b0 |= (U & 0xffu) << (8 * i);
                b1 |= ((U >> 8) & 0xffu) << (8 * i);
                b2 |= ((U >> 16) & 0xffu) << (8 * i);
            }
            w[0][q] = b0, w[1][q] = b1, w[2][q] = b2;
        }
        uint4 *dst = reinterpret_cast<uint4 *>(ws.planes) + (size_t)kc * np + 1 + 3 * m;
#pragma unroll
        for (int p = 0; p < 3; p++) dst[p] = make_uint4(w[p][0], w[p][1], w[p][2], w[p][3]);
    }
}

// ---- kernel 1: weights x planes on the tensor cores -> int64 column sums -------
// TMEM holds two accumulator buffers of ncols columns each: the MMAs of tile
// segment s go to buffer s & 1, so the drain of one segment overlaps the MMAs
// of the next.  A drain warp reads its 32 lanes' plane columns with 16-column
// tcgen05.ld loads and one wait, then recombines every row in registers.
// A drain pass covers 32 rows: columns [0, 112) hold the ones row and rows
// 0-31, columns [96, 208) rows 32-63.
constexpr int QGM_DRAIN_LD = 7;
constexpr int QGM_DRAIN_ROWS = 32;

__global__ void __launch_bounds__(QGM_THREADS, 1)
    qgm_gemm_kernel(const QWeightDesc w, const QGemmWs ws, int M, int np, int nst) {
    extern __shared__ __align__(1024) uint8_t smem[];
    // full[nst], empty[nst], tmem full[2], tmem empty[2], mma done
    __shared__ __align__(8) unsigned long long bars[2 * QGM_MAX_NST + 5];
    __shared__ uint32_t s_tmem;
    __shared__ int s_abort;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x, cta = blockIdx.x;
    const int slot_bytes = qgm_slot_bytes(np), wslot = qgm_wbytes(np), ups = qgm_ups(np);
    const uint32_t b_full = smem_u32(&bars[0]), b_empty = smem_u32(&bars[QGM_MAX_NST]);
    const uint32_t b_tfull = smem_u32(&bars[2 * QGM_MAX_NST]), b_tempty = smem_u32(&bars[2 * QGM_MAX_NST + 2]);
    const uint32_t b_done = smem_u32(&bars[2 * QGM_MAX_NST + 4]);
    const int ncols = np <= 32 ? 32 : (np <= 64 ? 64 : (np <= 128 ? 128 : 256));  // one buffer; two are allocated
    if (tid == 0) {
        for (int i = 0; i < nst; i++) {
            mbar_init(b_full + 8 * i, 1);
            mbar_init(b_empty + 8 * i, 1);  // arrived by tcgen05.commit
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(b_tfull + 8 * i, 1);
            mbar_init(b_tempty + 8 * i, 4);  // one arrival per draining warp
        }
        mbar_init(b_done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        s_abort = 0;
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_tmem)),
                     "r"(2 * ncols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    pdl_launch_dependents();
    const uint32_t tmem = s_tmem;
    const uint32_t ring = smem_u32(smem);

    if (warp == 5) {
        // ---- producer: weights (immutable) may stream before the planes exist
        if (lane == 0) {
            QgmWalk wk(w.KS, w.ntiles, G, cta, ups);
            uint32_t it = 0, slot = 0, par = 0;
            // Fill every slot with its weights first: under programmatic
            // dependent launch this runs while the previous kernels finish.
            // The planes come from the previous kernel, so their copies into
            // the same slots follow griddepcontrol.wait.
            int pk0[QGM_MAX_NST], pnks[QGM_MAX_NST];
            while (it < (uint32_t)nst && wk.more()) {
                int t, k0, nks;
                bool se;
                wk.next(t, k0, nks, se);
                const uint32_t wbytes = (uint32_t)nks * QGM_TN * 16, pbytes = (uint32_t)nks * np * 16;
                mbar_expect_tx(b_full + 8 * it, wbytes + pbytes);
                tma_load_1d(ring + it * slot_bytes,
                            reinterpret_cast<const uint8_t *>(w.w) + ((size_t)t * w.KS + k0) * QGM_TN * 16, wbytes,
                            b_full + 8 * it);
                pk0[it] = k0, pnks[it] = nks;
                it++;
            }
            pdl_wait();
            for (uint32_t i = 0; i < it; i++)
                tma_load_1d(ring + i * slot_bytes + wslot, ws.planes + (size_t)pk0[i] * np * 16,
                            (uint32_t)pnks[i] * np * 16, b_full + 8 * i);
            slot = it % (uint32_t)nst;
            par = it / (uint32_t)nst;
            while (wk.more()) {
                int t, k0, nks;
                bool se;
                wk.next(t, k0, nks, se);
                if (*(volatile int *)&s_abort || !mbar_wait(b_empty + 8 * slot, par ^ 1)) {
                    atomicOr(&qgm_error_flag, 1u);
                    s_abort = 1;
                    break;
                }
                const uint32_t wbytes = (uint32_t)nks * QGM_TN * 16, pbytes = (uint32_t)nks * np * 16;
                const uint32_t dst = ring + slot * slot_bytes;
                mbar_expect_tx(b_full + 8 * slot, wbytes + pbytes);
                tma_load_1d(dst, reinterpret_cast<const uint8_t *>(w.w) + ((size_t)t * w.KS + k0) * QGM_TN * 16, wbytes,
                            b_full + 8 * slot);
                tma_load_1d(dst + wslot, ws.planes + (size_t)k0 * np * 16, pbytes, b_full + 8 * slot);
                it++;
                if (++slot == (uint32_t)nst) slot = 0, par ^= 1;
            }
        }
    } else if (warp == 4) {
        // ---- MMA issuer
        if (lane == 0) {
            QgmWalk wk(w.KS, w.ntiles, G, cta, ups);
            const uint32_t idesc = qgm_idesc(np);
            uint32_t slot = 0, par = 0, seg = 0;
            bool seg_start = true, ok = true;
            while (wk.more() && ok) {
                int t, k0, nks;
                bool se;
                wk.next(t, k0, nks, se);
                const uint32_t buf = seg & 1;
                // the buffer's previous segment (seg - 2) has been drained
                if (seg_start && seg >= 2 && !mbar_wait(b_tempty + 8 * buf, ((seg >> 1) - 1) & 1)) ok = false;
                if (ok && !mbar_wait(b_full + 8 * slot, par)) ok = false;
                if (!ok) {
                    atomicOr(&qgm_error_flag, 1u);
                    s_abort = 1;
                    break;
                }
                tc_fence_after();
                const uint32_t a0 = ring + slot * slot_bytes, p0 = a0 + wslot;
                const uint32_t acc = tmem + buf * (uint32_t)ncols;
                for (int kk = 0; kk < nks / 2; kk++) {
                    const uint64_t da = umma_sdesc(a0 + kk * 2 * QGM_TN * 16, QGM_TN * 16, 128);
                    const uint64_t db = umma_sdesc(p0 + kk * 2 * np * 16, np * 16, 128);
                    umma_i8(acc, da, db, idesc, (seg_start && kk == 0) ? 0u : 1u);
                }
                umma_commit(b_empty + 8 * slot);  // the slot is free once these MMAs complete
                seg_start = false;
                if (se) {
                    umma_commit(b_tfull + 8 * buf);  // this tile segment's sums are complete in TMEM
                    seg++;
                    seg_start = true;
                }
                if (++slot == (uint32_t)nst) slot = 0, par ^= 1;
            }
            // leave no tensor-core work running: this commit tracks every MMA issued
            umma_commit(b_done);
            if (!mbar_wait(b_done, 0)) atomicOr(&qgm_error_flag, 1u);
        }
    } else {
        // ---- warps 0-3: drain TMEM per tile segment into exact int64 column sums
        pdl_wait();  // the previous finish kernel has cleared the sums
        QgmWalk wk(w.KS, w.ntiles, G, cta, ups);
        uint32_t seg = 0;
        const int col = warp * 32 + lane;  // output column within the tile (= TMEM lane)
        const int rows_a = min(M, QGM_DRAIN_ROWS);
        const int nld_a = (3 * rows_a + 1 + 15) >> 4;          // pass A: columns [0, 16 nld_a)
        const int nld_b = M > QGM_DRAIN_ROWS ? (3 * M + 1 - 96 + 15) >> 4 : 0;  // pass B: [96, ...)
        while (wk.more()) {
            int t, k0, nks;
            bool se;
            wk.next(t, k0, nks, se);
            if (!se) continue;
            const uint32_t buf = seg & 1;
            const bool ok = !s_abort && mbar_wait(b_tfull + 8 * buf, (seg >> 1) & 1);
            if (!ok) {
                atomicOr(&qgm_error_flag, 1u);
                s_abort = 1;
                break;
            }
            tc_fence_after();
            const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16) + buf * (uint32_t)ncols;
            long long *out = ws.acc + (size_t)t * QGM_TN + col;
            uint32_t d[QGM_DRAIN_LD * 16];
#pragma unroll
            for (int j = 0; j < QGM_DRAIN_LD; j++)
                if (j < nld_a) tmem_ld16(lane_base + 16 * j, d + 16 * j);
            tmem_wait_ld(d);
            // D[0] = sum_k w over this segment's k range (the ones row)
            const long long ones = (long long)(int)d[0];
#pragma unroll
            for (int m = 0; m < QGM_DRAIN_ROWS; m++) {
                if (m < M) {
                    const long long s = (long long)(int)d[1 + 3 * m] + ((long long)(int)d[2 + 3 * m] << 8) +
                                        ((long long)(int)d[3 + 3 * m] << 16) - (ones << 23);
                    if (s != 0)
                        atomicAdd(reinterpret_cast<unsigned long long *>(out + (size_t)m * ws.ld_acc),
                                  (unsigned long long)s);
                }
            }
            if (nld_b > 0) {
#pragma unroll
                for (int j = 0; j < QGM_DRAIN_LD; j++)
                    if (j < nld_b) tmem_ld16(lane_base + 96 + 16 * j, d + 16 * j);
                tmem_wait_ld(d);
#pragma unroll
                for (int mm = 0; mm < QGM_DRAIN_ROWS; mm++) {
                    const int m = QGM_DRAIN_ROWS + mm;  // columns 1+3m.. = 96 + (1+3mm)..
                    if (m < M) {
                        const long long s = (long long)(int)d[1 + 3 * mm] + ((long long)(int)d[2 + 3 * mm] << 8) +
                                            ((long long)(int)d[3 + 3 * mm] << 16) - (ones << 23);
                        if (s != 0)
                            atomicAdd(reinterpret_cast<unsigned long long *>(out + (size_t)m * ws.ld_acc),
                                      (unsigned long long)s);
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(b_tempty + 8 * buf);  // the segment has left TMEM
            seg++;
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * ncols) : "memory");
}

// ---- kernel 2: scale, epilogue, clear the sums ------------------------------------
// CTA (tile, g) handles rows [g*R, g*R + R) of one 128-column tile; thread
// (c, h) owns column c of rows g*R + h, + 2, + 4, ...  R is picked on the
// host so the grid stays near one wave: these CTAs are short, so many small
// ones are bound by the CTA launch rate and few large ones leave SMs idle.
// Every global value a thread needs is loaded in one batch before the
// dependent work.  The epilogues are those of qgemv.cu for any row count.
constexpr int QGM_FIN_THREADS = 256;

// J = rows per thread (R = 2J rows per CTA); sized arrays keep registers low.
template <int EPI, int J>
__global__ void __launch_bounds__(QGM_FIN_THREADS) qgm_finish_kernel(const QGemvArgs a, const QGemmWs ws) {
    constexpr int QGM_FIN_MAXJ = J;
    constexpr int R = 2 * J;
    __shared__ float ys[R * QGM_TN];  // rows of this CTA, local index
    __shared__ float s_bv[R][QGM_TN / 32];
    __shared__ int s_bi[R][QGM_TN / 32];
    pdl_launch_dependents();
    pdl_wait();
    const int tile = blockIdx.x, tid = threadIdx.x;
    const int m0 = blockIdx.y * R, nr = min(R, a.M - m0);  // rows of this CTA
    const int c = tid & (QGM_TN - 1), h = tid >> 7;        // column, first local row
    const int n = tile * QGM_TN + c;
    const int lane = tid & 31, wic = c >> 5;               // warp index within the row
    // 1. the exact sums and the row factors, all loads in flight together
    long long t[QGM_FIN_MAXJ];
    int sh[QGM_FIN_MAXJ];
    double rs[QGM_FIN_MAXJ];
#pragma unroll
    for (int j = 0; j < QGM_FIN_MAXJ; j++) {
        const int r = h + 2 * j;
        if (r < nr) {
            t[j] = __ldcg(ws.acc + (size_t)(m0 + r) * ws.ld_acc + n);
            sh[j] = ws.shift[m0 + r];
            rs[j] = ws.rstd[m0 + r];
        }
    }
#pragma unroll
    for (int j = 0; j < QGM_FIN_MAXJ; j++) {
        const int r = h + 2 * j;
        if (r < nr) ws.acc[(size_t)(m0 + r) * ws.ld_acc + n] = 0;
    }
    const float sc = (EPI == QEPI_SWIGLU && (c & 31) >= 16) ? a.w.scale_up : a.w.scale;
#pragma unroll
    for (int j = 0; j < QGM_FIN_MAXJ; j++) {
        const int r = h + 2 * j;
        if (r < nr) ys[r * QGM_TN + c] = gemv_out(t[j], gemv_factor(sh[j], sc, rs[j]));
    }
    __syncthreads();
    // 2. epilogue
    if (EPI == QEPI_STORE || EPI == QEPI_LOGITS || EPI == QEPI_BIAS) {
        const float bias = (EPI == QEPI_BIAS && n < a.w.N) ? a.bias[n] : 0.f;
#pragma unroll
        for (int j = 0; j < QGM_FIN_MAXJ; j++) {
            const int r = h + 2 * j;
            if (r < nr && n < a.w.N) {
                const float y = ys[r * QGM_TN + c];
                a.out[(size_t)(m0 + r) * a.ldo + n] = EPI == QEPI_BIAS ? __fadd_rn(y, bias) : y;
            }
        }
    } else if (EPI == QEPI_RESID) {
        float o[QGM_FIN_MAXJ];
#pragma unroll
        for (int j = 0; j < QGM_FIN_MAXJ; j++) {
            const int r = h + 2 * j;
            if (r < nr && n < a.w.N) o[j] = a.out[(size_t)(m0 + r) * a.ldo + n];
        }
#pragma unroll
        for (int j = 0; j < QGM_FIN_MAXJ; j++) {
            const int r = h + 2 * j;
            if (r < nr && n < a.w.N)  // x = x + proj (llama.rs:564,568)
                a.out[(size_t)(m0 + r) * a.ldo + n] = __fadd_rn(o[j], ys[r * QGM_TN + c]);
        }
    } else if (EPI == QEPI_SWIGLU) {
        const int within = n & 31;
        if (within < 16) {
            const int jf = (n >> 5) * 16 + within;
#pragma unroll
            for (int j = 0; j < QGM_FIN_MAXJ; j++) {
                const int r = h + 2 * j;
                if (r < nr && jf < a.F)
                    a.out[(size_t)(m0 + r) * a.ldo + jf] =
                        __fmul_rn(silu_f64(ys[r * QGM_TN + c]), ys[r * QGM_TN + c + 16]);
            }
        }
    } else if (EPI == QEPI_QKV) {
        const int qk = a.q_dim + a.kv_dim;
        int pos[QGM_FIN_MAXJ];
#pragma unroll
        for (int j = 0; j < QGM_FIN_MAXJ; j++) {
            const int r = h + 2 * j;
            pos[j] = r < nr ? a.pos[m0 + r] : -1;
        }
        const bool rope = n < qk;
        const int nn = n < a.q_dim ? n : n - a.q_dim;
        const int d = nn % a.hd, i = d >> 1;
        float cs[QGM_FIN_MAXJ], sn[QGM_FIN_MAXJ];
        int page[QGM_FIN_MAXJ];
#pragma unroll
        for (int j = 0; j < QGM_FIN_MAXJ; j++) {
            const int r = h + 2 * j;
            const bool live = r < nr && pos[j] >= 0 && pos[j] < a.max_pos && n < a.w.N;
            cs[j] = (live && rope) ? a.rope_cos[(size_t)pos[j] * (a.hd / 2) + i] : 0.f;
            sn[j] = (live && rope) ? a.rope_sin[(size_t)pos[j] * (a.hd / 2) + i] : 0.f;
            page[j] = (live && n >= a.q_dim) ? a.page_table[(size_t)(m0 + r) * a.max_pages + pos[j] / a.page_size] : 0;
        }
#pragma unroll
        for (int j = 0; j < QGM_FIN_MAXJ; j++) {
            const int r = h + 2 * j;
            if (!(r < nr && pos[j] >= 0 && pos[j] < a.max_pos && n < a.w.N)) continue;
            const int m = m0 + r;
            const float y = ys[r * QGM_TN + c];
            float val = y;
            if (rope) {
                // rope_with_freqs_preloaded (cpu.rs:650-661)
                const float partner = ys[r * QGM_TN + (c ^ 1)];
                val = (d & 1) ? __fadd_rn(__fmul_rn(partner, sn[j]), __fmul_rn(y, cs[j]))
                              : __fsub_rn(__fmul_rn(y, cs[j]), __fmul_rn(partner, sn[j]));
            }
            if (n < a.q_dim) {
                a.q_out[(size_t)m * a.q_dim + n] = __fmul_rn(val, a.q_scale);
            } else {
                const bool is_k = n < qk;
                const int kn = is_k ? n - a.q_dim : n - qk;
                const int kh = kn / a.hd, dd = kn - kh * a.hd;
                const size_t idx =
                    (((size_t)page[j] * a.n_kv + kh) * a.page_size + pos[j] % a.page_size) * a.hd + dd;
                void *cache = is_k ? a.kcache : a.vcache;
                if (a.kv_f32)
                    reinterpret_cast<float *>(cache)[idx] = val;
                else
                    reinterpret_cast<__nv_bfloat16 *>(cache)[idx] = __float2bfloat16_rn(val);
            }
        }
    }
    if (EPI == QEPI_LOGITS) {
        // per-tile argmax candidate of every row; ties resolve to the larger index
#pragma unroll
        for (int j = 0; j < QGM_FIN_MAXJ; j++) {
            const int r = h + 2 * j;
            if (r >= nr) break;  // uniform over each warp (a warp holds one row parity)
            float best = ys[r * QGM_TN + c];
            int bi = n < a.w.N ? n : -1;
            for (int o = 16; o > 0; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, best, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (oi >= 0 && (bi < 0 || ov > best || (ov == best && oi > bi))) best = ov, bi = oi;
            }
            if (lane == 0) s_bv[r][wic] = best, s_bi[r][wic] = bi;
        }
        __syncthreads();
        if (tid < nr) {
            float bv = s_bv[tid][0];
            int bj = s_bi[tid][0];
            for (int k = 1; k < QGM_TN / 32; k++) {
                const float ov = s_bv[tid][k];
                const int oi = s_bi[tid][k];
                if (oi >= 0 && (bj < 0 || ov > bv || (ov == bv && oi > bj))) bv = ov, bj = oi;
            }
            a.cand_val[(size_t)(m0 + tid) * a.w.ntiles + tile] = bv;
            a.cand_idx[(size_t)(m0 + tid) * a.w.ntiles + tile] = bj;
        }
    }
}

// ---- finish + the next linear's planes, one row per cluster ----------------------
// When a linear's output row is the next linear's input (o -> gate/up with the
// post-attention RMSNorm, gate/up -> down, down -> the next layer's qkv or the
// lm_head with their RMSNorm), one launch finishes the sums and writes the
// next GEMM's byte planes.  The QGF_CLUSTER CTAs of a cluster own one row:
// each finishes a contiguous run of whole 16-feature chunks (sums -> f32,
// residual add or SwiGLU, store; clears the sums) and keeps the values in
// shared memory; the CTAs exchange their partial sum of squares and maximum
// through distributed shared memory and add them in rank order, so every CTA
// derives the same exponent and RMSNorm factor (the planes kernel's rules);
// then each quantizes its run into the planes.
constexpr int QGF_CLUSTER = 8;
constexpr int QGF_THREADS = 256;
constexpr int QGF_J = 16;                                     // features per thread
constexpr int QGF_MAX_PER = QGF_THREADS * QGF_J;             // per CTA
constexpr int QGF_MAX_K = QGF_CLUSTER * QGF_MAX_PER;         // 32768 features per row

template <int EPI>
__global__ void __cluster_dims__(QGF_CLUSTER, 1, 1) __launch_bounds__(QGF_THREADS)
    qgm_finish_planes_kernel(const QGemvArgs a, const QGemmWs ws, const float *norm_next, float eps, int np) {
    static_assert(EPI == QEPI_RESID || EPI == QEPI_SWIGLU, "row finish: residual or SwiGLU");
    __shared__ float vals[QGF_MAX_PER];
    __shared__ double w_ssq[QGF_THREADS / 32];
    __shared__ float w_amx[QGF_THREADS / 32];
    __shared__ double c_ssq;  // this CTA's partials, read by the cluster
    __shared__ float c_amx;
    __shared__ int s_shift;
    pdl_launch_dependents();
    pdl_wait();
    cg::cluster_group cl = cg::this_cluster();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int m = blockIdx.y;
    const int rank = (int)cl.block_rank();
    const int K = EPI == QEPI_SWIGLU ? a.F : a.w.N;  // features of the row = the next linear's K
    const int nchunk = (K + 15) >> 4, cpc = (nchunk + QGF_CLUSTER - 1) / QGF_CLUSTER;
    const int kc0 = min(nchunk, rank * cpc), kc1 = min(nchunk, kc0 + cpc);
    const int f0 = kc0 * 16, f1 = min(K, kc1 * 16), nf = f1 - f0;
    long long *acc = ws.acc + (size_t)m * ws.ld_acc;
    float *out = a.out + (size_t)m * a.ldo;
    const int sh0 = ws.shift[m];
    const double rs0 = ws.rstd[m];
    // 1. finish: every load of the thread in flight together
    if (EPI == QEPI_RESID) {
        long long t[QGF_J];
        float x[QGF_J];
#pragma unroll
        for (int j = 0; j < QGF_J; j++) {
            const int i = tid + QGF_THREADS * j;
            if (i < nf) t[j] = __ldcg(acc + f0 + i), x[j] = out[f0 + i];
        }
        const double f = gemv_factor(sh0, a.w.scale, rs0);
#pragma unroll
        for (int j = 0; j < QGF_J; j++) {
            const int i = tid + QGF_THREADS * j;
            if (i < nf) {
                acc[f0 + i] = 0;
                const float v = __fadd_rn(x[j], gemv_out(t[j], f));  // x + proj (llama.rs:564,568)
                out[f0 + i] = v;
                vals[i] = v;
            }
        }
    } else {
        long long tg[QGF_J], tu[QGF_J];
#pragma unroll
        for (int j = 0; j < QGF_J; j++) {
            const int i = tid + QGF_THREADS * j;
            if (i < nf) {
                const int fi = f0 + i, col = (fi >> 4) * 32 + (fi & 15);
                tg[j] = __ldcg(acc + col), tu[j] = __ldcg(acc + col + 16);
            }
        }
        const double fg = gemv_factor(sh0, a.w.scale, rs0), fu = gemv_factor(sh0, a.w.scale_up, rs0);
#pragma unroll
        for (int j = 0; j < QGF_J; j++) {
            const int i = tid + QGF_THREADS * j;
            if (i < nf) {
                const int fi = f0 + i, col = (fi >> 4) * 32 + (fi & 15);
                acc[col] = 0, acc[col + 16] = 0;
                const float v = __fmul_rn(silu_f64(gemv_out(tg[j], fg)), gemv_out(tu[j], fu));
                out[fi] = v;
                vals[i] = v;
            }
        }
    }
    // padded columns past the last feature hold zero sums (zero weights); the
    // last CTA clears them anyway so the buffer is all zero for the next call
    if (rank == QGF_CLUSTER - 1) {
        const int used = EPI == QEPI_SWIGLU ? ((K + 15) >> 4) * 32 : K;
        for (int n = used + tid; n < a.w.ntiles * QGM_TN; n += QGF_THREADS) acc[n] = 0;
    }
    __syncthreads();
    // 2. this CTA's sum of squares (before the norm weight) and max |value|
    // (after it), as the planes kernel forms them
    float ssq = 0.f, amx = 0.f;
    for (int i = tid; i < nf; i += QGF_THREADS) {
        float v = vals[i];
        if (norm_next) {
            ssq = fmaf(v, v, ssq);
            v = __fmul_rn(v, __ldg(norm_next + f0 + i));
            vals[i] = v;
        }
        amx = fmaxf(amx, fabsf(v));
    }
    const double s = warp_sum_d((double)ssq);
    const float mx = warp_max_f(amx);
    if (lane == 0) w_ssq[warp] = s, w_amx[warp] = mx;
    __syncthreads();
    if (tid == 0) {
        double st = 0.0;
        float mt = 0.f;
        for (int w = 0; w < QGF_THREADS / 32; w++) st += w_ssq[w], mt = fmaxf(mt, w_amx[w]);
        c_ssq = st, c_amx = mt;
    }
    cl.sync();  // partials visible cluster-wide
    if (tid == 0) {
        double st = 0.0, mt = 0.0;
        for (int r = 0; r < QGF_CLUSTER; r++) {  // rank order: the same totals in every CTA
            st += *cl.map_shared_rank(&c_ssq, r);
            mt = fmax(mt, (double)*cl.map_shared_rank(&c_amx, r));
        }
        int e = 0;
        if (mt > 0.0) frexp(mt, &e);
        const int sh = (mt > 0.0) ? 22 - e : 0;  // |a * 2^sh| < 2^22
        s_shift = sh < -126 ? -126 : (sh > 126 ? 126 : sh);
        if (rank == 0) {
            // rmsnorm (cpu.rs:582-588): rstd = 1/sqrt(mean(x^2) + eps) in f64
            ws.rstd[m] = norm_next ? 1.0 / sqrt(st / (double)K + (double)eps) : 1.0;
            ws.shift[m] = s_shift;
        }
    }
    __syncthreads();
    // 3. planes of this CTA's chunks (U = A + 2^23, three unsigned bytes)
    const float sc = __int_as_float((s_shift + 127) << 23);
    for (int kc = kc0 + tid; kc < kc1; kc += QGF_THREADS) {
        const int i0 = (kc - kc0) * 16;
        uint32_t w[3][4];
#pragma unroll
        for (int q = 0; q < 4; q++) {
            uint32_t b0 = 0, b1 = 0, b2 = 0;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int k = i0 + q * 4 + i;
                const float v = f0 + k < K ? vals[k] : 0.f;
                const int A = __float_as_int(__fadd_rn(__fmul_rn(v, sc), 12582912.0f)) - 0x4B400000;
                const uint32_t U = (uint32_t)(A + (1 << 23));
                b0 |= (U & 0xffu) << (8 * i);
                b1 |= ((U >> 8) & 0xffu) << (8 * i);
                b2 |= ((U >> 16) & 0xffu) << (8 * i);
            }
            w[0][q] = b0, w[1][q] = b1, w[2][q] = b2;
        }
        uint4 *row = reinterpret_cast<uint4 *>(ws.planes) + (size_t)kc * np;
#pragma unroll
        for (int p = 0; p < 3; p++) row[1 + 3 * m + p] = make_uint4(w[p][0], w[p][1], w[p][2], w[p][3]);
        if (m == 0) {  // the all-ones row and the zero padding rows of this chunk
            row[0] = make_uint4(0x01010101u, 0x01010101u, 0x01010101u, 0x01010101u);
            for (int r = 3 * a.M + 1; r < np; r++) row[r] = make_uint4(0u, 0u, 0u, 0u);
        }
    }
    cl.sync();  // no CTA leaves while another may still read its partials
}

// ---- grouped scales (g = 32 or 64 rows of K per f32 scale and column) -------------
// y[m,n] = 2^-s_m sum_g scale[g,n] sum_{k in g} A[m,k] q[k,n]: each group's
// integer sum needs its own scale, so every group gets its own accumulator.
// CTA (tile, piece) owns a contiguous run of whole groups of one tile.  The
// producer streams stages of up to 16 k-steps of weights with the matching
// plane rows (as in qgm_gemm_kernel); the MMA thread issues a group's g/32
// products (K = 32 each) into one of QGG_NB TMEM buffers and commits it; the
// four drain warps read the group's sums (one column per lane, every plane
// row), release the buffer, and add sum * scale in f64 to per-row registers
// -- groups in ascending order.  The CTA's f64 partials go to
// part[tile][piece][row][128] without atomics; the finish kernel adds the
// pieces of a tile in piece order, so the result does not depend on timing.
constexpr int QGG_MAX_M = 32;  // rows per launch (3 * 32 + 1 = 97 plane rows, 112 TMEM columns)
constexpr int QGG_NB = 4;      // TMEM accumulator buffers of 128 columns
constexpr int QGG_STAGE_KS = 16;
// warps 0-3 and 6-9 drain (two teams of four, each team one column per lane
// and half of the rows), 4 issues the MMAs, 5 produces
constexpr int QGG_THREADS = 320;

__host__ __device__ inline int qgg_slot_bytes(int np) { return QGG_STAGE_KS * (QGM_TN + np) * 16; }

__global__ void __launch_bounds__(QGG_THREADS, 1)
    qgg_gemm_kernel(const QWeightDesc w, const QGemmWs ws, double *part, int M, int np, int nst, int S) {
    extern __shared__ __align__(1024) uint8_t smem[];
    // full[nst], empty[nst], tmem full[NB], tmem empty[NB], mma done
    __shared__ __align__(8) unsigned long long bars[2 * QGM_MAX_NST + 2 * QGG_NB + 1];
    __shared__ uint32_t s_tmem;
    __shared__ int s_abort;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tile = blockIdx.x, piece = blockIdx.y;
    const int R = w.group / 16;                 // k-steps per group
    const int NG = w.KS / R;                    // groups per tile
    const int g0 = (int)((long long)NG * piece / S), g1 = (int)((long long)NG * (piece + 1) / S);
    const int ks0 = g0 * R, ks1 = g1 * R;
    const int slot_bytes = qgg_slot_bytes(np), wslot = QGG_STAGE_KS * QGM_TN * 16;
    const uint32_t b_full = smem_u32(&bars[0]), b_empty = smem_u32(&bars[QGM_MAX_NST]);
    const uint32_t b_tfull = smem_u32(&bars[2 * QGM_MAX_NST]), b_tempty = b_tfull + 8 * QGG_NB;
    const uint32_t b_done = b_tempty + 8 * QGG_NB;
    if (tid == 0) {
        for (int i = 0; i < nst; i++) {
            mbar_init(b_full + 8 * i, 1);
            mbar_init(b_empty + 8 * i, 1);  // arrived by tcgen05.commit
        }
        for (int i = 0; i < QGG_NB; i++) {
            mbar_init(b_tfull + 8 * i, 1);
            mbar_init(b_tempty + 8 * i, 8);  // one arrival per draining warp
        }
        mbar_init(b_done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        s_abort = 0;
    }
    if (warp == 0) tmem_alloc(&s_tmem, 128 * QGG_NB);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    pdl_launch_dependents();
    const uint32_t tmem = s_tmem;
    const uint32_t ring = smem_u32(smem);

    if (warp == 5) {
        if (lane == 0) {  // producer
            uint32_t it = 0, slot = 0, par = 0;
            bool waited = false;
            for (int ks = ks0; ks < ks1; ks += QGG_STAGE_KS) {
                const int nks = min(QGG_STAGE_KS, ks1 - ks);
                if (it >= (uint32_t)nst) {
                    if (!waited) pdl_wait(), waited = true;
                    if (*(volatile int *)&s_abort || !mbar_wait(b_empty + 8 * slot, par ^ 1)) {
                        atomicOr(&qgm_error_flag, 1u);
                        s_abort = 1;
                        break;
                    }
                }
                const uint32_t wbytes = (uint32_t)nks * QGM_TN * 16, pbytes = (uint32_t)nks * np * 16;
                const uint32_t dst = ring + slot * slot_bytes;
                mbar_expect_tx(b_full + 8 * slot, wbytes + pbytes);
                tma_load_1d(dst, reinterpret_cast<const uint8_t *>(w.w) + ((size_t)tile * w.KS + ks) * QGM_TN * 16,
                            wbytes, b_full + 8 * slot);
                if (!waited) pdl_wait(), waited = true;  // the planes come from the previous kernel
                tma_load_1d(dst + wslot, ws.planes + (size_t)ks * np * 16, pbytes, b_full + 8 * slot);
                it++;
                if (++slot == (uint32_t)nst) slot = 0, par ^= 1;
            }
        }
    } else if (warp == 4) {
        if (lane == 0) {  // MMA issuer
            const uint32_t idesc = qgm_idesc(np);
            uint32_t slot = 0, par = 0;
            int gi = 0;
            bool ok = true;
            for (int ks = ks0; ks < ks1 && ok; ks += QGG_STAGE_KS) {
                const int nks = min(QGG_STAGE_KS, ks1 - ks);
                if (!mbar_wait(b_full + 8 * slot, par)) ok = false;
                tc_fence_after();
                const uint32_t a0 = ring + slot * slot_bytes, p0 = a0 + wslot;
                for (int gk = 0; gk < nks && ok; gk += R, gi++) {
                    const uint32_t buf = gi % QGG_NB;
                    if (gi >= QGG_NB && !mbar_wait(b_tempty + 8 * buf, (gi / QGG_NB - 1) & 1)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    for (int kk = 0; kk < R / 2; kk++) {
                        const int k = gk + 2 * kk;
                        const uint64_t da = umma_sdesc(a0 + k * QGM_TN * 16, QGM_TN * 16, 128);
                        const uint64_t db = umma_sdesc(p0 + k * np * 16, np * 16, 128);
                        umma_i8(tmem + buf * 128, da, db, idesc, kk == 0 ? 0u : 1u);
                    }
                    umma_commit(b_tfull + 8 * buf);  // the group's sums are complete
                }
                umma_commit(b_empty + 8 * slot);  // the slot is free once these products are done
                if (++slot == (uint32_t)nst) slot = 0, par ^= 1;
            }
            if (!ok) {
                atomicOr(&qgm_error_flag, 1u);
                s_abort = 1;
            }
            umma_commit(b_done);
            if (!mbar_wait(b_done, 0)) atomicOr(&qgm_error_flag, 1u);
        }
    } else {
        // ---- drain: one column per lane, half of the rows per team, groups in order
        pdl_wait();
        const int q = warp & 3;                   // TMEM lane quarter of this warp
        const int team = warp < 4 ? 0 : 1;  // rows [0, 16) or [16, 32)
        const int col = q * 32 + lane;
        const float *gs = w.gscale + (size_t)tile * NG * QGM_TN + col;
        const int nld = np >> 4;
        constexpr int HALF = QGG_MAX_M / 2;
        double acc[HALF];
#pragma unroll
        for (int m = 0; m < HALF; m++) acc[m] = 0.0;
        float sc_next = g0 < g1 ? __ldg(gs + (size_t)g0 * QGM_TN) : 0.f;
        for (int g = g0, gi = 0; g < g1; g++, gi++) {
            const uint32_t buf = gi % QGG_NB;
            const float sc = sc_next;
            if (g + 1 < g1) sc_next = __ldg(gs + (size_t)(g + 1) * QGM_TN);
            const bool ok = !s_abort && mbar_wait(b_tfull + 8 * buf, (gi / QGG_NB) & 1);
            if (__any_sync(0xffffffffu, !ok)) {
                atomicOr(&qgm_error_flag, 1u);
                s_abort = 1;
                break;
            }
            tc_fence_after();
            uint32_t d[7 * 16];
            const uint32_t lb = tmem + ((uint32_t)(q * 32) << 16) + buf * 128;
#pragma unroll
            for (int j = 0; j < 7; j++)
                if (j < nld) tmem_ld16(lb + 16 * j, d + 16 * j);
            tmem_wait_ld(d);
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(b_tempty + 8 * buf);  // the buffer may take the next group
            const long long ones = (long long)(int)d[0];
            const double scd = (double)sc;
            // static register indices: each team's rows are a compile-time range
            if (team == 0) {
#pragma unroll
                for (int i = 0; i < HALF; i++)
                    if (i < M) {
                        const long long t = (long long)(int)d[1 + 3 * i] + ((long long)(int)d[2 + 3 * i] << 8) +
                                            ((long long)(int)d[3 + 3 * i] << 16) - (ones << 23);
                        // |t| < 2^51: exact to f64 with an integer add and one f64 add
                        acc[i] = fma(i64_to_f64(t), scd, acc[i]);
                    }
            } else {
#pragma unroll
                for (int i = 0; i < HALF; i++)
                    if (HALF + i < M) {
                        const int m = HALF + i;
                        const long long t = (long long)(int)d[1 + 3 * m] + ((long long)(int)d[2 + 3 * m] << 8) +
                                            ((long long)(int)d[3 + 3 * m] << 16) - (ones << 23);
                        acc[i] = fma(i64_to_f64(t), scd, acc[i]);
                    }
            }
        }
        double *out = part + ((size_t)tile * S + piece) * QGG_MAX_M * QGM_TN + col;
#pragma unroll
        for (int i = 0; i < HALF; i++)
            if (team * HALF + i < M) out[(size_t)(team * HALF + i) * QGM_TN] = acc[i];
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, 128 * QGG_NB);
}

// y[m, n] = 2^-s_m * sum over the tile's pieces (in order) of the partials;
// then the STORE or BIAS epilogue.  One thread per (row, column).
template <int EPI>
__global__ void __launch_bounds__(QGM_TN) qgg_finish_kernel(const QGemvArgs a, const QGemmWs ws, const double *part,
                                                            int S) {
    pdl_launch_dependents();
    pdl_wait();
    const int tile = blockIdx.x, m = blockIdx.y, c = threadIdx.x;
    const int n = tile * QGM_TN + c;
    if (n >= a.w.N) return;
    const double *p = part + ((size_t)tile * S * QGG_MAX_M + m) * QGM_TN + c;
    double t = 0.0;
    for (int i = 0; i < S; i++) t += p[(size_t)i * QGG_MAX_M * QGM_TN];
    float y = (float)(t * pow2_neg(ws.shift[m]) * ws.rstd[m]);
    if (EPI == QEPI_BIAS) y = __fadd_rn(y, a.bias[n]);
    a.out[(size_t)m * a.ldo + n] = y;
}

int qgg_nst(int np, int *limit_out) {
    static int lim[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!lim[dev & 63]) SB_TRY(allow_max_dynamic_smem(qgg_gemm_kernel, &lim[dev & 63]));
    *limit_out = lim[dev & 63];
    return std::min(QGM_MAX_NST, lim[dev & 63] / qgg_slot_bytes(np));
}

int qgm_nst(int np, int *limit_out) {
    static int lim[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!lim[dev & 63]) SB_TRY(allow_max_dynamic_smem(qgm_gemm_kernel, &lim[dev & 63]));
    *limit_out = lim[dev & 63];
    return std::min(QGM_MAX_NST, lim[dev & 63] / qgm_slot_bytes(np));
}

template <int EPI>
int finish_launch(const QGemvArgs &a, const QGemmWs &ws, cudaStream_t st, bool pdl) {
    // rows per CTA: the smallest power of two (>= 2) that keeps the grid
    // within two CTAs per SM
    const int cap = 2 * device_props().sm_count;
    int R = 2;
    while (R < 32 && a.w.ntiles * ceil_div(a.M, R) > cap) R *= 2;
    const dim3 grid(a.w.ntiles, ceil_div(a.M, R));
    switch (R) {
    case 2: SB_CUDA_TRY(launch(qgm_finish_kernel<EPI, 1>, grid, dim3(QGM_FIN_THREADS), 0, st, pdl, a, ws)); break;
    case 4: SB_CUDA_TRY(launch(qgm_finish_kernel<EPI, 2>, grid, dim3(QGM_FIN_THREADS), 0, st, pdl, a, ws)); break;
    case 8: SB_CUDA_TRY(launch(qgm_finish_kernel<EPI, 4>, grid, dim3(QGM_FIN_THREADS), 0, st, pdl, a, ws)); break;
    case 16: SB_CUDA_TRY(launch(qgm_finish_kernel<EPI, 8>, grid, dim3(QGM_FIN_THREADS), 0, st, pdl, a, ws)); break;
    default: SB_CUDA_TRY(launch(qgm_finish_kernel<EPI, 16>, grid, dim3(QGM_FIN_THREADS), 0, st, pdl, a, ws)); break;
    }
    return SB_OK;
}

}  // namespace

size_t qgemm_planes_bytes(int K, int M) { return (size_t)ceil_div(K, 16) * qgemm_np(M) * 16; }

bool qgemm_supported(const QWeightDesc &w, int M) {
    return w.TN == QGM_TN && w.group == 0 && (w.KS % 2) == 0 && M > QG_MAX_M && M <= QGM_MAX_M && w.K <= 32768;
}

bool qgemm_grouped_supported(const QWeightDesc &w, int M) {
    return w.TN == QGM_TN && (w.group == 32 || w.group == 64) && w.gscale && w.K % w.group == 0 && M > QG_MAX_M &&
           M <= QGG_MAX_M && w.K <= 32768;
}

int qgemm_grouped_pieces(const QWeightDesc &w) {
    const int NG = w.KS / (w.group / 16);
    return std::max(1, std::min(NG, ceil_div(2 * device_props().sm_count, w.ntiles)));
}

size_t qgemm_grouped_part_doubles(const QWeightDesc &w) {
    return (size_t)w.ntiles * qgemm_grouped_pieces(w) * QGG_MAX_M * QGM_TN;
}

int qgemm_grouped_launch(int epi, const QGemvArgs &a, const QGemmWs &ws, double *part, cudaStream_t st, bool pdl) {
    SB_CHECK(qgemm_grouped_supported(a.w, a.M), SB_ERR_UNSUPPORTED,
             "qgemm (grouped): weight/rows not supported (TN %d, group %d, M %d)", a.w.TN, a.w.group, a.M);
    SB_CHECK(epi == QEPI_STORE || epi == QEPI_BIAS, SB_ERR_UNSUPPORTED, "qgemm (grouped): epilogue %d", epi);
    SB_CHECK(a.norm_w == nullptr, SB_ERR_ARG, "qgemm (grouped): no fused RMSNorm");
    SB_CHECK(ws.planes && ws.shift && ws.rstd && part, SB_ERR_ARG, "qgemm (grouped): missing scratch");
    const int np = qgemm_np(a.M);
    int limit = 0;
    const int nst = qgg_nst(np, &limit);
    SB_CHECK(nst >= 2, SB_ERR_SHAPE, "qgemm (grouped): %d B per stage (limit %d)", qgg_slot_bytes(np), limit);
    SB_CUDA_TRY(launch(qgm_planes_kernel, dim3(a.M + ceil_div(a.w.KS, 16)), dim3(QGM_PL_THREADS), 0, st, pdl, a, ws,
                       np));
    const int S = qgemm_grouped_pieces(a.w);
    SB_CUDA_TRY(launch(qgg_gemm_kernel, dim3(a.w.ntiles, S), dim3(QGG_THREADS), (size_t)nst * qgg_slot_bytes(np), st,
                       pdl, a.w, ws, part, a.M, np, nst, S));
    if (epi == QEPI_BIAS)
        SB_CUDA_TRY(launch(qgg_finish_kernel<QEPI_BIAS>, dim3(a.w.ntiles, a.M), dim3(QGM_TN), 0, st, pdl, a, ws,
                           (const double *)part, S));
    else
        SB_CUDA_TRY(launch(qgg_finish_kernel<QEPI_STORE>, dim3(a.w.ntiles, a.M), dim3(QGM_TN), 0, st, pdl, a, ws,
                           (const double *)part, S));
    return SB_OK;
}

int qgemm_error_peek(unsigned *host, cudaStream_t st) {
    SB_CUDA_TRY(cudaMemcpyFromSymbolAsync(host, qgm_error_flag, sizeof(unsigned), 0, cudaMemcpyDeviceToHost, st));
    return SB_OK;
}

int qgemm_check_error() {
    unsigned f = 0;
    SB_CUDA_TRY(cudaMemcpyFromSymbol(&f, qgm_error_flag, sizeof f));
    if (f) {
        const unsigned zero = 0;
        cudaMemcpyToSymbol(qgm_error_flag, &zero, sizeof zero);
        return set_error(SB_ERR_TIMEOUT, "qgemm: a bounded pipeline wait timed out");
    }
    return SB_OK;
}

int qgemm_launch(int epi, const QGemvArgs &a, const QGemmWs &ws, cudaStream_t st, bool pdl) {
    return qgemm_launch_chained(epi, a, ws, st, pdl, true, nullptr, false);
}

int qgemm_launch_chained(int epi, const QGemvArgs &a, const QGemmWs &ws, cudaStream_t st, bool pdl, bool planes,
                         const QGemmNext *next, bool skip_finish) {
    SB_CHECK(qgemm_supported(a.w, a.M), SB_ERR_UNSUPPORTED, "qgemm: weight/rows not supported (TN %d, group %d, M %d)",
             a.w.TN, a.w.group, a.M);
    SB_CHECK(ws.planes && ws.acc && ws.shift && ws.rstd && ws.ld_acc >= a.w.ntiles * QGM_TN, SB_ERR_ARG,
             "qgemm: missing scratch");
    SB_CHECK(a.norm_w == nullptr || epi == QEPI_QKV || epi == QEPI_SWIGLU || epi == QEPI_LOGITS, SB_ERR_ARG,
             "qgemm: epilogue %d takes no fused RMSNorm", epi);
    const int np = qgemm_np(a.M);
    int limit = 0;
    const int nst = qgm_nst(np, &limit);
    SB_CHECK(nst >= 2, SB_ERR_SHAPE, "qgemm: %d rows need %d B per stage (limit %d)", a.M, qgm_slot_bytes(np), limit);
    if (next) {
        SB_CHECK(epi == QEPI_RESID || epi == QEPI_SWIGLU, SB_ERR_ARG, "qgemm: epilogue %d has no row finish", epi);
        const int K = epi == QEPI_SWIGLU ? a.F : a.w.N;
        SB_CHECK(K <= QGF_MAX_K, SB_ERR_SHAPE, "qgemm: row finish of %d features (max %d)", K, QGF_MAX_K);
        SB_CHECK((size_t)ceil_div(K, 16) * np * 16 <= next->planes_bytes, SB_ERR_SHAPE,
                 "qgemm: planes of %d features x %d rows exceed the scratch", K, a.M);
    }
    if (planes)
        SB_CUDA_TRY(launch(qgm_planes_kernel, dim3(a.M + ceil_div(a.w.KS, 16)), dim3(QGM_PL_THREADS), 0, st, pdl, a,
                           ws, np));
    const int upt = ceil_div(a.w.KS, QGM_UNIT_KS);
    const int G = std::max(1, std::min(device_props().sm_count, a.w.ntiles * upt / 2));
    SB_CUDA_TRY(launch(qgm_gemm_kernel, dim3(G), dim3(QGM_THREADS), (size_t)nst * qgm_slot_bytes(np), st, pdl, a.w, ws,
                       a.M, np, nst));
    if (skip_finish) return SB_OK;  // the consumer of the sums finishes them (and clears them)
    if (next) {
        if (epi == QEPI_RESID)
            SB_CUDA_TRY(launch(qgm_finish_planes_kernel<QEPI_RESID>, dim3(QGF_CLUSTER, a.M), dim3(QGF_THREADS), 0, st,
                               pdl, a, ws, next->norm_w, next->eps, np));
        else
            SB_CUDA_TRY(launch(qgm_finish_planes_kernel<QEPI_SWIGLU>, dim3(QGF_CLUSTER, a.M), dim3(QGF_THREADS), 0, st,
                               pdl, a, ws, next->norm_w, next->eps, np));
        return SB_OK;
    }
    switch (epi) {
    case QEPI_STORE: return finish_launch<QEPI_STORE>(a, ws, st, pdl);
    case QEPI_BIAS: return finish_launch<QEPI_BIAS>(a, ws, st, pdl);
    case QEPI_RESID: return finish_launch<QEPI_RESID>(a, ws, st, pdl);
    case QEPI_SWIGLU: return finish_launch<QEPI_SWIGLU>(a, ws, st, pdl);
    case QEPI_QKV: return finish_launch<QEPI_QKV>(a, ws, st, pdl);
    case QEPI_LOGITS: return finish_launch<QEPI_LOGITS>(a, ws, st, pdl);
    default: return set_error(SB_ERR_ARG, "qgemm: unknown epilogue %d", epi);
    }
}

}  // namespace sb
