// Batched int8 linear on the 5th-generation tensor cores (tcgen05 + TMEM),
// for 5 to 64 activation rows (batched decode, the quantized-linear sweep).
#pragma once

#include "qgemv.cuh"

namespace sb {

constexpr int QGM_MAX_M = 64;

// Plane rows of the MMA's B operand for M activation rows: three byte planes
// per row plus one all-ones row, padded to a multiple of 16.
inline int qgemm_np(int M) { return (3 * M + 1 + 15) / 16 * 16; }

// Scratch of one batched linear (device memory, owned by the caller).
struct QGemmWs {
    uint8_t *planes = nullptr;  // [KS][np][16] fixed-point planes of the M input rows
    long long *acc = nullptr;   // [M][ld_acc] exact column sums (all zero between calls)
    int *shift = nullptr;       // [M] per-row exponent
    double *rstd = nullptr;     // [M] per-row RMSNorm factor (1 without norm)
    int ld_acc = 0;             // >= ntiles * 128
};
size_t qgemm_planes_bytes(int K, int M);

// Whether the tensor-core path takes this weight and row count: 128-column
// tiles, per-tensor scale, K a multiple of 32 up to 32768, 5 <= M <= 64.
bool qgemm_supported(const QWeightDesc &w, int M);

// y = epilogue(x W) for M rows, as qgemv_launch (same QGemvArgs and epilogues)
// in three launches: quantize the rows into planes, stream the weights
// through the tensor cores into exact int64 column sums, finish (scale +
// epilogue; clears the sums).  pdl enables programmatic dependent launch.
int qgemm_launch(int epi, const QGemvArgs &a, const QGemmWs &ws, cudaStream_t st, bool pdl);
// The next linear of a chain, when this linear's output row is its input:
// its fused RMSNorm weight (nullptr: none) and eps, and the size of the
// planes scratch.
struct QGemmNext {
    const float *norm_w = nullptr;
    float eps = 1e-5f;
    size_t planes_bytes = 0;
};
// qgemm_launch as one link of a chain.  planes = false skips the planes
// kernel (the previous link already wrote this input's planes, shift and
// rstd into ws).  With next, the finish is one launch of clusters (one row
// each; epilogues RESID and SWIGLU, at most 32768 output features) that
// also writes the next linear's planes, shift and rstd into ws, so the next
// link runs with planes = false.
// skip_finish: only the planes (if asked) and the GEMM; the caller's next
// kernel consumes and clears the int64 sums (the attention's fused q|k|v
// epilogue).
int qgemm_launch_chained(int epi, const QGemvArgs &a, const QGemmWs &ws, cudaStream_t st, bool pdl, bool planes,
                         const QGemmNext *next, bool skip_finish = false);
// Group-scaled weights (g = 32 or 64) on the tensor cores, 5 to 32 rows per
// launch: one TMEM accumulator per group, the group scales applied in f64 as
// the groups are drained; per-(tile, piece) f64 partials in `part`
// (qgemm_grouped_part_doubles of them) are summed in piece order by the finish
// kernel.  Epilogues STORE and BIAS.
bool qgemm_grouped_supported(const QWeightDesc &w, int M);
size_t qgemm_grouped_part_doubles(const QWeightDesc &w);
int qgemm_grouped_launch(int epi, const QGemvArgs &a, const QGemmWs &ws, double *part, cudaStream_t st, bool pdl);
// Queues a copy of the GEMM kernels' error word into *host (pinned) on st.
int qgemm_error_peek(unsigned *host, cudaStream_t st);
// Reports (and clears) a timed-out pipeline wait of the GEMM kernel.
int qgemm_check_error();

}  // namespace sb
