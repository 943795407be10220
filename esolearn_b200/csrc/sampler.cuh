// Device sampler: sample_token (generate.rs:92-165) for rows of logits.
#pragma once

#include "sb_common.cuh"

namespace sb {

// One token per row of logits [rows][ld] (first n columns): temperature /
// top-k / top-p exactly as the reference orders them, the draw from each
// row's fastrand state rng[row] (advanced by one draw unless the row is
// greedy).  prob: scratch of rows * n doubles.  out: [rows] token ids.
int sample_rows_launch(const float *logits, int rows, int n, int ld, float temperature, int top_k, float top_p,
                       uint64_t *rng, double *prob, int *out, cudaStream_t st);

}  // namespace sb
