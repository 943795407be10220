// Device sampler: sample_token (generate.rs:92-165) for rows of logits.
#pragma once

#include "misc.cuh"
#include "sb_common.cuh"

namespace sb {

// One token per row of logits [rows][ld] (first n columns): temperature /
// top-k / top-p exactly as the reference orders them, the draw from each
// row's fastrand state rng[row] (advanced by one draw unless the row is
// greedy).  prob: scratch of rows * n doubles.  out: [rows] token ids.
int sample_rows_launch(const float *logits, int rows, int n, int ld, float temperature, int top_k, float top_p,
                       uint64_t *rng, double *prob, int *out, cudaStream_t st);

// Sampling parameters of a device decode loop; max_draws caps the tokens
// drawn per row.
struct SampleCfg {
    float temperature = 1.0f;
    int top_k = 0;
    float top_p = 1.0f;
    int max_draws = 0x7fffffff;
};
// The token step of a sampled decode loop for rows 0..rows-1 of the
// sequence state s: rows inside their prompt draw nothing; from the last
// prompt position on each row samples its next token from its logits row
// (as sample_rows_launch, with its generator rng[row]), records it in s.out
// and feeds it to the next step, until max_draws tokens were drawn.  Every
// row's position advances by one.
int sample_step_launch(const float *logits, int rows, int n, int ld, const SampleCfg &c, uint64_t *rng, double *prob,
                       const SeqState &s, cudaStream_t st);

}  // namespace sb
