// Small kernels around the decode step and the MathBackend op surface.
#pragma once

#include "sb_common.cuh"

namespace sb {

// Per-sequence device state that lets decode steps run without the host.
struct SeqState {
    int *tok = nullptr;         // [B] token fed to the next step
    int *pos = nullptr;         // [B] position of the next step
    const int *prompt = nullptr;     // [B][max_prompt]
    const int *prompt_len = nullptr; // [B]; 0 = always take tok[b]
    int max_prompt = 0;
    int *out = nullptr;         // [B][max_gen] generated tokens
    int *ngen = nullptr;        // [B]
    int max_gen = 0;
    int *last = nullptr;        // [B] argmax of the last step
};

// x[b] = embed[token(b)] with token(b) = prompt[b][pos] while pos < prompt_len,
// else tok[b] (embedding lookup, cpu.rs:485-498).
int embed_launch(const float *embed, int h, int V, SeqState s, int B, float *x, cudaStream_t st, bool pdl);
// Reduce per-tile (value, index) candidates to the argmax of each row (ties ->
// last index, generate.rs:167-173), record it, feed it to the next step and
// advance the position.
// With tp > 1 the candidates of tp ranks are concatenated, rank t's at
// offset t * rank_stride, and rank t's indices are local to its vocabulary
// slice starting at t * idx_stride.
int argmax_step_launch(const float *cand_val, const int *cand_idx, int ntiles, SeqState s, int B,
                       cudaStream_t st, bool pdl, int tp = 1, int rank_stride = 0, int idx_stride = 0);

int rmsnorm_launch(const float *x, const float *w, int rows, int d, float eps, float *out, cudaStream_t st);
int rope_launch(const float *x, int seq, int n_heads, int hd, int start_pos, const float *freqs, float scale,
                float *out, cudaStream_t st);
int swiglu_launch(const float *g, const float *u, size_t n, float *out, cudaStream_t st);
int argmax_rows_launch(const float *x, int rows, int n, int *out, cudaStream_t st);

// quantize_symmetric on device (bit-exact with quantize.rs:16-32).
int quantize_device(const float *w, size_t n, int8_t *q, float *scale_dev, unsigned *amax_scratch,
                    cudaStream_t st);

// Seeded weights of LlamaModel::new generated on the device.
//
// A target [K,N] matrix is made of up to three column segments; element
// (r, c) of segment i is normal sample base_i + r*width_i + (c - c0_i) of the
// fastrand stream (transposed: base_i + c*K + r).  gen_absmax folds |w| into
// *amax (as float bits); gen_quantize writes int8 [K,N] with the scale of
// quantize_symmetric.
struct GenSpec {
    int K = 0, N = 0;
    int nseg = 1;
    int c0[3] = {0, 0, 0};
    int width[3] = {0, 0, 0};
    uint64_t base[3] = {0, 0, 0};
    int transposed = 0;
    const float *src = nullptr;  // when set, values come from this f32 [N,K] (transposed) or [K,N] buffer
};
int gen_absmax(const GenSpec &g, uint64_t seed, unsigned *amax, cudaStream_t st);
int gen_quantize(const GenSpec &g, uint64_t seed, const unsigned *amax, int8_t *q, float *scale_out,
                 cudaStream_t st);
// out[i] = sample(first_sample + i), i < n (f32 embedding table).
int gen_normal_f32(uint64_t seed, uint64_t first_sample, size_t n, float *out, cudaStream_t st);

// A [K, N] matrix read from up to three checkpoint tensors in the HF layout
// [out, in] (row = output column n, the source is transposed), stacked
// along n: column n of segment i (n in [c0[i], c0[i+1])) is source row
// row0[i] + n - c0[i] of p[i], and k is source column k0 + k; ld = elements
// per source row.  dtype: SB_DTYPE_F32, SB_DTYPE_BF16 or SB_DTYPE_F16.  With
// row0 / k0 offsets the same tensors give a tensor-parallel rank's slice.
struct SrcSpec {
    int K = 0, N = 0;
    int nseg = 1;
    int c0[3] = {0, 0, 0};
    const void *p[3] = {nullptr, nullptr, nullptr};
    long long ld[3] = {0, 0, 0};
    long long row0[3] = {0, 0, 0};
    long long k0 = 0;
    int dtype = 0;
};
// absmax of every value of g (the full tensor); then q = quantize_symmetric
// of the values of `part` with the scale of that absmax, written [N, K]
// row-major (the transpose of the reference [K, N] layout), the scale also
// to *scale_out (device).  Bit-exact with the host quantizer.
int src_absmax(const SrcSpec &g, unsigned *amax, cudaStream_t st);
int src_quantize(const SrcSpec &part, const unsigned *amax, int8_t *q, float *scale_out, cudaStream_t st);
// f32 copy of n values of dtype at src (device), e.g. an embedding table.
int src_to_f32(const void *src, int dtype, size_t n, float *out, cudaStream_t st);

}  // namespace sb
