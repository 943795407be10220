/*
 * scry_oracle.h -- CPU restatement of scry-llm's int8 Llama decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the
 * B200 engine (libscryb200.so).  Only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline / --impl reference leg may load it.  The product
 * never links or calls it.
 *
 * Every function restates one item of the reference (Rust, crate scry-llm);
 * citations are path:line inside the reference project.  The reference cannot
 * be built here (no cargo/rustc), so the restatement follows the source
 * operation by operation, in the same floating-point order, compiled with
 * -ffp-contract=off so no FMA contraction happens (Rust never contracts).
 *
 * Parity pins: the quantizer and the unit-level ops are checked against the
 * reference's own unit tests (quantize.rs:46-83, backend/cpu.rs:1500-1756,
 * tests/llama_smoke.rs invariants) in tests/test_oracle.py.  The seeded
 * weight generator restates fastrand 2.3.0 (Cargo.lock:903-904, not vendored
 * in the reference): its bit-equality with a Rust build is UNPINNED, so
 * model-level parity is pinned at the weight file -- the engine consumes the
 * int8 tensors this oracle produces.
 */
#ifndef SCRY_ORACLE_H
#define SCRY_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- fastrand 2.3.0 (wyrand) ------------------------------------------ */
/* Rng::with_seed / gen_u64 / f64, as used by nn/init.rs:2-14. */
uint64_t orc_rng_u64(uint64_t *state);
double orc_rng_f64(uint64_t *state);
/* Rng::usize(0..n) (Lemire multiply-shift with rejection). */
uint64_t orc_rng_below(uint64_t *state, uint64_t n);
/* init::normal_sample (nn/init.rs:2-9): Box-Muller from two f64 draws. */
float orc_normal_sample(uint64_t *state, float mean, float std);
/* init::normal_vec (nn/init.rs:12-14), sequential. */
void orc_normal_vec(uint64_t *state, size_t n, float mean, float std, float *out);
/* Same stream as orc_normal_vec, computed in parallel: sample i of the
 * stream starting at draw index `first_draw` (draws are counter based:
 * state_n = seed + n*C0). Bit-identical to the sequential version. */
void orc_normal_vec_at(uint64_t seed, uint64_t first_draw, size_t n, float mean, float std,
                       float *out);

/* ---- quantize.rs ----------------------------------------------------- */
/* quantize_symmetric (quantize.rs:16-32). Returns the scale. */
float orc_quantize_symmetric(const float *w, size_t n, int8_t *q);
/* dequantize (quantize.rs:35-40). */
void orc_dequantize(const int8_t *q, size_t n, float scale, float *out);
/* Per-group variant (derived, no reference counterpart): groups of `group`
 * consecutive rows k of a [K,N] matrix share scale[k/group, n] = absmax/127. */
void orc_quantize_grouped(const float *w, int k, int n, int group, int8_t *q, float *scales);

/* ---- backend/cpu.rs ops ---------------------------------------------- */
/* matmul_i8_f32_tiled (cpu.rs:1129-1160): C[m,n] = sum_p A[m,p]*(q[p,n]*scale). */
void orc_matmul_i8_f32(const float *a, const int8_t *q, float scale, int m, int k, int n,
                       float *c);
/* Same arithmetic with B given transposed (q_t[n,k]); bit-identical to
 * orc_matmul_i8_f32 on the transposed int8 matrix.  Used for lm_head
 * (llama.rs:759-762 is a trans_b matmul). */
void orc_matmul_i8_f32_tb(const float *a, const int8_t *q_t, float scale, int m, int k, int n,
                          float *c);
/* Per-group variant of cpu.rs:1129-1160 (derived): term = a*(q*scale[p/g,n]). */
void orc_matmul_i8_f32_grouped(const float *a, const int8_t *q, const float *scales, int group,
                               int m, int k, int n, float *c);
/* rmsnorm (cpu.rs:574-599). */
void orc_rmsnorm(const float *x, const float *w, int rows, int d, float eps, float *out);
/* rope_with_freqs_preloaded (cpu.rs:635-664). */
void orc_rope(const float *x, int seq, int n_heads, int hd, int start_pos, const float *freqs,
              float *out);
/* scale (cpu.rs:509-511). */
void orc_scale(const float *x, size_t n, float s, float *out);
/* swiglu (cpu.rs:666-678) with silu_scalar (cpu.rs:1119-1122). */
void orc_swiglu(const float *g, const float *u, size_t n, float *out);
/* softmax (cpu.rs:336-366). */
void orc_softmax(const float *x, int rows, int cols, float *out);
/* gemv_trans_b_into (cpu.rs:825-842) and gemv_into (cpu.rs:846-871). */
void orc_gemv_trans_b(const float *v, const float *mat_t, int k, int n, float *out);
void orc_gemv(const float *v, const float *mat, int k, int n, float *out);
/* gather_reshape_repeat_kv (cpu.rs:707-730). */
void orc_gather_reshape_repeat_kv(const float *cache, int cached_len, int n_kv, int n_q, int hd,
                                  float *out);
/* compute_rope_freqs (llama.rs:1035-1067); scaling may be NULL, else
 * {factor, low_freq_factor, high_freq_factor, original_max_position_embeddings}. */
void orc_compute_rope_freqs(int hd, float theta, const double *scaling, double *out);
/* generate.rs:167-173 argmax (ties resolve to the LAST maximal index). */
int64_t orc_argmax(const float *x, size_t n);

/* ---- model (llama.rs) ------------------------------------------------- */
typedef struct {
    int vocab_size, hidden_size, intermediate_size, n_layers, n_heads, n_kv_heads, max_seq_len;
    float rms_norm_eps, rope_theta;
    int tie_word_embeddings;
    int has_rope_scaling;
    double rope_scaling[4]; /* factor, low, high, original_max_position_embeddings */
} orc_config;

typedef struct orc_llama orc_llama;
typedef struct orc_cache orc_cache;

/* Weight slots of one decoder layer. */
enum { ORC_QKV = 0, ORC_O = 1, ORC_GATE = 2, ORC_UP = 3, ORC_DOWN = 4 };

/* LlamaModel::new (llama.rs:593-680) with every projection quantized by
 * quantize_symmetric -- the fused qkv_proj as one tensor, o/gate/up/down and
 * the lm_head ([V,h], per-tensor scale) each as one tensor. */
orc_llama *orc_llama_new_random(const orc_config *cfg, uint64_t seed);
/* A model of the given shape with seeded uniform int8 weights, for timing
 * the CPU path only (no parity meaning). */
orc_llama *orc_llama_new_uniform(const orc_config *cfg, uint64_t seed);
/* Quantize an f32 model given tensor by tensor (same layout as llama.rs). */
orc_llama *orc_llama_new_empty(const orc_config *cfg);
void orc_llama_free(orc_llama *m);
/* Raw access for exporting weights to the engine. */
int8_t *orc_llama_weight(orc_llama *m, int layer, int slot, float *scale_out, int *k, int *n);
int8_t *orc_llama_lm_head(orc_llama *m, float *scale_out); /* [V,h] row-major */
float *orc_llama_embed(orc_llama *m);                        /* [V,h] f32 */
float *orc_llama_norm(orc_llama *m, int layer, int which);  /* which: 0 input, 1 post; layer -1 final */
void orc_llama_set_scale(orc_llama *m, int layer, int slot, float scale); /* layer -1: lm_head */

/* LlamaKvCache::new (kv_cache.rs:134-145). kv_bf16 != 0 rounds every K/V
 * element to bf16 (RNE) on append: a derived variant that mirrors the
 * engine's bf16 cache; 0 is the reference's f32 cache. */
orc_cache *orc_cache_new(const orc_llama *m, int max_seq, int kv_bf16);
void orc_cache_free(orc_cache *c);
/* forward_with_llama_cache (llama.rs:744-763) -> logits [V]. If `trace` is
 * non-NULL it receives the residual stream after every layer [n_layers, h]. */
void orc_forward_with_cache(const orc_llama *m, orc_cache *c, int token, int pos, float *logits,
                            float *trace);
/* n consecutive forward_with_cache calls (tokens[i] at position pos0 + i)
 * evaluated layer by layer for all n tokens; bit-identical logits and cache.
 * logits_all [n, V] and logits_last [V] are optional. */
void orc_forward_tokens(const orc_llama *m, orc_cache *c, const int *tokens, int n, int pos0,
                        float *logits_all, float *logits_last);
/* Deep copy of a cache; truncation to len cached positions; its length. */
orc_cache *orc_cache_clone(const orc_cache *src);
void orc_cache_truncate(orc_cache *c, int len);
int orc_cache_len(const orc_cache *c);
/* Fill rows 0..len-1 with seeded values and set the length (timing only). */
void orc_cache_fill(orc_cache *c, int len, uint64_t seed);
/* generate (generate.rs:51-89) with temperature 0 (greedy). */
void orc_generate_greedy(const orc_llama *m, const int *prompt, int n_prompt, int max_tokens,
                         int kv_bf16, int *out_tokens);
/* sample_token (generate.rs:92-165) on host logits. */
int64_t orc_sample_token(const float *logits, size_t n, float temperature, size_t top_k,
                         float top_p, uint64_t *rng_state);

void orc_set_threads(int n);
int orc_get_threads(void);

#ifdef __cplusplus
}
#endif
#endif
