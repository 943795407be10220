/*
 * sb_api.h -- C ABI of libscryb200.so, the B200-native engine for
 * scry-llm's int8 (W8A32) Llama decode path.
 *
 * Plain C types only (pointers, sizes, ints, floats): a Rust FFI crate
 * (`scry-b200-sys`), ctypes or any other FFI binds it directly.  Every entry
 * point returns an sb_status; on failure sb_last_error() gives the message.
 * Each declaration names the reference interface it replaces (paths are
 * inside the reference project, crate scry-llm).
 *
 * Threading: like the reference CUDA backend (backend/cuda.rs:26-79, one
 * thread-local GpuCtx), one host thread drives one device at a time.
 * Streams are passed as `void*` (a cudaStream_t; NULL = legacy default).
 */
#ifndef SB_API_H
#define SB_API_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int sb_status;
enum {
    SB_OK = 0,
    SB_ERR_CUDA = 1,        /* a CUDA runtime call failed */
    SB_ERR_NCCL = 2,        /* a collective failed */
    SB_ERR_TIMEOUT = 3,     /* a bounded device wait gave up */
    SB_ERR_SHAPE = 4,       /* shapes inconsistent or unsupported */
    SB_ERR_OOM = 5,         /* device allocation failed */
    SB_ERR_ARG = 6,         /* bad argument (null pointer, range) */
    SB_ERR_STATE = 7,       /* call out of order (not initialised, no weights) */
    SB_ERR_UNSUPPORTED = 8, /* configuration not built into this library */
};

enum { SB_DTYPE_F32 = 0, SB_DTYPE_BF16 = 1, SB_DTYPE_F16 = 2 };
enum { SB_KV_BF16 = 0, SB_KV_F32 = 1 };

/* Message of the last failure on this thread; returns its status code. */
int sb_last_error(char *buf, size_t len);
/* ABI revision of this header (bumped on any signature change). */
int sb_abi_version(void);

/* ---- device (replaces backend/cuda.rs:39-59 init_gpu / GpuCtx) --------- */
/* Select and initialise `device` for the calling thread. */
sb_status sb_init(int device);
sb_status sb_device_info(int *sm_count, int *cc_major, int *cc_minor, size_t *hbm_bytes);

/* ---- DeviceBackend storage (backend/mod.rs:12-45) ----------------------- */
/* zeros(): zero-filled device buffer. */
sb_status sb_alloc(void **dptr, size_t bytes);
sb_status sb_free(void *dptr);
/* from_vec() / to_vec(): host<->device copies on `stream` (synchronous
 * when stream is NULL). */
sb_status sb_memcpy_h2d(void *dst, const void *src, size_t bytes, void *stream);
sb_status sb_memcpy_d2h(void *dst, const void *src, size_t bytes, void *stream);
sb_status sb_stream_sync(void *stream);

/* ---- quantize.rs ------------------------------------------------------- */
/* quantize_symmetric (quantize.rs:16-32) on the host; bit-exact. */
sb_status sb_quantize_symmetric_host(const float *w, size_t n, int8_t *q, float *scale);
/* Same on device buffers (w, q, scale all device pointers); bit-exact. */
sb_status sb_quantize_symmetric(const float *w, size_t n, int8_t *q, float *scale, void *stream);

/* ---- I8Storage: packed int8 weights (backend/mod.rs:15-21) -------------
 * A [K,N] int8 matrix in the reference layout (linear.rs:17, row-major
 * [in,out]) is re-packed once into column tiles streamed by the GEMV.
 * Re-packing only permutes the int8 values.  group = 0 is the reference's
 * per-tensor scale; group = 32 or 64 keeps f32 scales[ceil(K/g), N]. */
typedef struct sb_qweight sb_qweight;
sb_status sb_qweight_create(int K, int N, int group, sb_qweight **out);
/* Same with an explicit tile width tile_n in {16, 32, 64, 128, 256} (0 =
 * the GEMV's choice).  128-column tiles let 5-64-row products run on the
 * tensor cores (see sb_matmul_i8_f32).  No reference counterpart: the
 * reference keeps [K,N] as is; this only picks the on-device packing. */
sb_status sb_qweight_create_tn(int K, int N, int group, int tile_n, sb_qweight **out);
/* q: host [K,N] int8; scales: host, 1 value (group 0) or [ceil(K/g), N]. */
sb_status sb_qweight_load(sb_qweight *w, const int8_t *q, const float *scales);
sb_status sb_qweight_destroy(sb_qweight *w);

/* matmul_i8_f32 (backend/mod.rs:521-533; CPU cpu.rs:1129-1160):
 * c[M,N] = a[M,K] . dequant(q)[K,N], f32 accumulate.  a, c are device
 * pointers; a_dtype is SB_DTYPE_F32 or SB_DTYPE_BF16.  1-4 rows run the
 * GEMV; 5 or more rows of a per-tensor-scaled weight with 128-column tiles
 * run on the tcgen05 tensor cores, at most 64 rows per launch (same
 * fixed-point arithmetic, same results as row-by-row GEMVs); other shapes
 * run the GEMV 4 rows at a time.  Uses a library-owned workspace on the
 * current device. */
sb_status sb_matmul_i8_f32(const sb_qweight *w, const void *a, int a_dtype, int M, float *c,
                           void *stream);
/* matmul_i8_f32_bias (backend/mod.rs:537-557): c = a . dequant(q) + bias. */
sb_status sb_matmul_i8_f32_bias(const sb_qweight *w, const void *a, int a_dtype, int M,
                                const float *bias, float *c, void *stream);

/* ---- I8Storage exactly as the reference trait hands it over -------------
 * DeviceBackend::i8_from_vec(data: Vec<i8>) -> I8Storage (backend/mod.rs:18)
 * carries no shape, and MathBackend::matmul_i8_f32(a, b_q, scale, m, k, n)
 * (backend/mod.rs:521-533) passes the scale and the [k, n] view with every
 * call.  sb_i8 is that storage: the bytes are copied to the current device
 * as given (row-major [k, n] in the reference layout, linear.rs:17); the
 * first matmul on it with a given (k, n) packs a copy into 128-column tiles
 * (the layout the GEMV and the tensor-core GEMM stream) and later calls with
 * that view reuse it.  A storage may be shared by several owners (the
 * trait's Clone), one call at a time. */
typedef struct sb_i8 sb_i8;
/* i8_from_vec (backend/mod.rs:18): n int8 values from host memory. */
sb_status sb_i8_from_vec(const int8_t *data, size_t n, sb_i8 **out);
/* i8_to_vec (backend/mod.rs:20): the n bytes back to host memory. */
sb_status sb_i8_to_vec(const sb_i8 *b, int8_t *data, size_t n);
sb_status sb_i8_len(const sb_i8 *b, size_t *n);
sb_status sb_i8_destroy(sb_i8 *b);
/* matmul_i8_f32 (backend/mod.rs:521-533; CPU cpu.rs:1129-1160):
 * c[m,n] = a[m,k] . (b_q[k,n] * scale), f32 accumulate.  a, c: device f32
 * (the Storage of the trait).  SB_ERR_SHAPE when k*n exceeds the storage.
 * Same kernels and arithmetic as sb_matmul_i8_f32. */
sb_status sb_i8_matmul_f32(const float *a, sb_i8 *b_q, float scale, int m, int k, int n, float *c,
                           void *stream);
/* matmul_i8_f32_bias (backend/mod.rs:537-557): c = a . dequant(b_q) + bias[n]. */
sb_status sb_i8_matmul_f32_bias(const float *a, sb_i8 *b_q, float scale, const float *bias, int m,
                                int k, int n, float *c, void *stream);

/* ---- Llama ops of MathBackend (device pointers) ------------------------ */
/* rmsnorm (backend/mod.rs rmsnorm; cpu.rs:574-599). */
sb_status sb_rmsnorm(const float *x, const float *w, int rows, int d, float eps, float *out,
                     void *stream);
/* rope_with_freqs_preloaded (cpu.rs:635-664) when scale == 1, and
 * rope_with_freqs_scaled_preloaded (backend/mod.rs:219-230) otherwise. */
sb_status sb_rope_with_freqs(const float *x, int seq, int n_heads, int head_dim, int start_pos,
                             const float *freqs, float scale, float *out, void *stream);
/* swiglu (cpu.rs:666-678). */
sb_status sb_swiglu(const float *gate, const float *up, size_t n, float *out, void *stream);
/* argmax over each row, ties -> last index (generate.rs:167-173). */
sb_status sb_argmax_rows(const float *x, int rows, int n, int32_t *out, void *stream);
/* sample_token (generate.rs:92-165) on the device, one token per row of
 * logits [rows][ld] (the first n columns): temperature < 1e-8 is the argmax
 * (no draw); otherwise f64 temperature scaling, top-k, softmax, top-p and
 * weighted_sample in the reference's order.  rng_state: device [rows]
 * fastrand (wyrand) states, advanced by one draw per sampled row, so the
 * draws equal the reference's Rng::f64 stream.  Ties at the top-p cut are
 * kept lowest index first; sums run in a fixed tree order, so a token can
 * differ from the reference's only when the draw or top_p lies within f64
 * rounding of a running sum.  out: device [rows].  Uses a library-owned
 * workspace of rows * n doubles. */
sb_status sb_sample_rows(const float *logits, int rows, int n, int ld, float temperature, int top_k,
                         float top_p, uint64_t *rng_state, int32_t *out, void *stream);

/* ---- paged GQA decode attention ----------------------------------------
 * Replaces llama.rs:414-456 (gather_reshape_repeat_kv + strided-batched
 * QK^T + softmax + AV).  q: [B, n_heads*hd] f32, already RoPE'd and
 * scaled by 1/sqrt(hd).  K/V caches: [pages][n_kv][page_size][hd] in
 * kv_dtype.  page_table: [B, max_pages] int32.  ctx_len: [B] int32 device.
 * out: [B, n_heads*hd] f32.  Uses a library-owned workspace. */
sb_status sb_attn_decode_paged(const float *q, const void *k_cache, const void *v_cache,
                               int kv_dtype, const int32_t *page_table, int max_pages,
                               const int32_t *ctx_len, int B, int n_heads, int n_kv, int head_dim,
                               int page_size, int max_ctx, float *out, void *stream);

/* Same computation as sb_attn_decode_paged, but it never allocates device
 * memory.  No counterpart in the reference: it exists for callers that
 * cannot let the library cudaMalloc a workspace -- hosts whose device
 * memory is owned by their own pool, and decode loops that cannot take the
 * synchronisation of an allocation mid-step.  Its split scratch is a fixed
 * array inside the library (16 KiB of counters, 1 MiB of partials, held on
 * every GPU that loads the library until exit); shapes needing more
 * (B*n_kv > 4096, or B*n_heads*splits*(head_dim+2)*4 bytes > 1 MiB, with
 * the split count sb_attn_decode_paged would choose) fail with SB_ERR_SHAPE.
 * The first call on a device resolves the array's address (make it before
 * any stream capture).  Calls share the array: calls that overlap on the
 * GPU race and must be ordered by the caller. */
sb_status sb_attn_decode_paged_noalloc(const float *q, const void *k_cache, const void *v_cache,
                                       int kv_dtype, const int32_t *page_table, int max_pages,
                                       const int32_t *ctx_len, int B, int n_heads, int n_kv,
                                       int head_dim, int page_size, int max_ctx, float *out,
                                       void *stream);

/* ---- the quantized Llama engine ----------------------------------------
 * Replaces LlamaModel (llama.rs:583-964) + LlamaKvCache (kv_cache.rs:134-145)
 * behind CausalLM (generate.rs:5-21).  Every projection is an int8 weight
 * with the reference per-tensor scale; embeddings and norm weights stay f32.
 * One decode step of every active sequence is one CUDA-graph replay. */
typedef struct sb_llama_config {
    int32_t vocab_size, hidden_size, intermediate_size, n_layers, n_heads, n_kv_heads;
    int32_t max_seq_len; /* KV capacity per sequence, in positions */
    float rms_norm_eps, rope_theta;
    int32_t tie_word_embeddings;
    int32_t has_rope_scaling;
    double rope_scaling[4]; /* factor, low_freq_factor, high_freq_factor, original_max_pos */
    int32_t max_batch;      /* sequences decoded together (rows of every GEMV) */
    int32_t page_size;      /* KV positions per page */
    int32_t kv_dtype;       /* SB_KV_BF16 or SB_KV_F32 */
} sb_llama_config;

typedef struct sb_llama sb_llama;
enum { SB_W_QKV = 0, SB_W_O = 1, SB_W_GATE = 2, SB_W_UP = 3, SB_W_DOWN = 4, SB_W_LM_HEAD = 5 };
enum { SB_F_EMBED = 0, SB_F_NORM_IN = 1, SB_F_NORM_POST = 2, SB_F_NORM_FINAL = 3 };

/* LlamaModel construction; allocates weights, KV pages and scratch. */
sb_status sb_llama_create(const sb_llama_config *cfg, sb_llama **out);

/* ---- tensor parallelism over the GPUs of one node ----------------------
 * No reference counterpart (the reference decodes on one device).  A model
 * of tp_size ranks, one process (or thread) and one GPU per rank: column
 * slices of q|k|v (by heads), gate and up (by ffn columns) and of the
 * lm_head (by vocabulary rows), row slices of o and down; the KV cache holds
 * the rank's kv heads.  After o and down the partial residual updates are
 * summed over the ranks with an NCCL all-reduce over NVLink (libnccl.so.2,
 * loaded at the first call); the greedy token is the argmax over every
 * rank's vocabulary slice (ties -> last index), identical on all ranks.
 * Every rank makes the same calls in the same order (they are collective),
 * with the same arguments; outputs (tokens, argmax, logits) are the full
 * ones on every rank.  Weights: sb_llama_init_random and
 * sb_llama_load_qweight take the FULL tensors (same seed / same data on every
 * rank) and keep the rank's slice; per-tensor scales are those of the full
 * tensors, so every shard holds the reference's int8 values bit for bit.
 * sb_llama_get_qweight returns the rank's slice. */
#define SB_TP_ID_BYTES 128
/* A fresh communicator id (rank 0 makes it and sends it to the others). */
sb_status sb_tp_unique_id(uint8_t *id);
/* Rank tp_rank of tp_size joins the communicator `id` (waits at most 120 s
 * for the others: SB_ERR_TIMEOUT) and allocates its shard of the model. */
sb_status sb_llama_create_tp(const sb_llama_config *cfg, int tp_rank, int tp_size, const uint8_t *id,
                             sb_llama **out);
/* Diagnostic of the tensor-parallel failure path (no reference counterpart):
 * runs one slice of the peer all-reduce on the current device against a
 * stand-in peer that never writes.  Its bounded wait (about 2 s) must give up
 * and raise the error word -- *timed_out = 1 -- leaving the device usable;
 * *seconds is the wall time of the attempt.  The same bound turns a rank
 * that stops answering mid-step into SB_ERR_TIMEOUT on the others. */
sb_status sb_tp_probe_timeout(int *timed_out, double *seconds);
/* Host-only: rank tp_rank's slice of the full reference tensor of `slot`
 * (SB_W_*; SB_W_LM_HEAD is [V,h]) in the reference layout, and its shape.
 * With full == NULL only rows/cols are returned. */
sb_status sb_tp_shard_qweight(const sb_llama_config *cfg, int slot, int tp_rank, int tp_size, const int8_t *full,
                              int8_t *shard, int *rows, int *cols);
sb_status sb_llama_destroy(sb_llama *m);
/* LlamaModel::new (llama.rs:593-680) generated on the device with the
 * fastrand stream and draw order of the reference, then quantized per
 * tensor (quantize.rs:16-32) and packed.  No host copy of the weights. */
sb_status sb_llama_init_random(sb_llama *m, uint64_t seed);
/* Load one quantized projection, reference layout [K,N] (layer -1 = lm_head,
 * given as [V,h] like llama.rs:943-948). */
sb_status sb_llama_load_qweight(sb_llama *m, int layer, int slot, const int8_t *q, float scale);
/* Read back one quantized projection in the reference layout (inverse of
 * sb_llama_load_qweight; the lm_head comes back as [V,h]).  q: host buffer
 * of K*N bytes; scale: host float. */
sb_status sb_llama_get_qweight(sb_llama *m, int layer, int slot, int8_t *q, float *scale);
/* LlamaModel::from_safetensors for one projection (llama.rs:768-958), with
 * the checkpoint's own bytes: every part is a host tensor in the HF layout
 * [out, in] (row-major) and dtype SB_DTYPE_F32, SB_DTYPE_BF16 or SB_DTYPE_F16.
 * On the device: the exact conversion to f32 (llama.rs:795-808), the
 * transpose to [in, out] (llama.rs:815-825), for slot SB_W_QKV the q|k|v
 * column concatenation of parts q [n_heads*hd, h], k and v [n_kv*hd, h]
 * (llama.rs:1009-1029), quantize_symmetric of the whole tensor (quantize.rs
 * :16-32, bit-exact with sb_quantize_symmetric_host) and the packing.
 * layer -1 is the lm_head [V, h] (llama.rs:943-948); other slots take one
 * part: o [h, q], gate and up [ffn, h] (gate before up), down [h, ffn].
 * Under tensor parallelism the parts are the FULL tensors and the rank keeps
 * its slice, the scale being the full tensor's.  The raw bytes pass through
 * a staging buffer the model keeps (grown to the largest tensor) until
 * sb_llama_destroy. */
sb_status sb_llama_load_hf(sb_llama *m, int layer, int slot, int dtype, int n_parts,
                           const void *const *parts, const int64_t *part_rows, int64_t cols);
/* The f32 tensors from checkpoint bytes (converted on the device): which =
 * SB_F_EMBED ([V,h], n = V*h), SB_F_NORM_IN / SB_F_NORM_POST of `layer` or
 * SB_F_NORM_FINAL (n = h). */
sb_status sb_llama_load_hf_f32(sb_llama *m, int which, int layer, int dtype, const void *data, int64_t n);
/* Load an f32 tensor: embed [V,h] or a norm weight [h]. */
sb_status sb_llama_load_f32(sb_llama *m, int which, int layer, const float *data);
/* Forget all cached positions (LlamaKvCache::new). */
sb_status sb_llama_reset(sb_llama *m);
/* forward_with_llama_cache (llama.rs:744-763) for `batch` sequences:
 * token[b] at position pos[b] of sequence b.  Optional outputs (host):
 * logits [batch, V] f32, argmax [batch] (ties -> last). */
sb_status sb_llama_forward(sb_llama *m, int batch, const int32_t *tokens, const int32_t *pos,
                           float *logits, int32_t *argmax);
/* CausalLM::forward (generate.rs:9; LlamaModel::forward, llama.rs:683-700):
 * logits [n, V] (host) of every position of the token sequence, run from
 * position 0 as batched prefill chunks of max_batch positions (every
 * projection of a chunk one tensor-core GEMM when max_batch >= 5).  Uses
 * sequence slot 0's KV pages as its scratch: slot 0's cached positions are
 * overwritten (other slots are untouched).  n <= max_seq_len. */
sb_status sb_llama_forward_seq(sb_llama *m, const int32_t *tokens, int n, float *logits);
/* sample_token (generate.rs:92-165) for each of the `batch` rows of logits
 * the last sb_llama_forward left on the device (see sb_sample_rows): only
 * the tokens come back to the host, not [batch, V] logits.  rng_state: host
 * [batch] fastrand states, advanced in place.  Single-GPU models only
 * (SB_ERR_UNSUPPORTED under tensor parallelism). */
sb_status sb_llama_sample(sb_llama *m, int batch, float temperature, int top_k, float top_p,
                          uint64_t *rng_state, int32_t *tokens);
/* Sampled generation as a device loop (generate.rs:68-86 with
 * temperature > 0): from this call on, every decode step that sb_llama_step
 * queues ends in sample_token on the device for rows 0..batch-1 instead of
 * the argmax, and feeds the sampled token to the next step with no host
 * round trip.  A row draws nothing while it is inside its prompt; from its
 * last prompt position on it draws one token per step from its own fastrand
 * state, until max_draws tokens were drawn (later steps draw nothing).
 * sb_llama_prefill also samples the first generated token.  rng_state: host
 * [batch] states, copied to the device; sb_llama_get_rng reads the advanced
 * states back, sb_llama_tokens the tokens.  sb_llama_forward and
 * sb_llama_forward_batch keep returning argmax tokens.  Single-GPU models
 * only (SB_ERR_UNSUPPORTED under tensor parallelism).  Replaces the host
 * loop around sb_llama_sample. */
sb_status sb_llama_set_sampling(sb_llama *m, int batch, float temperature, int top_k, float top_p,
                                int max_draws, const uint64_t *rng_state);
/* Back to greedy (argmax) steps. */
sb_status sb_llama_clear_sampling(sb_llama *m);
/* The device generators of rows 0..batch-1 (host out [batch]). */
sb_status sb_llama_get_rng(sb_llama *m, int batch, uint64_t *rng_state);
/* generate (generate.rs:51-89) with temperature 0, for `batch` prompts of
 * equal length: prompts [batch, n_prompt], out [batch, max_tokens]. */
sb_status sb_llama_generate_greedy(sb_llama *m, int batch, const int32_t *prompts, int n_prompt,
                                   int max_tokens, int32_t *out);
/* Residual stream after every layer of the last sb_llama_forward call,
 * [n_layers, batch, h] (host), when tracing was enabled at that call. */
sb_status sb_llama_set_trace(sb_llama *m, int enabled);
sb_status sb_llama_get_trace(sb_llama *m, float *out);

/* Benchmark helpers: queue n decode steps of the current batch on the
 * engine stream (device-driven tokens and positions; no host sync). */
sb_status sb_llama_begin(sb_llama *m, int batch, const int32_t *prompts, int n_prompt);
/* Batched prefill, the decode-step counterpart of LlamaModel::forward over a
 * prompt (llama.rs:683-700): each sequence's prompt runs in chunks of up to
 * max_batch positions, every position one row of a batched step (all rows
 * on that sequence's KV pages), so each chunk's projections are one
 * tensor-core GEMM.  Leaves `batch` sequences as sb_llama_begin +
 * sb_llama_step(n_prompt) would: the prompt cached, the argmax after the last
 * prompt token recorded as generated token 0 and fed to the next step. */
sb_status sb_llama_prefill(sb_llama *m, int batch, const int32_t *prompts, int n_prompt);
sb_status sb_llama_step(sb_llama *m, int n_steps);
sb_status sb_llama_tokens(sb_llama *m, int32_t *out, int max_tokens, int *n_out);
void *sb_llama_stream(sb_llama *m);
/* One eager (non-graph) decode step of the current batch with a CUDA event
 * pair around every kernel on the engine stream: per-class device time in
 * ms (GEMV = all int8 projections, attention, other = embed + argmax) and
 * the int8 weight bytes those GEMVs read.  Advances the sequences like
 * sb_llama_step(m, 1). */
sb_status sb_llama_profile_step(sb_llama *m, float *gemv_ms, float *attn_ms, float *other_ms,
                                int *launches);
/* Bytes the engine streams per decode step at the current context (int8
 * weights + scales + KV read), for roofline accounting. */
sb_status sb_llama_step_bytes(sb_llama *m, double *weight_bytes, double *kv_bytes_per_pos);
/* Kernel launches one decode step of `batch` sequences makes: 1 when the
 * step runs as the persistent single-kernel step (batch 1 on supported
 * shapes), else the per-operation kernel count.  No reference counterpart
 * (the reference runs on the CPU); it documents which device path runs. */
sb_status sb_llama_step_launches(sb_llama *m, int batch, int *launches);
/* How the attention of one decode step of `batch` sequences divides its
 * work (no reference counterpart; it documents which device path runs and
 * lets tests assert that a multi-split path was exercised).  Persistent
 * batch-1 step: *splits = 0, *tensor_map = 0, *chunk = KV positions per ring
 * stage (the (kv head, chunk) units are spread over all SMs).  Batched step:
 * *splits = context splits per (sequence, kv head), *tensor_map = 1 when the
 * tensor-map kernel runs (then *chunk = 64, its tile), else 0. */
sb_status sb_llama_attn_plan(sb_llama *m, int batch, int *splits, int *tensor_map, int *chunk);
/* Timeline of the persistent batch-1 step (a profiling aid; no reference
 * counterpart).  When enabled, every later step records, per phase p (6 per
 * layer: qkv, attention, o, gate/up, SwiGLU, down; then lm_head and the
 * argmax) and per CTA c, five %globaltimer readings in ns: the phase's start
 * after its grid barrier, the end of its input stage, the moments its first
 * and its last weight stage were ready (GEMV phases; 0 otherwise), and its
 * end before the arrival: out[(p * ctas + c) * 5 + i].  SB_ERR_UNSUPPORTED when the model
 * does not run the persistent step.  get: *phases and *ctas always; out
 * (cap slots) when non-NULL, for the last step.  The timeline is compiled
 * into the step kernel only in a profiling build (SB_STEP_TIMELINE=1 in the
 * environment of `python -m esolearn_b200.build`); otherwise enabling it
 * returns SB_ERR_UNSUPPORTED. */
sb_status sb_llama_set_timeline(sb_llama *m, int enabled);
sb_status sb_llama_get_timeline(sb_llama *m, uint64_t *out, size_t cap, int *phases, int *ctas);

#ifdef __cplusplus
}
#endif
#endif /* SB_API_H */
