// Paged, GQA-aware decode attention over a bf16 (or f32) KV cache.
#pragma once

#include <cuda.h>  // CUtensorMap (types only; the encoder is resolved at run time)

#include "sb_common.cuh"

namespace sb {

struct AttnArgs {
    const float *q = nullptr;  // [B, n_heads*hd], RoPE'd and scaled by 1/sqrt(hd)
    const void *kc = nullptr;  // [pages][n_kv][page_size][hd]
    const void *vc = nullptr;
    int kv_f32 = 0;
    const int *page_table = nullptr;  // [B, max_pages]
    int max_pages = 0;
    const int *len = nullptr;  // [B] device: context length, or position when len_is_pos
    int len_is_pos = 0;        // context = len[b] + 1 (the position just written)
    int B = 1, n_heads = 0, n_kv = 0, hd = 0, page_size = 0;
    int n_splits = 1;   // context splits per (sequence, kv head)
    float *out = nullptr;           // [B, n_heads*hd]
    float *part = nullptr;          // scratch [B][n_heads][n_splits][hd+2]
    unsigned *counters = nullptr;   // scratch [B][n_kv], zero between launches
    // Tensor-map path (bf16 cache, 2-8 query heads per kv head, pages of a
    // multiple of 64 positions): K and V of every layer as [rows][hd] 2-D
    // tensors; this layer's (page, head, slot) row is tm_row0 + (page*n_kv +
    // head)*page_size + slot.
    int tma = 0;
    long long tm_row0 = 0;
    CUtensorMap tmk, tmv;
    // Tensor-map path with one split: the q|k|v projection's epilogue done
    // here instead of in its own kernel.  q, k and v of row b come from the
    // GEMM's exact int64 column sums qkv_sums[b * ld_sums + n] (cleared after
    // use), y = sum * 2^-shift[b] * qkv_scale * rstd[b]; RoPE from the
    // rope_cos / rope_sin rows of the position, q scaled by q_scale; the new
    // K/V row is written to the cache at position len[b] (when 0 <= it <
    // max_pos) before the tile holding it is loaded.
    const long long *qkv_sums = nullptr;
    int ld_sums = 0;
    const int *shift = nullptr;
    const double *rstd = nullptr;
    float qkv_scale = 0.f, q_scale = 1.f;
    const float *rope_cos = nullptr, *rope_sin = nullptr;
    int max_pos = 0;
};

// Causal attention of a prefill chunk (attention_prefill.cu): rows 0..M-1
// are positions pos[r] of one sequence whose pages are page_table[0 ..
// max_pages); row r attends to positions 0..pos[r].  q: [M, n_heads*hd]
// (RoPE'd, scaled by 1/sqrt(hd)); out: [M, n_heads*hd].  bf16 cache, head_dim
// 64 or 128.  Each K/V tile is read once per 16 rows and q head.
struct PrefillAttnArgs {
    const float *q = nullptr;
    const void *kc = nullptr, *vc = nullptr;  // this layer's [pages][n_kv][page_size][hd]
    int kv_f32 = 0;
    const int *page_table = nullptr;  // the sequence's pages
    int max_pages = 0;
    const int *pos = nullptr;  // [M] device
    int M = 0, n_heads = 0, n_kv = 0, hd = 0, page_size = 0;
    float *out = nullptr;
};
bool attn_prefill_supported(int hd, int kv_f32);
int attn_prefill_launch(const PrefillAttnArgs &a, cudaStream_t st, bool pdl);

// Queues a copy of the tensor-map kernel's error word into *host (pinned) on st.
int attn_tc_error_peek(unsigned *host, cudaStream_t st);
// Reports (and clears) a timed-out wait of the tensor-map kernel.
int attn_tc_check_error();
// Encode a [rows][hd] bf16 tensor map over a KV cache for the tensor-map path.
int attn_make_tensor_map(CUtensorMap *map, const void *base, long long rows, int hd);

// Splits per (sequence, kv head) for a given max context on this device:
// enough CTAs for two waves, and at most about 256 positions per split.
int attn_pick_splits(int B, int n_kv, int max_ctx);
size_t attn_scratch_floats(int B, int n_heads, int n_splits, int hd);
// Runs the tensor-core kernel (attention_tc.cu) for bf16 caches with 2, 4 or
// 8 query heads per kv head, the SIMT kernel (attention.cu) otherwise.
int attn_launch(const AttnArgs &a, cudaStream_t st, bool pdl);
bool attn_tc_supported(const AttnArgs &a);
int attn_tc_launch(const AttnArgs &a, cudaStream_t st, bool pdl);

}  // namespace sb
