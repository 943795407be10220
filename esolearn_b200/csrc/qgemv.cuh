// Dequant-fused int8 GEMV / skinny GEMM for decode (M <= 4 rows).
#pragma once

#include "sb_common.cuh"

namespace sb {

// Epilogue applied to y[m,n] = scale * rstd[m] * sum_k a[m,k] q[k,n].
enum QEpi {
    QEPI_STORE = 0,   // out[m,n] = y
    QEPI_RESID = 1,   // out[m,n] = out[m,n] + y          (llama.rs:564,568)
    QEPI_SWIGLU = 2,  // out[m,j] = silu(gate_j) * up_j   (llama.rs:490-500)
    QEPI_QKV = 3,     // RoPE q/k, scale q, write q and the paged K/V cache (llama.rs:386-408)
    QEPI_LOGITS = 4,  // out[m,n] = y and a per-tile argmax candidate (llama.rs:762)
    QEPI_BIAS = 5,    // out[m,n] = y + bias[n]           (backend/mod.rs:537-557)
};

// Packed int8 weight resident on the device.
//
// Layout: column tiles of TN columns; inside a tile, k-steps of 16 rows;
// inside a k-step, TN columns x 16 consecutive k bytes.  Byte (k, n) sits
// at ((tile*KS + k/16)*TN + n%TN)*16 + k%16 with tile = n/TN.  Every
// k-step of a tile is one contiguous TN*16-byte run, so a warp's 16-byte
// loads are fully coalesced.  Padding rows/columns hold zeros.
struct QWeightDesc {
    const uint4 *w = nullptr;
    const float *gscale = nullptr;  // grouped scales [ntiles][NG][TN] (group > 0)
    float scale = 0.0f;             // per-tensor scale (group == 0)
    float scale_up = 0.0f;          // SwiGLU-paired weights: scale of the up columns
    int K = 0, N = 0;               // logical shape (N counts packed columns)
    int KS = 0;                     // padded K / 16
    int TN = 0, ntiles = 0;
    int group = 0;
};

struct QGemvArgs {
    QWeightDesc w;
    int M = 1;
    const void *x = nullptr;  // activations [M, ldx]
    int ldx = 0;
    int x_bf16 = 0;
    const float *norm_w = nullptr;  // fused RMSNorm weight [K] (nullptr: no norm)
    float eps = 1e-5f;
    // STORE / RESID / SWIGLU / LOGITS / BIAS output
    float *out = nullptr;
    int ldo = 0;
    const float *bias = nullptr;
    int F = 0;  // SWIGLU: number of output features
    // QKV
    float *q_out = nullptr;
    int q_dim = 0, kv_dim = 0, hd = 0, n_kv = 0;
    void *kcache = nullptr, *vcache = nullptr;
    int kv_f32 = 0, page_size = 0, max_pages = 0;
    const int *page_table = nullptr;
    const int *pos = nullptr;
    int max_pos = 0;  // positions outside [0, max_pos) are not written
    const float *rope_cos = nullptr, *rope_sin = nullptr;
    float q_scale = 1.0f;
    // LOGITS
    float *cand_val = nullptr;
    int *cand_idx = nullptr;
};

constexpr int QG_THREADS = 288;  // 8 consumer warps + 1 TMA producer warp
constexpr int QG_MAX_M = 4;

// Tile width for an N-column weight read by M-row GEMVs on this device.
int qgemv_pick_tn(int N, int K, int min_tn);
size_t qweight_bytes(int K, int N, int TN);
size_t qweight_scale_count(int K, int N, int TN, int group);
size_t qgemv_smem_bytes(int M, int KS, int TN, bool norm);

// Launch one GEMV.  pdl enables programmatic dependent launch.
// qgemv_check_error() reports (and clears) a timed-out pipeline wait.
int qgemv_check_error();
// Queues a copy of the GEMV's error word into *host (pinned) on st.
int qgemv_error_peek(unsigned *host, cudaStream_t st);
int qgemv_launch(int epi, const QGemvArgs &a, cudaStream_t st, bool pdl);
// Split-K GEMV (qgemv_sk.cu) for 1-4 rows of a per-tensor weight with
// 128-column tiles and fewer tiles than SMs (STORE / BIAS epilogues): CTA
// (tile, k range), exact int64 sums in a workspace of qgemv_splitk_ws_bytes
// (zero before the first call; every call leaves it zero), the last split of
// a tile applies the epilogue.  Bit-identical to qgemv_launch.
bool qgemv_splitk_wanted(const QWeightDesc &w, int M);
size_t qgemv_splitk_ws_bytes(const QWeightDesc &w, int M);
int qgemv_splitk_launch(int epi, const QGemvArgs &a, void *ws, cudaStream_t st);

// Permute a device [K,N] int8 matrix into the packed layout.  With
// pair_F > 0 the source is two [K,F] matrices (gate then up, concatenated
// along N) interleaved in blocks of 16 columns: [g0..g15, u0..u15, g16..].
// With src_tr the source is stored transposed, [N,K] (the lm_head's [V,h]).
int qweight_pack(const int8_t *src, int K, int N, int TN, int pair_F, int src_tr, uint4 *dst, cudaStream_t st);
// Inverse of qweight_pack (src_tr = 0): packed -> [K,N] (or gate, up [K,F] each).
int qweight_unpack(const uint4 *src, int K, int N, int TN, int pair_F, int8_t *dst, cudaStream_t st);
// Grouped scales [NG, N] (device) into [ntiles][NG][TN].
int qscale_pack(const float *src, int K, int N, int TN, int group, float *dst, cudaStream_t st);

}  // namespace sb
