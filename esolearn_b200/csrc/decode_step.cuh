// Persistent decode step: one cooperative kernel per llama decode step of a
// single sequence (see decode_step.cu).
#pragma once

#include "misc.cuh"
#include "tp_comm.cuh"
#include "qgemv.cuh"

namespace sb {

constexpr int DS_TN = 128;  // tile width of every packed weight the persistent step reads
constexpr int DS_CONSUMERS = 256;
constexpr int DS_THREADS = DS_CONSUMERS + 32;
// A ring stage is 32 KB: two 16 KB work units of one weight tile (16
// k-steps; one unit at a tile edge), or one KV chunk (K rows in the first
// half, V rows in the second).  Two k-steps per consumer warp per stage
// amortise the per-stage mbarrier handshake.
constexpr int DS_STAGE = 32768;
constexpr int DS_UNIT_KS = 8;                    // k-steps per 16 KB work unit (the split granularity)
constexpr int DS_KPS = DS_STAGE / (DS_TN * 16);  // k-steps per full stage (16)
constexpr int DS_KV_HALF = DS_STAGE / 2;         // bytes of K (and of V) per attention stage
constexpr int DS_QMAX_H = 8;   // input quads per consumer thread for rows of width h or q_dim (<= 8192)
constexpr int DS_QMAX_F = 16;  // ... for the SwiGLU row of width F (<= 16384)
constexpr int DS_MAX_NST = 16;
constexpr int DS_STAMPS = 5;  // timeline readings per phase and CTA

struct DsSmem {
    size_t ring, pa, red, qs, kvnew, bars, total;
};

// pa: the fixed-point planes of a GEMV input; during attention, the
// cross-warp reduction of the per-head outputs; in the attention-combine
// input stage, the table of partial-record weights (mtab bytes).
__host__ __device__ inline DsSmem ds_layout(int nst, int ksmax, int rep, int hd, int chunk, int mtab) {
    DsSmem L;
    L.ring = 0;
    L.pa = (size_t)nst * DS_STAGE;
    size_t pa = (size_t)48 * ksmax;
    const size_t att_red = (size_t)8 * rep * (hd + 2) * 4;
    if (att_red > pa) pa = att_red;
    if ((size_t)mtab > pa) pa = (size_t)mtab;
    L.red = L.pa + ((pa + 127) & ~(size_t)127);
    L.qs = L.red + (size_t)8 * DS_TN * 8;
    L.kvnew = L.qs + (size_t)rep * hd * 4;
    L.bars = L.kvnew + (size_t)2 * hd * 4;
    L.total = L.bars + (size_t)2 * nst * 8;
    return L;
}


// Floats per attention partial record: hd outputs, the running max and sum,
// padded so every record starts on a 16-byte boundary.
#define DS_REC(hd) ((hd) + 4)

struct DsLayer {
    const uint4 *w[4] = {nullptr, nullptr, nullptr, nullptr};  // qkv, o, gate/up (paired), down
    float scale[4] = {0.f, 0.f, 0.f, 0.f};
    float scale_up = 0.f;  // up half of the gate/up pair
};

struct DsArgs {
    int L = 0, h = 0, F = 0, V = 0, nh = 0, nkv = 0, hd = 0, q_dim = 0, kv_dim = 0;
    int V_lm = 0;  // lm_head rows (logits) of this rank: V, or the rank's slice under tensor parallelism
    int ks_h = 0, ks_q = 0, ks_f = 0;                        // input widths / 16, rounded up
    int nt_qkv = 0, nt_o = 0, nt_gu = 0, nt_down = 0, nt_lm = 0;  // 128-column tiles
    const DsLayer *layers = nullptr;                         // [L] (device)
    const uint4 *lm_w = nullptr;
    float lm_scale = 0.f;
    const float *embed = nullptr, *norm_in = nullptr, *norm_post = nullptr, *norm_final = nullptr;
    float eps = 1e-5f, q_scale = 1.f;
    void *kc = nullptr, *vc = nullptr;
    size_t layer_kv_bytes = 0;
    int kv_f32 = 0;
    int page_size = 0, max_pages = 0, max_pos = 0;
    int chunk = 0;  // positions per K (or V) ring stage; divides page_size
    const int *page_table = nullptr;
    const float *rope_cos = nullptr, *rope_sin = nullptr;
    SeqState seq;
    float *x = nullptr;         // [2][h] residual stream, alternating versions
    long long *acc = nullptr;   // [3][acc_n] exact int64 column sums of the last three GEMVs
    int acc_n = 0;
    float *part = nullptr;      // attention partials [nkv][grid][rep][DS_REC(hd)]
    float *act = nullptr;       // [F] SwiGLU output
    float *logits = nullptr;    // [V]
    float *cand_val = nullptr;  // [grid] per-CTA argmax candidates
    int *cand_idx = nullptr;
    unsigned *sync = nullptr;   // [0] phase arrivals, [1] exits, [2] abort flag (zeroed by the host)
    float *trace = nullptr;     // [L][h] residual after each layer, or nullptr
    unsigned long long *stamps = nullptr;  // optional timeline [phases][grid][DS_STAMPS] (%globaltimer ns)
    int greedy = 1;  // 1: the last CTA records the argmax and advances the sequence; 0: a sampler follows
    // >= 0: this step's token and position, given at launch (the host wrote no
    // sequence state for it; the prompt is then empty); else read from seq
    int tok_in = -1, pos_in = -1;
    // Tensor parallelism (tp > 1): shapes above are this rank's shard (heads,
    // ffn columns, vocabulary rows); the o and down partial products and the
    // argmax candidates travel through cells[r] = rank r's [2][tp][h + 2]
    // 8-byte cells (value, epoch), mapped into every rank.  The exchanges of
    // one step use epochs epoch0 + 1 .. epoch0 + 2L + 1 (one per o, one per
    // down, one for the argmax); slot parity = epoch & 1.
    int tp = 1, tp_rank = 0;
    uint2 *cells[TP_MAX_RANKS] = {};
    unsigned epoch0 = 0;
    int v_off = 0;  // first vocabulary index of this rank's lm_head rows
    int nst = 0;                // ring stages
    int mtab_bytes = 0;         // attention-combine table (ds_mtab_bytes)
};

// Whether the persistent step handles this model shape (batch 1).  When it
// does, *chunk receives the KV positions per ring stage.
bool ds_supported(int h, int F, int q_dim, int hd, int rep, int kv_f32, int page_size, int *chunk);
// Ring depth and dynamic shared memory for the shape; 0 stages when it does not fit.
int ds_plan(int ksmax, int rep, int hd, int chunk, int kv_f32, int mtab, int *nst, size_t *smem);
// Number of CTAs (one per SM).
int ds_grid();
// Whether the step kernels were compiled with the phase timeline (SB_STEP_TIMELINE).
bool ds_timeline_built();
size_t ds_part_floats(int nkv, int rep, int hd);
int ds_mtab_bytes(int nh, int nkv);
int ds_launch(const DsArgs &a, int rep, cudaStream_t st);
// Queues a copy of the abort flag into *host (pinned) on st, for a check after the
// caller's next synchronisation.
int ds_error_peek(const unsigned *sync_dev, unsigned *host, cudaStream_t st);
// Reads and clears the abort flag; SB_ERR_TIMEOUT when a bounded wait ran out.
int ds_check_error(unsigned *sync_dev, cudaStream_t st);

}  // namespace sb
