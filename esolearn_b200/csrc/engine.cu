// The quantized Llama decode engine behind sb_llama_* (sb_api.h).
//
// Replaces LlamaModel::forward_with_llama_cache (llama.rs:744-763) and the
// generate() loop (generate.rs:51-89) for int8 weights.  One decode step of
// `M` sequences is 5 kernels per layer plus embedding, lm_head and argmax:
//
//   embed -> [ QKV GEMV (input RMSNorm fused; RoPE, q scale, K/V page write
//              in the epilogue) -> paged GQA attention -> O GEMV (+residual)
//              -> gate/up GEMV (post-attention RMSNorm fused; SwiGLU in the
//              epilogue) -> down GEMV (+residual) ] x L
//   -> lm_head GEMV (final RMSNorm fused; logits + per-tile argmax)
//   -> argmax (token bookkeeping on device)
//
// The step reads every position-dependent value (token, position, page
// table) from device memory, so it is captured once per batch size as a
// CUDA graph and replayed; consecutive kernels use programmatic dependent
// launch so the next GEMV starts streaming its weights while the previous
// kernel drains.
//
// A single sequence (batch 1) runs instead as one persistent cooperative
// kernel per step (decode_step.cu) whenever the shape allows it; every
// packed weight then uses the 128-column tiles that kernel streams.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <vector>

#include "attention.cuh"
#include "decode_step.cuh"
#include "misc.cuh"
#include "qgemm.cuh"
#include "qgemv.cuh"
#include "sampler.cuh"
#include "tp_comm.cuh"

namespace sb {

struct DevBuf {
    void *p = nullptr;
    size_t bytes = 0;
};

}  // namespace sb

using namespace sb;

struct sb_llama {
    sb_llama_config cfg{};
    int dev = 0;
    // h, V: full hidden size and vocabulary; F, nh, nkv, q/kv dims and Vl:
    // this rank's share under tensor parallelism (the full values at tp = 1)
    int h = 0, F = 0, V = 0, L = 0, nh = 0, nkv = 0, hd = 0, q_dim = 0, kv_dim = 0, qkv_dim = 0;
    int Vl = 0;
    int tp = 1, tp_rank = 0;
    TpComm comm;
    float *cand_all_val = nullptr, *logits_all = nullptr;  // all ranks' candidates / logits
    int *cand_all_idx = nullptr;
    int B = 1, P = 64, pps = 0;
    cudaStream_t st = nullptr;
    std::vector<void *> allocs;

    // weights
    struct Layer {
        QWeightDesc qkv, o, gu, down;
        bool has[5] = {false, false, false, false, false};
    };
    std::vector<Layer> layers;
    QWeightDesc lm;
    bool has_lm = false;
    float *embed = nullptr, *norm_in = nullptr, *norm_post = nullptr, *norm_final = nullptr;
    int8_t *stage = nullptr;  // gate staging for gate/up pairing
    size_t stage_bytes = 0;
    void *raw = nullptr;      // checkpoint tensors as read (sb_llama_load_hf), grown on demand
    size_t raw_bytes = 0;
    int staged_gate_layer = -1;
    float staged_gate_scale = 0.0f;
    unsigned *amax = nullptr;
    float *scale_dev = nullptr;

    // KV cache
    void *kc = nullptr, *vc = nullptr;
    size_t layer_kv_elems = 0;
    int kv_f32 = 0;
    int *page_table = nullptr;
    float *rope_cos = nullptr, *rope_sin = nullptr;

    // activations
    float *x = nullptr, *q = nullptr, *attn = nullptr, *act = nullptr, *logits = nullptr, *cand_val = nullptr;
    int *cand_idx = nullptr;
    float *att_part = nullptr;
    unsigned *att_cnt = nullptr;
    int att_splits = 1;
    bool att_tma = false;  // K/V tensor maps for the tensor-map attention kernel
    CUtensorMap att_tmk, att_tmv;

    // sequence state
    SeqState seq;
    int *d_tok = nullptr, *d_pos = nullptr, *d_prompt = nullptr, *d_plen = nullptr, *d_out = nullptr,
        *d_ngen = nullptr, *d_last = nullptr;
    double *samp_prob = nullptr;  // device sampler: [B][V] probabilities, rng states, tokens
    uint64_t *d_rng = nullptr;
    int *d_samp = nullptr;
    int active = 0;  // batch of the current begin()
    int steps = 0;   // steps queued since begin()

    // graphs per batch size: greedy steps, and steps ending in the device sampler
    std::vector<cudaGraphExec_t> graphs, sgraphs, pgraphs;  // + prefill chunks (rows = positions of one sequence)
    // device sampling loop (sb_llama_set_sampling)
    bool samp_on = false;
    SampleCfg samp;
    int *d_state_bak = nullptr;  // [4][B] sequence state saved around a graph capture's warm-up
    std::vector<DsLayer> ds_tab;  // the layer table last uploaded for the step kernel
    bool trace = false;
    float *trace_buf = nullptr;
    int trace_batch = 0;

    // persistent batch-1 step
    bool ds_ok = false;
    unsigned ds_epoch = 0;  // tensor parallelism: epochs of the step kernel's exchanges so far
    unsigned *err_host = nullptr;  // pinned [5]: the kernels' error words, read with a step's own sync
    int ds_chunk = 0, ds_nst = 0;
    DsLayer *ds_layers = nullptr;  // device copy of the per-layer weight table
    float *ds_x = nullptr;
    long long *ds_acc = nullptr;
    int ds_acc_n = 0;
    float *ds_part = nullptr, *ds_cand_val = nullptr;
    int *ds_cand_idx = nullptr;
    unsigned *ds_sync = nullptr;
    unsigned long long *ds_stamps = nullptr;  // timeline of the last step (sb_llama_set_timeline)

    // batched steps of 5-64 sequences: tensor-core linears and their scratch
    QGemmWs gws;
};

namespace {

int dalloc(sb_llama *m, void **p, size_t bytes) {
    if (bytes == 0) bytes = 16;
    cudaError_t e = cudaMalloc(p, bytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return set_error(SB_ERR_OOM, "cudaMalloc(%zu) failed: %s", bytes, cudaGetErrorString(e));
    }
    m->allocs.push_back(*p);
    SB_CUDA_TRY(cudaMemsetAsync(*p, 0, bytes, m->st));
    return SB_OK;
}

template <typename T>
int dalloc_t(sb_llama *m, T **p, size_t count) {
    return dalloc(m, reinterpret_cast<void **>(p), count * sizeof(T));
}

int make_qweight(sb_llama *m, QWeightDesc &d, int K, int N, int min_tn) {
    d.K = K;
    d.N = N;
    d.KS = ceil_div(K, 16);
    d.TN = (m->ds_ok || m->B > QG_MAX_M) ? DS_TN : qgemv_pick_tn(N, K, min_tn);
    d.ntiles = ceil_div(N, d.TN);
    d.group = 0;
    void *p = nullptr;
    SB_TRY(dalloc(m, &p, qweight_bytes(K, N, d.TN)));
    d.w = reinterpret_cast<const uint4 *>(p);
    return SB_OK;
}

void host_rope_tables(const sb_llama_config &c, int hd, std::vector<float> &cs, std::vector<float> &sn) {
    // compute_rope_freqs (llama.rs:1035-1067) in f64, cast to f32 (llama.rs:621),
    // then cos/sin of pos * f64(freq) in f64 rounded to f32 (cpu.rs:650-653).
    const int half = hd / 2;
    std::vector<double> fr(half);
    const double th = (double)c.rope_theta;
    for (int i = 0; i < half; i++) fr[i] = 1.0 / std::pow(th, 2.0 * (double)i / (double)hd);
    if (c.has_rope_scaling) {
        const double factor = c.rope_scaling[0], low = c.rope_scaling[1], high = c.rope_scaling[2],
                     old_ctx = c.rope_scaling[3];
        const double low_wl = old_ctx / low, high_wl = old_ctx / high;
        for (int i = 0; i < half; i++) {
            const double wl = 2.0 * 3.14159265358979323846 / fr[i];
            double sf;
            if (wl < high_wl) sf = 1.0;
            else if (wl > low_wl) sf = factor;
            else {
                const double smooth = (old_ctx / wl - low) / (high - low);
                sf = 1.0 / ((1.0 - smooth) / factor + smooth);
            }
            fr[i] /= sf;
        }
    }
    cs.resize((size_t)c.max_seq_len * half);
    sn.resize((size_t)c.max_seq_len * half);
    for (int p = 0; p < c.max_seq_len; p++)
        for (int i = 0; i < half; i++) {
            const double angle = (double)p * (double)(float)fr[i];
            cs[(size_t)p * half + i] = (float)std::cos(angle);
            sn[(size_t)p * half + i] = (float)std::sin(angle);
        }
}

QGemvArgs gemv_common(const QWeightDesc &w, int M, const void *x, int ldx) {
    QGemvArgs a;
    a.w = w;
    a.M = M;
    a.x = x;
    a.ldx = ldx;
    return a;
}

// Per-kernel event timing of an eager step (sb_llama_profile_step).
struct StepProfiler {
    std::vector<cudaEvent_t> ev;  // pairs
    std::vector<int> cls;         // 0 gemv, 1 attention, 2 other
    cudaStream_t st = nullptr;
    int begin(int c) {
        cudaEvent_t a, b;
        SB_CUDA_TRY(cudaEventCreate(&a));
        SB_CUDA_TRY(cudaEventCreate(&b));
        ev.push_back(a);
        ev.push_back(b);
        cls.push_back(c);
        SB_CUDA_TRY(cudaEventRecord(a, st));
        return SB_OK;
    }
    int end() {
        SB_CUDA_TRY(cudaEventRecord(ev.back(), st));
        return SB_OK;
    }
    ~StepProfiler() {
        for (auto e : ev) cudaEventDestroy(e);
    }
};

// Context splits of the tensor-map attention for M sequences: at most one
// wave of CTAs (two per SM fit), so every CTA streams one long run of tiles
// and none waits for a second wave; within the split scratch the engine
// allocated (M * splits <= B * att_splits).  Measured at 8B bs32 (256
// (sequence, kv head) pairs): 1 split 1.62 ms of attention per step, 2 splits
// 1.99 ms, 3 splits 2.19 ms, 4 splits 2.06 ms.
int tma_splits(const sb_llama *m, int M) {
    const int want = 2 * device_props().sm_count / std::max(1, M * m->nkv);
    const int cap = std::max(1, m->B * m->att_splits / M);
    return std::max(1, std::min({want, cap, ceil_div(m->cfg.max_seq_len, 128)}));
}

// O and down projections add into the residual stream x.  Under tensor
// parallelism each rank holds a row slice of the weight, so rank 0 adds its
// partial product to x and the other ranks store theirs; the sum over ranks
// (NCCL all-reduce over NVLink, in place) is then x + sum of partials
// (llama.rs:564,568).
int resid_epi(const sb_llama *m) { return (m->tp > 1 && m->tp_rank != 0) ? QEPI_STORE : QEPI_RESID; }
int tp_reduce_residual(sb_llama *m, int M, cudaStream_t st) {
    if (m->tp == 1) return SB_OK;
    return tp_allreduce_f32(m->comm, m->x, (size_t)M * m->h, st);
}

// One linear of a step: the GEMV for up to 4 rows, the tensor-core GEMM for
// 5-64 (every weight then has 128-column tiles).
int engine_linear(sb_llama *m, int epi, const QGemvArgs &a, cudaStream_t st, bool pdl) {
    if (a.M > QG_MAX_M) return qgemm_launch(epi, a, m->gws, st, pdl);
    return qgemv_launch(epi, a, st, pdl);
}

#define SB_PROF(p, c, expr)                \
    do {                                   \
        if (p) SB_TRY((p)->begin(c));      \
        SB_TRY(expr);                      \
        if (p) SB_TRY((p)->end());         \
    } while (0)

// Enqueue one decode step for M sequences on st.
// What a queued step ends in, and how its attention runs: greedy (argmax),
// sampled (the device sampler), or a prefill chunk -- rows are consecutive
// prompt positions of one sequence (page-table row 0 holds its pages), the
// attention may read each K/V tile once for all rows (attention_prefill.cu),
// and the step ends in the argmax.
enum StepKind { STEP_GREEDY = 0, STEP_SAMPLED = 1, STEP_PREFILL = 2 };

int enqueue_step(sb_llama *m, int M, cudaStream_t st, bool pdl, bool trace, StepProfiler *prof = nullptr,
                 int kind = STEP_GREEDY) {
    const bool sampled = kind == STEP_SAMPLED;
    // The prefill kernel replaces the per-row attention where that runs on the
    // SIMT kernel (one query head per kv head); with 2-8 heads per kv head the
    // tensor-map kernel is as fast or faster (its grid has 8x more CTAs).
    const bool flash =
        kind == STEP_PREFILL && M > 1 && m->nh == m->nkv && attn_prefill_supported(m->hd, m->kv_f32);
    // Batches of 5+ rows on one GPU chain the tensor-core linears: the finish
    // of o, gate/up and down (whose output row is the next linear's input)
    // also writes the next linear's planes, one launch instead of two.
    const bool chain = M > QG_MAX_M && m->tp == 1;
    bool planes_ready = false;  // the previous link wrote this linear's planes
    // With the tensor-map attention in one split, the q|k|v GEMM's epilogue
    // (RoPE, q scale, the K/V row write) runs inside the attention kernel,
    // which reads the GEMM's sums: one launch less per layer.
    const bool fuse_qkv = M > QG_MAX_M && m->att_tma && tma_splits(m, M) == 1 && kind != STEP_PREFILL;
    auto linear = [&](int epi, const QGemvArgs &a, const float *next_norm) -> int {
        if (!chain) {
            if (epi == QEPI_QKV && fuse_qkv)
                return qgemm_launch_chained(epi, a, m->gws, st, pdl, true, nullptr, true);
            return engine_linear(m, epi, a, st, pdl);
        }
        const bool chained = epi == QEPI_RESID || epi == QEPI_SWIGLU;
        QGemmNext nx;
        nx.norm_w = next_norm;
        nx.eps = m->cfg.rms_norm_eps;
        nx.planes_bytes = qgemm_planes_bytes(std::max({m->h, m->F, m->q_dim}), m->B);
        const bool need = !planes_ready;
        planes_ready = chained;
        return qgemm_launch_chained(epi, a, m->gws, st, pdl, need, chained ? &nx : nullptr,
                                    epi == QEPI_QKV && fuse_qkv);
    };
    SB_PROF(prof, 2, embed_launch(m->embed, m->h, m->V, m->seq, M, m->x, st, pdl));
    for (int l = 0; l < m->L; l++) {
        const sb_llama::Layer &ly = m->layers[l];
        const size_t kvoff = (size_t)l * m->layer_kv_elems * (m->kv_f32 ? 4 : 2);
        {
            QGemvArgs a = gemv_common(ly.qkv, M, m->x, m->h);
            a.norm_w = m->norm_in + (size_t)l * m->h;
            a.eps = m->cfg.rms_norm_eps;
            a.q_out = m->q;
            a.q_dim = m->q_dim;
            a.kv_dim = m->kv_dim;
            a.hd = m->hd;
            a.n_kv = m->nkv;
            a.kcache = (char *)m->kc + kvoff;
            a.vcache = (char *)m->vc + kvoff;
            a.kv_f32 = m->kv_f32;
            a.page_size = m->P;
            a.max_pages = m->pps;
            a.page_table = m->page_table;
            a.pos = m->d_pos;
            a.max_pos = m->cfg.max_seq_len;
            a.rope_cos = m->rope_cos;
            a.rope_sin = m->rope_sin;
            a.q_scale = (float)(1.0 / std::sqrt((double)m->hd));  // llama.rs:394
            SB_PROF(prof, 0, linear(QEPI_QKV, a, nullptr));
        }
        if (flash) {
            PrefillAttnArgs a;
            a.q = m->q;
            a.kc = (char *)m->kc + kvoff;
            a.vc = (char *)m->vc + kvoff;
            a.kv_f32 = m->kv_f32;
            a.page_table = m->page_table;
            a.max_pages = m->pps;
            a.pos = m->d_pos;
            a.M = M;
            a.n_heads = m->nh;
            a.n_kv = m->nkv;
            a.hd = m->hd;
            a.page_size = m->P;
            a.out = m->attn;
            SB_PROF(prof, 1, attn_prefill_launch(a, st, pdl));
        } else {
            AttnArgs a;
            a.q = m->q;
            a.kc = (char *)m->kc + kvoff;
            a.vc = (char *)m->vc + kvoff;
            a.kv_f32 = m->kv_f32;
            a.page_table = m->page_table;
            a.max_pages = m->pps;
            a.len = m->d_pos;
            a.len_is_pos = 1;
            a.B = M;
            a.n_heads = m->nh;
            a.n_kv = m->nkv;
            a.hd = m->hd;
            a.page_size = m->P;
            a.n_splits = m->att_tma ? tma_splits(m, M) : m->att_splits;
            a.out = m->attn;
            a.part = m->att_part;
            a.counters = m->att_cnt;
            if (m->att_tma) {
                a.tma = 1;
                a.tmk = m->att_tmk;
                a.tmv = m->att_tmv;
                a.tm_row0 = (long long)l * (long long)(m->layer_kv_elems / m->hd);
            }
            if (fuse_qkv) {
                a.qkv_sums = m->gws.acc;
                a.ld_sums = m->gws.ld_acc;
                a.shift = m->gws.shift;
                a.rstd = m->gws.rstd;
                a.qkv_scale = ly.qkv.scale;
                a.q_scale = (float)(1.0 / std::sqrt((double)m->hd));  // llama.rs:394
                a.rope_cos = m->rope_cos;
                a.rope_sin = m->rope_sin;
                a.max_pos = m->cfg.max_seq_len;
            }
            SB_PROF(prof, 1, attn_launch(a, st, pdl));
        }
        {
            QGemvArgs a = gemv_common(ly.o, M, m->attn, m->q_dim);
            a.out = m->x;
            a.ldo = m->h;
            SB_PROF(prof, 0, linear(resid_epi(m), a, m->norm_post + (size_t)l * m->h));
            SB_TRY(tp_reduce_residual(m, M, st));
        }
        {
            QGemvArgs a = gemv_common(ly.gu, M, m->x, m->h);
            a.norm_w = m->norm_post + (size_t)l * m->h;
            a.eps = m->cfg.rms_norm_eps;
            a.out = m->act;
            a.ldo = m->F;
            a.F = m->F;
            SB_PROF(prof, 0, linear(QEPI_SWIGLU, a, nullptr));
        }
        {
            QGemvArgs a = gemv_common(ly.down, M, m->act, m->F);
            a.out = m->x;
            a.ldo = m->h;
            SB_PROF(prof, 0, linear(resid_epi(m), a, l + 1 < m->L ? m->norm_in + (size_t)(l + 1) * m->h : m->norm_final));
            SB_TRY(tp_reduce_residual(m, M, st));
        }
        if (trace)
            SB_CUDA_TRY(cudaMemcpyAsync(m->trace_buf + (size_t)l * M * m->h, m->x, sizeof(float) * M * m->h,
                                        cudaMemcpyDeviceToDevice, st));
    }
    {
        QGemvArgs a = gemv_common(m->lm, M, m->x, m->h);
        a.norm_w = m->norm_final;
        a.eps = m->cfg.rms_norm_eps;
        a.out = m->logits;
        a.ldo = m->Vl;
        a.cand_val = m->cand_val;
        a.cand_idx = m->cand_idx;
        SB_PROF(prof, 0, linear(QEPI_LOGITS, a, nullptr));
    }
    if (m->tp > 1) {
        // every rank's per-tile candidates [rank][row][tile]; rank r's columns start at r * Vl
        const size_t n = (size_t)M * m->lm.ntiles;
        SB_TRY(tp_allgather32(m->comm, m->cand_val, m->cand_all_val, n, st));
        SB_TRY(tp_allgather32(m->comm, m->cand_idx, m->cand_all_idx, n, st));
        SB_PROF(prof, 2, argmax_step_launch(m->cand_all_val, m->cand_all_idx, m->lm.ntiles, m->seq, M, st, pdl,
                                            m->tp, (int)n, m->Vl));
    } else if (sampled) {
        SB_PROF(prof, 2, sample_step_launch(m->logits, M, m->V, m->Vl, m->samp, m->d_rng, m->samp_prob, m->seq, st));
    } else {
        SB_PROF(prof, 2, argmax_step_launch(m->cand_val, m->cand_idx, m->lm.ntiles, m->seq, M, st, pdl));
    }
    return SB_OK;
}

int check_ready(sb_llama *m) {
    for (int l = 0; l < m->L; l++)
        for (int s = 0; s < 5; s++)
            SB_CHECK(m->layers[l].has[s], SB_ERR_STATE, "weight (layer %d, slot %d) not loaded", l, s);
    SB_CHECK(m->has_lm, SB_ERR_STATE, "lm_head not loaded");
    return SB_OK;
}

int set_state(sb_llama *m, int M, const int32_t *tok, const int32_t *pos, const int32_t *plen);

// One batch-1 step as the persistent kernel (m->ds_ok).
// tok_in / pos_in >= 0: the step's token and position as launch arguments
// (no sequence state uploaded first).
int ds_step(sb_llama *m, bool sampled = false, int tok_in = -1, int pos_in = -1) {
    std::vector<DsLayer> tab(m->L);
    for (int l = 0; l < m->L; l++) {
        const sb_llama::Layer &ly = m->layers[l];
        const QWeightDesc *w[4] = {&ly.qkv, &ly.o, &ly.gu, &ly.down};
        for (int i = 0; i < 4; i++) {
            tab[l].w[i] = w[i]->w;
            tab[l].scale[i] = w[i]->scale;
        }
        tab[l].scale_up = ly.gu.scale_up;
    }
    if (m->ds_tab.size() != tab.size() ||
        std::memcmp(m->ds_tab.data(), tab.data(), sizeof(DsLayer) * tab.size()) != 0) {
        // weights were (re)loaded: upload the table once, not every step
        SB_CUDA_TRY(cudaMemcpyAsync(m->ds_layers, tab.data(), sizeof(DsLayer) * tab.size(), cudaMemcpyHostToDevice,
                                    m->st));
        SB_CUDA_TRY(cudaStreamSynchronize(m->st));  // tab is a local: the copy must finish before it goes
        m->ds_tab = tab;
    }
    DsArgs a;
    a.L = m->L;
    a.h = m->h;
    a.F = m->F;
    a.V = m->V;
    a.V_lm = m->Vl;
    a.nh = m->nh;
    a.nkv = m->nkv;
    a.hd = m->hd;
    a.q_dim = m->q_dim;
    a.kv_dim = m->kv_dim;
    a.ks_h = ceil_div(m->h, 16);
    a.ks_q = ceil_div(m->q_dim, 16);
    a.ks_f = ceil_div(m->F, 16);
    const sb_llama::Layer &l0 = m->layers[0];
    a.nt_qkv = l0.qkv.ntiles;
    a.nt_o = l0.o.ntiles;
    a.nt_gu = l0.gu.ntiles;
    a.nt_down = l0.down.ntiles;
    a.nt_lm = m->lm.ntiles;
    a.layers = m->ds_layers;
    a.lm_w = m->lm.w;
    a.lm_scale = m->lm.scale;
    a.embed = m->embed;
    a.norm_in = m->norm_in;
    a.norm_post = m->norm_post;
    a.norm_final = m->norm_final;
    a.eps = m->cfg.rms_norm_eps;
    a.q_scale = (float)(1.0 / std::sqrt((double)m->hd));  // llama.rs:394
    a.kc = m->kc;
    a.vc = m->vc;
    a.layer_kv_bytes = m->layer_kv_elems * (m->kv_f32 ? 4 : 2);
    a.kv_f32 = m->kv_f32;
    a.page_size = m->P;
    a.max_pages = m->pps;
    a.max_pos = m->cfg.max_seq_len;
    a.chunk = m->ds_chunk;
    a.page_table = m->page_table;
    a.rope_cos = m->rope_cos;
    a.rope_sin = m->rope_sin;
    a.seq = m->seq;
    a.x = m->ds_x;
    a.acc = m->ds_acc;
    a.acc_n = m->ds_acc_n;
    a.part = m->ds_part;
    a.act = m->act;
    a.logits = m->logits;
    a.cand_val = m->ds_cand_val;
    a.cand_idx = m->ds_cand_idx;
    a.sync = m->ds_sync;
    a.trace = m->trace ? m->trace_buf : nullptr;
    a.nst = m->ds_nst;
    a.mtab_bytes = ds_mtab_bytes(m->nh, m->nkv);
    a.stamps = m->ds_stamps;
    a.greedy = sampled ? 0 : 1;
    a.tok_in = tok_in;
    a.pos_in = pos_in;
    if (m->tp > 1) {
        a.tp = m->tp;
        a.tp_rank = m->tp_rank;
        for (int r = 0; r < m->tp; r++) a.cells[r] = m->comm.cells[r];
        a.epoch0 = m->ds_epoch;
        a.v_off = m->tp_rank * m->Vl;
        m->ds_epoch += 2 * m->L + 1;  // the exchanges of this step
    }
    SB_TRY(ds_launch(a, m->nh / m->nkv, m->st));
    if (sampled) SB_TRY(sample_step_launch(m->logits, 1, m->V, m->Vl, m->samp, m->d_rng, m->samp_prob, m->seq, m->st));
    return SB_OK;
}

// Errors a bounded device wait may have left behind.
// Queue copies of every kernel error word into the pinned err_host, so the
// caller's one synchronisation also brings them back (no extra round trips).
// step_only: the call ran only the persistent step kernel, whose abort flag
// is then the only word it can have set.
int queue_error_peeks(sb_llama *m, bool step_only = false) {
    unsigned *h = m->err_host;
    h[0] = h[1] = h[2] = h[3] = h[4] = 0;
    if (m->ds_ok) SB_TRY(ds_error_peek(m->ds_sync, h + 0, m->st));
    if (step_only) return SB_OK;
    SB_TRY(qgemm_error_peek(h + 1, m->st));
    SB_TRY(attn_tc_error_peek(h + 2, m->st));
    if (m->tp > 1) SB_TRY(tp_error_peek(m->comm, h + 3, m->st));
    return qgemv_error_peek(h + 4, m->st);
}

int check_device_errors(sb_llama *m) {
    if (m->ds_ok) SB_TRY(ds_check_error(m->ds_sync, m->st));
    SB_TRY(qgemm_check_error());
    SB_TRY(attn_tc_check_error());
    if (m->tp > 1) SB_TRY(tp_check_error(m->comm));
    return qgemv_check_error();
}

int get_graph(sb_llama *m, int M, cudaGraphExec_t *out, int kind = STEP_GREEDY) {
    std::vector<cudaGraphExec_t> &cache = kind == STEP_SAMPLED ? m->sgraphs : kind == STEP_PREFILL ? m->pgraphs : m->graphs;
    if (cache[M]) {
        *out = cache[M];
        return SB_OK;
    }
    // Warm up once outside capture (sets kernel attributes, loads modules)
    // at position -1, which writes no K/V row, reads no context and draws
    // nothing, so the caches of live sequences are untouched; the sequence
    // state of rows 0..M-1 is saved around it and put back.
    const size_t sb = sizeof(int) * M;
    int *bak = m->d_state_bak;
    SB_CUDA_TRY(cudaMemcpyAsync(bak, m->d_tok, sb, cudaMemcpyDeviceToDevice, m->st));
    SB_CUDA_TRY(cudaMemcpyAsync(bak + m->B, m->d_pos, sb, cudaMemcpyDeviceToDevice, m->st));
    SB_CUDA_TRY(cudaMemcpyAsync(bak + 2 * m->B, m->d_plen, sb, cudaMemcpyDeviceToDevice, m->st));
    SB_CUDA_TRY(cudaMemcpyAsync(bak + 3 * m->B, m->d_ngen, sizeof(int) * m->B, cudaMemcpyDeviceToDevice, m->st));
    std::vector<int32_t> zero(M, 0), before(M, -1);
    SB_TRY(set_state(m, M, zero.data(), before.data(), zero.data()));
    SB_TRY(enqueue_step(m, M, m->st, true, false, nullptr, kind));
    SB_CUDA_TRY(cudaMemcpyAsync(m->d_tok, bak, sb, cudaMemcpyDeviceToDevice, m->st));
    SB_CUDA_TRY(cudaMemcpyAsync(m->d_pos, bak + m->B, sb, cudaMemcpyDeviceToDevice, m->st));
    SB_CUDA_TRY(cudaMemcpyAsync(m->d_plen, bak + 2 * m->B, sb, cudaMemcpyDeviceToDevice, m->st));
    SB_CUDA_TRY(cudaMemcpyAsync(m->d_ngen, bak + 3 * m->B, sizeof(int) * m->B, cudaMemcpyDeviceToDevice, m->st));
    SB_CUDA_TRY(cudaStreamSynchronize(m->st));
    cudaGraph_t g = nullptr;
    SB_CUDA_TRY(cudaStreamBeginCapture(m->st, cudaStreamCaptureModeThreadLocal));
    int rc = enqueue_step(m, M, m->st, true, false, nullptr, kind);
    cudaError_t e = cudaStreamEndCapture(m->st, &g);
    if (rc != SB_OK) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    SB_CUDA_TRY(e);
    cudaGraphExec_t ge = nullptr;
    e = cudaGraphInstantiate(&ge, g, 0);
    cudaGraphDestroy(g);
    SB_CUDA_TRY(e);
    cache[M] = ge;
    *out = ge;
    return SB_OK;
}

// Put sequences 0..M-1 at the given start state (host arrays).
int set_state(sb_llama *m, int M, const int32_t *tok, const int32_t *pos, const int32_t *plen) {
    SB_CUDA_TRY(cudaMemcpyAsync(m->d_tok, tok, sizeof(int) * M, cudaMemcpyHostToDevice, m->st));
    SB_CUDA_TRY(cudaMemcpyAsync(m->d_pos, pos, sizeof(int) * M, cudaMemcpyHostToDevice, m->st));
    SB_CUDA_TRY(cudaMemcpyAsync(m->d_plen, plen, sizeof(int) * M, cudaMemcpyHostToDevice, m->st));
    SB_CUDA_TRY(cudaMemsetAsync(m->d_ngen, 0, sizeof(int) * m->B, m->st));
    return SB_OK;
}

}  // namespace

extern "C" {

}  // extern "C"

namespace {

// Rank r's slice of a full reference tensor under tensor parallelism
// (Megatron-style): column slices of q|k|v (by heads), gate and up (by ffn
// columns); row slices of o (by heads), down (by ffn rows) and the [V,h]
// lm_head (by vocabulary rows).  Shapes in rows x cols of the reference
// layout; with src == nullptr only the shapes are returned.
int tp_shard(const sb_llama_config &c, int slot, int r, int T, const int8_t *src, int8_t *dst, int *rows,
             int *cols) {
    SB_CHECK(T >= 1 && r >= 0 && r < T, SB_ERR_ARG, "tensor parallel rank %d of %d", r, T);
    SB_CHECK(c.n_heads > 0 && c.n_kv_heads > 0 && c.hidden_size % c.n_heads == 0, SB_ERR_SHAPE, "bad head counts");
    SB_CHECK(c.n_heads % T == 0 && c.n_kv_heads % T == 0 && c.intermediate_size % T == 0 && c.vocab_size % T == 0,
             SB_ERR_SHAPE, "tensor parallel %d must divide heads, kv heads, ffn and vocab", T);
    const int h = c.hidden_size, hd = h / c.n_heads;
    const int Qf = c.n_heads * hd, KVf = c.n_kv_heads * hd, q = Qf / T, kv = KVf / T;
    const int F = c.intermediate_size, Fl = F / T, V = c.vocab_size, Vl = V / T;
    // full cols (row stride), row offset, row count, then up to three column runs (src col, count)
    int fc = 0, r0 = 0, nr = 0, nrun = 1, c0[3] = {0, 0, 0}, cn[3] = {0, 0, 0};
    switch (slot) {
    case SB_W_QKV:
        fc = Qf + 2 * KVf, nr = h, nrun = 3;
        c0[0] = r * q, cn[0] = q, c0[1] = Qf + r * kv, cn[1] = kv, c0[2] = Qf + KVf + r * kv, cn[2] = kv;
        break;
    case SB_W_O: fc = h, r0 = r * q, nr = q, cn[0] = h; break;
    case SB_W_GATE:
    case SB_W_UP: fc = F, nr = h, c0[0] = r * Fl, cn[0] = Fl; break;
    case SB_W_DOWN: fc = h, r0 = r * Fl, nr = Fl, cn[0] = h; break;
    case SB_W_LM_HEAD: fc = h, r0 = r * Vl, nr = Vl, cn[0] = h; break;
    default: return set_error(SB_ERR_ARG, "tp_shard: unknown weight slot %d", slot);
    }
    int nc = 0;
    for (int i = 0; i < nrun; i++) nc += cn[i];
    if (rows) *rows = nr;
    if (cols) *cols = nc;
    if (!src) return SB_OK;
    SB_CHECK(dst, SB_ERR_ARG, "tp_shard: null destination");
    for (int i = 0; i < nr; i++) {
        const int8_t *srow = src + (size_t)(r0 + i) * fc;
        int8_t *drow = dst + (size_t)i * nc;
        for (int k = 0; k < nrun; k++) {
            std::memcpy(drow, srow + c0[k], (size_t)cn[k]);
            drow += cn[k];
        }
    }
    return SB_OK;
}

int llama_create(const sb_llama_config *cfg, int tp_rank, int tp_size, const uint8_t *tp_id, sb_llama **out) {
    SB_CHECK(cfg && out, SB_ERR_ARG, "sb_llama_create: null argument");
    const sb_llama_config &c = *cfg;
    SB_CHECK(tp_size >= 1 && tp_rank >= 0 && tp_rank < tp_size, SB_ERR_ARG, "tensor parallel rank %d of %d", tp_rank,
             tp_size);
    SB_CHECK(tp_size == 1 || tp_id, SB_ERR_ARG, "sb_llama_create_tp: null communicator id");
    SB_CHECK(c.n_heads % tp_size == 0 && c.n_kv_heads % tp_size == 0 && c.intermediate_size % tp_size == 0 &&
                 c.vocab_size % tp_size == 0,
             SB_ERR_SHAPE, "tensor parallel %d must divide heads %d, kv heads %d, ffn %d and vocab %d", tp_size,
             c.n_heads, c.n_kv_heads, c.intermediate_size, c.vocab_size);
    SB_CHECK(c.hidden_size > 0 && c.n_heads > 0 && c.n_kv_heads > 0 && c.n_layers > 0 && c.vocab_size > 0 &&
                 c.intermediate_size > 0 && c.max_seq_len > 0,
             SB_ERR_SHAPE, "sb_llama_create: non-positive dimension");
    SB_CHECK(c.hidden_size % c.n_heads == 0 && c.n_heads % c.n_kv_heads == 0, SB_ERR_SHAPE,
             "sb_llama_create: hidden %% heads or heads %% kv_heads != 0");
    SB_CHECK(c.max_batch >= 1 && c.max_batch <= QGM_MAX_M, SB_ERR_UNSUPPORTED,
             "sb_llama_create: max_batch %d outside 1..%d", c.max_batch, QGM_MAX_M);
    if (c.max_batch > QG_MAX_M) {
        // the tensor-core path reads the input in 32-element k steps
        const int qd = c.hidden_size / c.n_heads * (c.n_heads / tp_size);
        SB_CHECK(c.hidden_size % 32 == 0 && (c.intermediate_size / tp_size) % 32 == 0 && qd % 32 == 0,
                 SB_ERR_UNSUPPORTED,
                 "sb_llama_create: batches above %d need hidden, q and ffn sizes (per rank) that are multiples of 32",
                 QG_MAX_M);
    }
    const int hd = c.hidden_size / c.n_heads;
    SB_CHECK(hd == 64 || hd == 128, SB_ERR_UNSUPPORTED, "sb_llama_create: head_dim %d not in {64,128}", hd);

    sb_llama *m = new sb_llama();
    m->cfg = c;
    cudaGetDevice(&m->dev);
    m->tp = tp_size;
    m->tp_rank = tp_rank;
    m->h = c.hidden_size;
    m->F = c.intermediate_size / tp_size;
    m->V = c.vocab_size;
    m->Vl = c.vocab_size / tp_size;
    m->L = c.n_layers;
    m->nh = c.n_heads / tp_size;
    m->nkv = c.n_kv_heads / tp_size;
    m->hd = hd;
    m->q_dim = m->nh * hd;
    m->kv_dim = m->nkv * hd;
    m->qkv_dim = m->q_dim + 2 * m->kv_dim;
    m->B = c.max_batch;
    m->P = c.page_size > 0 ? c.page_size : 64;
    m->pps = ceil_div(c.max_seq_len, m->P);
    m->kv_f32 = c.kv_dtype == SB_KV_F32;
    m->graphs.assign(m->B + 1, nullptr);
    m->sgraphs.assign(m->B + 1, nullptr);
    m->pgraphs.assign(m->B + 1, nullptr);
    auto fail = [&](int rc) {
        sb_llama_destroy(m);
        return rc;
    };
    if (cudaStreamCreateWithFlags(&m->st, cudaStreamNonBlocking) != cudaSuccess)
        return fail(set_error(SB_ERR_CUDA, "cudaStreamCreate failed"));
    if (cudaMallocHost(&m->err_host, 8 * sizeof(unsigned)) != cudaSuccess)
        return fail(set_error(SB_ERR_OOM, "cudaMallocHost failed"));

    int rc = SB_OK;
    if (tp_size > 1 && (rc = tp_init(m->comm, tp_id, tp_rank, tp_size, 120.0)) != SB_OK) return fail(rc);
    if (tp_size > 1 && (rc = tp_setup_p2p(m->comm, m->B * m->h, m->st)) != SB_OK) return fail(rc);
    {
        int chunk = 0;
        if (ds_supported(m->h, m->F, m->q_dim, hd, m->nh / m->nkv, m->kv_f32, m->P, &chunk)) {
            const int ksmax = ceil_div(std::max(std::max(m->h, m->F), m->q_dim), 16);
            int nst = 0;
            size_t smem = 0;
            int coop = 0;
            cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, m->dev);
            if (coop && ds_plan(ksmax, m->nh / m->nkv, hd, chunk, m->kv_f32, ds_mtab_bytes(m->nh, m->nkv), &nst, &smem) == SB_OK &&
                nst >= 3) {
                m->ds_ok = true;
                m->ds_chunk = chunk;
                m->ds_nst = nst;
            }
        }
    }
    if (tp_size > 1) {
        // The persistent step under tensor parallelism exchanges through cells
        // in every rank's memory: all ranks must have peer access and the
        // kernel; they agree (one all-gather) before sharing the cells.
        int *flags = nullptr;
        int mine = (m->ds_ok && m->comm.p2p) ? 1 : 0;
        std::vector<int> all(tp_size, 0);
        if (cudaMalloc(&flags, sizeof(int) * (tp_size + 1)) != cudaSuccess) return fail(set_error(SB_ERR_OOM, "flags"));
        rc = SB_OK;
        if (cudaMemcpyAsync(flags + tp_size, &mine, sizeof(int), cudaMemcpyHostToDevice, m->st) != cudaSuccess)
            rc = set_error(SB_ERR_CUDA, "sb_llama_create: flag upload failed");
        if (rc == SB_OK) rc = tp_allgather32(m->comm, flags + tp_size, flags, 1, m->st);
        if (rc == SB_OK && (cudaMemcpyAsync(all.data(), flags, sizeof(int) * tp_size, cudaMemcpyDeviceToHost, m->st) !=
                                cudaSuccess ||
                            cudaStreamSynchronize(m->st) != cudaSuccess))
            rc = set_error(SB_ERR_CUDA, "sb_llama_create: flag exchange failed");
        cudaFree(flags);
        if (rc != SB_OK) return fail(rc);
        bool every = true;
        for (int v : all) every = every && v == 1;
        m->ds_ok = every;
        if (every) {
            uint2 *mapped[TP_MAX_RANKS] = {};
            if ((rc = tp_share_cells(m->comm, (size_t)2 * tp_size * (m->h + 2), m->st, mapped)) != SB_OK)
                return fail(rc);
        }
    }
    m->layers.resize(m->L);
    const int gu_cols = ceil_div(m->F, 16) * 32;  // gate/up interleaved in blocks of 16
    for (int l = 0; l < m->L && rc == SB_OK; l++) {
        sb_llama::Layer &ly = m->layers[l];
        if ((rc = make_qweight(m, ly.qkv, m->h, m->qkv_dim, 16)) != SB_OK) break;
        if ((rc = make_qweight(m, ly.o, m->q_dim, m->h, 16)) != SB_OK) break;
        if ((rc = make_qweight(m, ly.gu, m->h, gu_cols, 32)) != SB_OK) break;
        if ((rc = make_qweight(m, ly.down, m->F, m->h, 16)) != SB_OK) break;
    }
    if (rc == SB_OK) rc = make_qweight(m, m->lm, m->h, m->Vl, 16);
    if (rc == SB_OK) rc = dalloc_t(m, &m->embed, (size_t)m->V * m->h);
    if (rc == SB_OK) rc = dalloc_t(m, &m->norm_in, (size_t)m->L * m->h);
    if (rc == SB_OK) rc = dalloc_t(m, &m->norm_post, (size_t)m->L * m->h);
    if (rc == SB_OK) rc = dalloc_t(m, &m->norm_final, (size_t)m->h);
    if (rc != SB_OK) return fail(rc);
    {
        // RMSNorm::new initialises weights to 1.0 (rmsnorm.rs:17-22).
        std::vector<float> ones((size_t)m->L * m->h, 1.0f);
        cudaMemcpyAsync(m->norm_in, ones.data(), sizeof(float) * ones.size(), cudaMemcpyHostToDevice, m->st);
        cudaMemcpyAsync(m->norm_post, ones.data(), sizeof(float) * ones.size(), cudaMemcpyHostToDevice, m->st);
        cudaMemcpyAsync(m->norm_final, ones.data(), sizeof(float) * m->h, cudaMemcpyHostToDevice, m->st);
        cudaStreamSynchronize(m->st);
    }
    // staging for gate/up pairing and for on-device generation
    m->stage_bytes = std::max<size_t>((size_t)2 * m->h * m->F, (size_t)m->Vl * m->h);
    m->stage_bytes = std::max<size_t>(m->stage_bytes, (size_t)m->h * m->qkv_dim);
    if ((rc = dalloc(m, (void **)&m->stage, m->stage_bytes)) != SB_OK) return fail(rc);
    if ((rc = dalloc_t(m, &m->amax, 4)) != SB_OK) return fail(rc);
    if ((rc = dalloc_t(m, &m->scale_dev, 4)) != SB_OK) return fail(rc);

    // KV cache: pages [B*pps][n_kv][P][hd] per layer; sequence b owns pages b*pps...
    m->layer_kv_elems = (size_t)m->B * m->pps * m->nkv * m->P * m->hd;
    const size_t esz = m->kv_f32 ? 4 : 2;
    if ((rc = dalloc(m, &m->kc, m->layer_kv_elems * esz * m->L)) != SB_OK) return fail(rc);
    if ((rc = dalloc(m, &m->vc, m->layer_kv_elems * esz * m->L)) != SB_OK) return fail(rc);
    if (!m->kv_f32 && m->P % 64 == 0 && m->hd % 64 == 0) {
        // every layer's K (and V) cache as one [rows][hd] tensor for the tensor-map attention
        const long long rows = (long long)m->L * (long long)(m->layer_kv_elems / m->hd);
        m->att_tma = attn_make_tensor_map(&m->att_tmk, m->kc, rows, m->hd) == SB_OK &&
                     attn_make_tensor_map(&m->att_tmv, m->vc, rows, m->hd) == SB_OK;
    }
    {
        std::vector<int> pt((size_t)m->B * m->pps);
        for (int b = 0; b < m->B; b++)
            for (int i = 0; i < m->pps; i++) pt[(size_t)b * m->pps + i] = b * m->pps + i;
        if ((rc = dalloc_t(m, &m->page_table, pt.size())) != SB_OK) return fail(rc);
        cudaMemcpyAsync(m->page_table, pt.data(), sizeof(int) * pt.size(), cudaMemcpyHostToDevice, m->st);
        std::vector<float> cs, sn;
        host_rope_tables(c, hd, cs, sn);
        if ((rc = dalloc_t(m, &m->rope_cos, cs.size())) != SB_OK) return fail(rc);
        if ((rc = dalloc_t(m, &m->rope_sin, sn.size())) != SB_OK) return fail(rc);
        cudaMemcpyAsync(m->rope_cos, cs.data(), sizeof(float) * cs.size(), cudaMemcpyHostToDevice, m->st);
        cudaMemcpyAsync(m->rope_sin, sn.data(), sizeof(float) * sn.size(), cudaMemcpyHostToDevice, m->st);
        cudaStreamSynchronize(m->st);
    }
    // activations
    const int B = m->B;
    if ((rc = dalloc_t(m, &m->x, (size_t)B * m->h)) != SB_OK) return fail(rc);
    if ((rc = dalloc_t(m, &m->q, (size_t)B * m->q_dim)) != SB_OK) return fail(rc);
    if ((rc = dalloc_t(m, &m->attn, (size_t)B * m->q_dim)) != SB_OK) return fail(rc);
    if ((rc = dalloc_t(m, &m->act, (size_t)B * m->F)) != SB_OK) return fail(rc);
    if ((rc = dalloc_t(m, &m->logits, (size_t)B * m->Vl)) != SB_OK) return fail(rc);
    if ((rc = dalloc_t(m, &m->cand_val, (size_t)B * m->lm.ntiles)) != SB_OK) return fail(rc);
    if ((rc = dalloc_t(m, &m->cand_idx, (size_t)B * m->lm.ntiles)) != SB_OK) return fail(rc);
    m->att_splits = attn_pick_splits(B, m->nkv, c.max_seq_len);
    if ((rc = dalloc_t(m, &m->att_part, attn_scratch_floats(B, m->nh, m->att_splits, hd))) != SB_OK) return fail(rc);
    if ((rc = dalloc_t(m, &m->att_cnt, (size_t)B * m->nkv)) != SB_OK) return fail(rc);

    // sequence state
    if ((rc = dalloc_t(m, &m->d_tok, B)) != SB_OK) return fail(rc);
    if ((rc = dalloc_t(m, &m->d_pos, B)) != SB_OK) return fail(rc);
    if ((rc = dalloc_t(m, &m->d_plen, B)) != SB_OK) return fail(rc);
    if ((rc = dalloc_t(m, &m->d_prompt, (size_t)B * c.max_seq_len)) != SB_OK) return fail(rc);
    if ((rc = dalloc_t(m, &m->d_out, (size_t)B * c.max_seq_len)) != SB_OK) return fail(rc);
    if ((rc = dalloc_t(m, &m->d_ngen, B)) != SB_OK) return fail(rc);
    if ((rc = dalloc_t(m, &m->d_last, B)) != SB_OK) return fail(rc);
    if ((rc = dalloc_t(m, &m->d_state_bak, (size_t)4 * B)) != SB_OK) return fail(rc);
    m->seq.tok = m->d_tok;
    m->seq.pos = m->d_pos;
    m->seq.prompt = m->d_prompt;
    m->seq.prompt_len = m->d_plen;
    m->seq.max_prompt = c.max_seq_len;
    m->seq.out = m->d_out;
    m->seq.ngen = m->d_ngen;
    m->seq.max_gen = c.max_seq_len;
    m->seq.last = m->d_last;
    if (m->ds_ok) {
        const int G = ds_grid();
        int nt = m->lm.ntiles;
        for (const auto &ly : m->layers) nt = std::max({nt, ly.qkv.ntiles, ly.o.ntiles, ly.gu.ntiles, ly.down.ntiles});
        m->ds_acc_n = nt * DS_TN;
        if ((rc = dalloc_t(m, &m->ds_layers, (size_t)m->L)) != SB_OK) return fail(rc);
        if ((rc = dalloc_t(m, &m->ds_x, (size_t)2 * m->h)) != SB_OK) return fail(rc);
        if ((rc = dalloc_t(m, &m->ds_acc, (size_t)3 * m->ds_acc_n)) != SB_OK) return fail(rc);
        if ((rc = dalloc_t(m, &m->ds_part, ds_part_floats(m->nkv, m->nh / m->nkv, m->hd))) != SB_OK) return fail(rc);
        if ((rc = dalloc_t(m, &m->ds_cand_val, (size_t)G)) != SB_OK) return fail(rc);
        if ((rc = dalloc_t(m, &m->ds_cand_idx, (size_t)G)) != SB_OK) return fail(rc);
        if ((rc = dalloc_t(m, &m->ds_sync, 4)) != SB_OK) return fail(rc);
    }
    if (B > QG_MAX_M) {
        int nt = m->lm.ntiles;
        for (const auto &ly : m->layers) nt = std::max({nt, ly.qkv.ntiles, ly.o.ntiles, ly.gu.ntiles, ly.down.ntiles});
        const int kmax = std::max(std::max(m->h, m->F), m->q_dim);
        m->gws.ld_acc = nt * DS_TN;
        if ((rc = dalloc(m, (void **)&m->gws.planes, qgemm_planes_bytes(kmax, B))) != SB_OK) return fail(rc);
        if ((rc = dalloc_t(m, &m->gws.acc, (size_t)B * m->gws.ld_acc)) != SB_OK) return fail(rc);
        if ((rc = dalloc_t(m, &m->gws.shift, (size_t)B)) != SB_OK) return fail(rc);
        if ((rc = dalloc_t(m, &m->gws.rstd, (size_t)B)) != SB_OK) return fail(rc);
    }
    if ((rc = dalloc_t(m, &m->trace_buf, (size_t)m->L * B * m->h)) != SB_OK) return fail(rc);
    if (tp_size > 1) {
        const size_t nc = (size_t)tp_size * B * m->lm.ntiles;
        if ((rc = dalloc_t(m, &m->cand_all_val, nc)) != SB_OK) return fail(rc);
        if ((rc = dalloc_t(m, &m->cand_all_idx, nc)) != SB_OK) return fail(rc);
        if ((rc = dalloc_t(m, &m->logits_all, (size_t)B * m->V)) != SB_OK) return fail(rc);
    }
    SB_CUDA_TRY(cudaStreamSynchronize(m->st));
    *out = m;
    return SB_OK;
}

}  // namespace

extern "C" {

sb_status sb_llama_create(const sb_llama_config *cfg, sb_llama **out) { return llama_create(cfg, 0, 1, nullptr, out); }

sb_status sb_llama_create_tp(const sb_llama_config *cfg, int tp_rank, int tp_size, const uint8_t *tp_id,
                             sb_llama **out) {
    return llama_create(cfg, tp_rank, tp_size, tp_id, out);
}

sb_status sb_tp_shard_qweight(const sb_llama_config *cfg, int slot, int tp_rank, int tp_size, const int8_t *full,
                              int8_t *shard, int *rows, int *cols) {
    SB_CHECK(cfg, SB_ERR_ARG, "sb_tp_shard_qweight: null config");
    return tp_shard(*cfg, slot, tp_rank, tp_size, full, shard, rows, cols);
}

sb_status sb_tp_probe_timeout(int *timed_out, double *seconds) {
    SB_CHECK(timed_out && seconds, SB_ERR_ARG, "sb_tp_probe_timeout: null argument");
    return tp_probe_timeout(timed_out, seconds);
}

sb_status sb_tp_unique_id(uint8_t *id) {
    SB_CHECK(id, SB_ERR_ARG, "sb_tp_unique_id: null argument");
    return tp_unique_id(id);
}

sb_status sb_llama_destroy(sb_llama *m) {
    if (!m) return SB_OK;
    if (m->st) cudaStreamSynchronize(m->st);
    for (auto g : m->graphs)
        if (g) cudaGraphExecDestroy(g);  // graphs hold NCCL calls: release them before the communicator
    for (auto g : m->sgraphs)
        if (g) cudaGraphExecDestroy(g);
    for (auto g : m->pgraphs)
        if (g) cudaGraphExecDestroy(g);
    tp_destroy(m->comm);
    for (void *p : m->allocs) cudaFree(p);
    if (m->raw) cudaFree(m->raw);
    if (m->err_host) cudaFreeHost(m->err_host);
    if (m->st) cudaStreamDestroy(m->st);
    delete m;
    return SB_OK;
}

sb_status sb_llama_load_f32(sb_llama *m, int which, int layer, const float *data) {
    SB_CHECK(m && data, SB_ERR_ARG, "sb_llama_load_f32: null argument");
    float *dst = nullptr;
    size_t n = m->h;
    switch (which) {
    case SB_F_EMBED: dst = m->embed, n = (size_t)m->V * m->h; break;
    case SB_F_NORM_IN:
        SB_CHECK(layer >= 0 && layer < m->L, SB_ERR_ARG, "bad layer %d", layer);
        dst = m->norm_in + (size_t)layer * m->h;
        break;
    case SB_F_NORM_POST:
        SB_CHECK(layer >= 0 && layer < m->L, SB_ERR_ARG, "bad layer %d", layer);
        dst = m->norm_post + (size_t)layer * m->h;
        break;
    case SB_F_NORM_FINAL: dst = m->norm_final; break;
    default: return set_error(SB_ERR_ARG, "sb_llama_load_f32: unknown tensor %d", which);
    }
    SB_CUDA_TRY(cudaMemcpyAsync(dst, data, sizeof(float) * n, cudaMemcpyHostToDevice, m->st));
    SB_CUDA_TRY(cudaStreamSynchronize(m->st));
    return SB_OK;
}

sb_status sb_llama_load_qweight(sb_llama *m, int layer, int slot, const int8_t *q, float scale) {
    SB_CHECK(m && q, SB_ERR_ARG, "sb_llama_load_qweight: null argument");
    std::vector<int8_t> shard;
    if (m->tp > 1) {  // keep this rank's slice of the full tensor (the scale is the full tensor's)
        SB_CHECK(layer < m->L && (layer < 0 || (slot >= 0 && slot < 5)), SB_ERR_ARG, "bad layer %d / slot %d", layer,
                 slot);
        const int sl = layer < 0 ? SB_W_LM_HEAD : slot;
        int rows = 0, cols = 0;
        SB_TRY(tp_shard(m->cfg, sl, m->tp_rank, m->tp, nullptr, nullptr, &rows, &cols));
        shard.resize((size_t)rows * cols);
        SB_TRY(tp_shard(m->cfg, sl, m->tp_rank, m->tp, q, shard.data(), nullptr, nullptr));
        q = shard.data();
    }
    if (layer < 0) {  // lm_head, [V,h] like llama.rs:943-948
        SB_CUDA_TRY(cudaMemcpyAsync(m->stage, q, (size_t)m->Vl * m->h, cudaMemcpyHostToDevice, m->st));
        SB_TRY(qweight_pack(m->stage, m->h, m->Vl, m->lm.TN, 0, 1, const_cast<uint4 *>(m->lm.w), m->st));
        m->lm.scale = scale;
        m->has_lm = true;
        SB_CUDA_TRY(cudaStreamSynchronize(m->st));
        return SB_OK;
    }
    SB_CHECK(layer < m->L && slot >= 0 && slot < 5, SB_ERR_ARG, "bad layer %d / slot %d", layer, slot);
    sb_llama::Layer &ly = m->layers[layer];
    QWeightDesc *d = nullptr;
    int K = 0, N = 0;
    switch (slot) {
    case SB_W_QKV: d = &ly.qkv, K = m->h, N = m->qkv_dim; break;
    case SB_W_O: d = &ly.o, K = m->q_dim, N = m->h; break;
    case SB_W_DOWN: d = &ly.down, K = m->F, N = m->h; break;
    case SB_W_GATE:
        SB_CUDA_TRY(cudaMemcpyAsync(m->stage, q, (size_t)m->h * m->F, cudaMemcpyHostToDevice, m->st));
        m->staged_gate_layer = layer;
        m->staged_gate_scale = scale;
        ly.has[SB_W_GATE] = true;
        SB_CUDA_TRY(cudaStreamSynchronize(m->st));
        return SB_OK;
    case SB_W_UP:
        SB_CHECK(m->staged_gate_layer == layer, SB_ERR_STATE,
                 "sb_llama_load_qweight: load gate before up for layer %d", layer);
        SB_CUDA_TRY(cudaMemcpyAsync(m->stage + (size_t)m->h * m->F, q, (size_t)m->h * m->F,
                                    cudaMemcpyHostToDevice, m->st));
        SB_TRY(qweight_pack(m->stage, m->h, ly.gu.N, ly.gu.TN, m->F, 0, const_cast<uint4 *>(ly.gu.w), m->st));
        ly.gu.scale = m->staged_gate_scale;
        ly.gu.scale_up = scale;
        ly.has[SB_W_UP] = true;
        m->staged_gate_layer = -1;
        SB_CUDA_TRY(cudaStreamSynchronize(m->st));
        return SB_OK;
    }
    SB_CUDA_TRY(cudaMemcpyAsync(m->stage, q, (size_t)K * N, cudaMemcpyHostToDevice, m->st));
    SB_TRY(qweight_pack(m->stage, K, N, d->TN, 0, 0, const_cast<uint4 *>(d->w), m->st));
    d->scale = scale;
    ly.has[slot] = true;
    SB_CUDA_TRY(cudaStreamSynchronize(m->st));
    return SB_OK;
}

namespace {

size_t dtype_bytes(int dtype) { return dtype == SB_DTYPE_F32 ? 4 : 2; }

// The raw-tensor staging buffer, at least `bytes` (the old one is freed).
int raw_reserve(sb_llama *m, size_t bytes) {
    if (m->raw_bytes >= bytes) return SB_OK;
    SB_CUDA_TRY(cudaStreamSynchronize(m->st));
    if (m->raw) cudaFree(m->raw);
    m->raw = nullptr;
    m->raw_bytes = 0;
    cudaError_t e = cudaMalloc(&m->raw, bytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return set_error(SB_ERR_OOM, "checkpoint staging of %zu bytes: %s", bytes, cudaGetErrorString(e));
    }
    m->raw_bytes = bytes;
    return SB_OK;
}

// Upload the parts (host, dtype, rows x cols each) one after another into
// the raw staging buffer; *dev[i] receives each part's device address.
int raw_upload(sb_llama *m, int dtype, int n_parts, const void *const *parts, const int64_t *rows, int64_t cols,
               const void **dev) {
    const size_t es = dtype_bytes(dtype);
    size_t total = 0;
    for (int i = 0; i < n_parts; i++) total += align_up((size_t)rows[i] * (size_t)cols * es, 256);
    SB_TRY(raw_reserve(m, total));
    size_t off = 0;
    for (int i = 0; i < n_parts; i++) {
        const size_t b = (size_t)rows[i] * (size_t)cols * es;
        char *d = static_cast<char *>(m->raw) + off;
        SB_CUDA_TRY(cudaMemcpyAsync(d, parts[i], b, cudaMemcpyHostToDevice, m->st));
        dev[i] = d;
        off += align_up(b, 256);
    }
    return SB_OK;
}

// quantize_symmetric of the full tensor `full` (its absmax), values of this
// rank's slice `part`, into m->stage + stage_off as [N, K]; the scale to *scale.
int quantize_src(sb_llama *m, const SrcSpec &full, const SrcSpec &part, size_t stage_off, float *scale) {
    SB_TRY(src_absmax(full, m->amax, m->st));
    SB_TRY(src_quantize(part, m->amax, m->stage + stage_off, m->scale_dev, m->st));
    SB_CUDA_TRY(cudaMemcpyAsync(scale, m->scale_dev, 4, cudaMemcpyDeviceToHost, m->st));
    SB_CUDA_TRY(cudaStreamSynchronize(m->st));
    return SB_OK;
}

}  // namespace

sb_status sb_llama_load_hf(sb_llama *m, int layer, int slot, int dtype, int n_parts, const void *const *parts,
                           const int64_t *part_rows, int64_t cols) {
    SB_CHECK(m && parts && part_rows, SB_ERR_ARG, "sb_llama_load_hf: null argument");
    SB_CHECK(dtype == SB_DTYPE_F32 || dtype == SB_DTYPE_BF16 || dtype == SB_DTYPE_F16, SB_ERR_ARG,
             "sb_llama_load_hf: dtype %d", dtype);
    SB_CHECK(layer < m->L && (layer < 0 || (slot >= 0 && slot < 5)), SB_ERR_ARG, "bad layer %d / slot %d", layer,
             slot);
    const int T = m->tp, r = m->tp_rank, h = m->h;
    const int F = m->F, Ff = F * T, q = m->q_dim, kv = m->kv_dim, Qf = q * T, KVf = kv * T, V = m->V, Vl = m->Vl;
    const int want_parts = (layer >= 0 && slot == SB_W_QKV) ? 3 : 1;
    SB_CHECK(n_parts == want_parts, SB_ERR_ARG, "sb_llama_load_hf: %d parts, expected %d", n_parts, want_parts);
    for (int i = 0; i < n_parts; i++) SB_CHECK(parts[i], SB_ERR_ARG, "sb_llama_load_hf: null part %d", i);
    // expected HF shapes [out, in] of the FULL tensors
    int64_t er[3] = {0, 0, 0}, ec = 0;
    if (layer < 0) er[0] = V, ec = h;
    else if (slot == SB_W_QKV) er[0] = Qf, er[1] = KVf, er[2] = KVf, ec = h;
    else if (slot == SB_W_O) er[0] = h, ec = Qf;
    else if (slot == SB_W_DOWN) er[0] = h, ec = Ff;
    else er[0] = Ff, ec = h;  // gate, up
    for (int i = 0; i < n_parts; i++)
        SB_CHECK(part_rows[i] == er[i] && cols == ec, SB_ERR_SHAPE,
                 "sb_llama_load_hf: part %d is [%lld, %lld], expected [%lld, %lld]", i, (long long)part_rows[i],
                 (long long)cols, (long long)er[i], (long long)ec);
    const void *dev[3] = {nullptr, nullptr, nullptr};
    SB_TRY(raw_upload(m, dtype, n_parts, parts, part_rows, cols, dev));
    SrcSpec full, part;
    full.dtype = dtype;
    for (int i = 0; i < n_parts; i++) full.p[i] = dev[i], full.ld[i] = cols;
    full.nseg = n_parts;
    if (layer < 0) {  // lm_head [V,h] (llama.rs:943-948): K = h, N = this rank's vocabulary rows
        full.K = h, full.N = V;
        part = full;
        part.N = Vl, part.row0[0] = (long long)r * Vl;
        float sc = 0.f;
        SB_TRY(quantize_src(m, full, part, 0, &sc));
        SB_TRY(qweight_pack(m->stage, h, Vl, m->lm.TN, 0, 1, const_cast<uint4 *>(m->lm.w), m->st));
        m->lm.scale = sc;
        m->has_lm = true;
        SB_CUDA_TRY(cudaStreamSynchronize(m->st));
        return SB_OK;
    }
    sb_llama::Layer &ly = m->layers[layer];
    switch (slot) {
    case SB_W_QKV:  // fuse_qkv_weights (llama.rs:1009-1029): q | k | v columns, one scale
        full.K = h, full.N = Qf + 2 * KVf;
        full.c0[1] = Qf, full.c0[2] = Qf + KVf;
        part = full;
        part.N = q + 2 * kv;
        part.c0[1] = q, part.c0[2] = q + kv;
        part.row0[0] = (long long)r * q, part.row0[1] = (long long)r * kv, part.row0[2] = (long long)r * kv;
        SB_TRY(quantize_src(m, full, part, 0, &ly.qkv.scale));
        SB_TRY(qweight_pack(m->stage, h, ly.qkv.N, ly.qkv.TN, 0, 1, const_cast<uint4 *>(ly.qkv.w), m->st));
        break;
    case SB_W_O:  // rows (in) of this rank's heads
        full.K = Qf, full.N = h;
        part = full;
        part.K = q, part.k0 = (long long)r * q;
        SB_TRY(quantize_src(m, full, part, 0, &ly.o.scale));
        SB_TRY(qweight_pack(m->stage, q, h, ly.o.TN, 0, 1, const_cast<uint4 *>(ly.o.w), m->st));
        break;
    case SB_W_DOWN:  // rows (in) of this rank's ffn features
        full.K = Ff, full.N = h;
        part = full;
        part.K = F, part.k0 = (long long)r * F;
        SB_TRY(quantize_src(m, full, part, 0, &ly.down.scale));
        SB_TRY(qweight_pack(m->stage, F, h, ly.down.TN, 0, 1, const_cast<uint4 *>(ly.down.w), m->st));
        break;
    case SB_W_GATE:
    case SB_W_UP: {  // this rank's ffn columns; gate and up are packed together once both are staged
        full.K = h, full.N = Ff;
        part = full;
        part.N = F, part.row0[0] = (long long)r * F;
        if (slot == SB_W_GATE) {
            SB_TRY(quantize_src(m, full, part, 0, &m->staged_gate_scale));
            m->staged_gate_layer = layer;
            ly.has[SB_W_GATE] = true;
            return SB_OK;
        }
        SB_CHECK(m->staged_gate_layer == layer, SB_ERR_STATE, "sb_llama_load_hf: load gate before up for layer %d",
                 layer);
        float su = 0.f;
        SB_TRY(quantize_src(m, full, part, (size_t)h * F, &su));
        SB_TRY(qweight_pack(m->stage, h, ly.gu.N, ly.gu.TN, F, 1, const_cast<uint4 *>(ly.gu.w), m->st));
        ly.gu.scale = m->staged_gate_scale;
        ly.gu.scale_up = su;
        m->staged_gate_layer = -1;
        break;
    }
    }
    ly.has[slot] = true;
    SB_CUDA_TRY(cudaStreamSynchronize(m->st));
    return SB_OK;
}

sb_status sb_llama_load_hf_f32(sb_llama *m, int which, int layer, int dtype, const void *data, int64_t n) {
    SB_CHECK(m && data, SB_ERR_ARG, "sb_llama_load_hf_f32: null argument");
    SB_CHECK(dtype == SB_DTYPE_F32 || dtype == SB_DTYPE_BF16 || dtype == SB_DTYPE_F16, SB_ERR_ARG,
             "sb_llama_load_hf_f32: dtype %d", dtype);
    float *dst = nullptr;
    int64_t want = m->h;
    switch (which) {
    case SB_F_EMBED: dst = m->embed, want = (int64_t)m->V * m->h; break;
    case SB_F_NORM_IN:
    case SB_F_NORM_POST:
        SB_CHECK(layer >= 0 && layer < m->L, SB_ERR_ARG, "sb_llama_load_hf_f32: layer %d", layer);
        dst = (which == SB_F_NORM_IN ? m->norm_in : m->norm_post) + (size_t)layer * m->h;
        break;
    case SB_F_NORM_FINAL: dst = m->norm_final; break;
    default: return set_error(SB_ERR_ARG, "sb_llama_load_hf_f32: tensor kind %d", which);
    }
    SB_CHECK(n == want, SB_ERR_SHAPE, "sb_llama_load_hf_f32: %lld values, expected %lld", (long long)n,
             (long long)want);
    const void *dev = nullptr;
    const int64_t rows = n;
    SB_TRY(raw_upload(m, dtype, 1, &data, &rows, 1, &dev));
    SB_TRY(src_to_f32(dev, dtype, (size_t)n, dst, m->st));
    SB_CUDA_TRY(cudaStreamSynchronize(m->st));
    return SB_OK;
}

sb_status sb_llama_get_qweight(sb_llama *m, int layer, int slot, int8_t *q, float *scale) {
    SB_CHECK(m && q && scale, SB_ERR_ARG, "sb_llama_get_qweight: null argument");
    if (layer < 0) {
        SB_TRY(qweight_unpack(m->lm.w, m->h, m->Vl, m->lm.TN, 0, m->stage, m->st));
        std::vector<int8_t> hv((size_t)m->h * m->Vl);
        SB_CUDA_TRY(cudaMemcpyAsync(hv.data(), m->stage, hv.size(), cudaMemcpyDeviceToHost, m->st));
        SB_CUDA_TRY(cudaStreamSynchronize(m->st));
        for (int k = 0; k < m->h; k++)
            for (int n = 0; n < m->Vl; n++) q[(size_t)n * m->h + k] = hv[(size_t)k * m->Vl + n];
        *scale = m->lm.scale;
        return SB_OK;
    }
    SB_CHECK(layer < m->L && slot >= 0 && slot < 5, SB_ERR_ARG, "bad layer %d / slot %d", layer, slot);
    const sb_llama::Layer &ly = m->layers[layer];
    const size_t kf = (size_t)m->h * m->F;
    switch (slot) {
    case SB_W_QKV:
        SB_TRY(qweight_unpack(ly.qkv.w, ly.qkv.K, ly.qkv.N, ly.qkv.TN, 0, m->stage, m->st));
        *scale = ly.qkv.scale;
        SB_CUDA_TRY(cudaMemcpyAsync(q, m->stage, (size_t)ly.qkv.K * ly.qkv.N, cudaMemcpyDeviceToHost, m->st));
        break;
    case SB_W_O:
        SB_TRY(qweight_unpack(ly.o.w, ly.o.K, ly.o.N, ly.o.TN, 0, m->stage, m->st));
        *scale = ly.o.scale;
        SB_CUDA_TRY(cudaMemcpyAsync(q, m->stage, (size_t)ly.o.K * ly.o.N, cudaMemcpyDeviceToHost, m->st));
        break;
    case SB_W_DOWN:
        SB_TRY(qweight_unpack(ly.down.w, ly.down.K, ly.down.N, ly.down.TN, 0, m->stage, m->st));
        *scale = ly.down.scale;
        SB_CUDA_TRY(cudaMemcpyAsync(q, m->stage, (size_t)ly.down.K * ly.down.N, cudaMemcpyDeviceToHost, m->st));
        break;
    default:  // gate / up
        SB_TRY(qweight_unpack(ly.gu.w, ly.gu.K, ly.gu.N, ly.gu.TN, m->F, m->stage, m->st));
        *scale = slot == SB_W_GATE ? ly.gu.scale : ly.gu.scale_up;
        SB_CUDA_TRY(cudaMemcpyAsync(q, m->stage + (slot == SB_W_GATE ? 0 : kf), kf, cudaMemcpyDeviceToHost, m->st));
        break;
    }
    SB_CUDA_TRY(cudaStreamSynchronize(m->st));
    return SB_OK;
}

sb_status sb_llama_init_random(sb_llama *m, uint64_t seed) {
    // LlamaModel::new (llama.rs:593-680) draw order: embed [V*h]; per layer
    // q, k, v, o, gate, up, down; lm_head [V*h] when untied.  Under tensor
    // parallelism every rank walks the same full stream: the scale comes from
    // the full tensor's absmax (spec `full`), the quantized values only for
    // this rank's slice (spec `part`, same sample indices).
    SB_CHECK(m, SB_ERR_ARG, "sb_llama_init_random: null model");
    const int h = m->h, V = m->V, T = m->tp, r = m->tp_rank;
    const int F = m->F, Ff = F * T;                       // local / full ffn
    const int q = m->q_dim, kv = m->kv_dim, Qf = q * T, KVf = kv * T;
    const int Vl = m->Vl;
    uint64_t sample = 0;
    SB_TRY(gen_normal_f32(seed, sample, (size_t)V * h, m->embed, m->st));
    sample += (uint64_t)V * h;
    auto quant = [&](const GenSpec &full, const GenSpec &part, int8_t *dst_stage, float *sc) -> int {
        SB_TRY(gen_absmax(full, seed, m->amax, m->st));
        SB_TRY(gen_quantize(part, seed, m->amax, dst_stage, m->scale_dev, m->st));
        SB_CUDA_TRY(cudaMemcpyAsync(sc, m->scale_dev, 4, cudaMemcpyDeviceToHost, m->st));
        SB_CUDA_TRY(cudaStreamSynchronize(m->st));
        return SB_OK;
    };
    // [K, N] matrix of the stream at `base` (row stride N): rows [r0, r0+k), cols [c0, c0+n)
    auto block = [&](uint64_t base, int N, int r0, int k, int c0, int n) {
        GenSpec g;
        g.K = k;
        g.N = n;
        g.width[0] = N;
        g.base[0] = base + (uint64_t)r0 * N + c0;
        return g;
    };
    for (int l = 0; l < m->L; l++) {
        sb_llama::Layer &ly = m->layers[l];
        const uint64_t bq = sample, bk = bq + (uint64_t)h * Qf, bv = bk + (uint64_t)h * KVf;
        GenSpec full;
        full.K = h;
        full.N = Qf + 2 * KVf;
        full.nseg = 3;
        full.c0[0] = 0, full.c0[1] = Qf, full.c0[2] = Qf + KVf;
        full.width[0] = Qf, full.width[1] = KVf, full.width[2] = KVf;
        full.base[0] = bq, full.base[1] = bk, full.base[2] = bv;
        GenSpec part = full;
        part.N = q + 2 * kv;
        part.c0[1] = q, part.c0[2] = q + kv;
        part.base[0] = bq + (uint64_t)r * q, part.base[1] = bk + (uint64_t)r * kv, part.base[2] = bv + (uint64_t)r * kv;
        sample = bv + (uint64_t)h * KVf;
        SB_TRY(quant(full, part, m->stage, &ly.qkv.scale));
        SB_TRY(qweight_pack(m->stage, h, ly.qkv.N, ly.qkv.TN, 0, 0, const_cast<uint4 *>(ly.qkv.w), m->st));
        SB_TRY(quant(block(sample, h, 0, Qf, 0, h), block(sample, h, r * q, q, 0, h), m->stage, &ly.o.scale));
        SB_TRY(qweight_pack(m->stage, q, h, ly.o.TN, 0, 0, const_cast<uint4 *>(ly.o.w), m->st));
        sample += (uint64_t)Qf * h;
        float sg = 0.0f, su = 0.0f;
        SB_TRY(quant(block(sample, Ff, 0, h, 0, Ff), block(sample, Ff, 0, h, r * F, F), m->stage, &sg));
        sample += (uint64_t)h * Ff;
        SB_TRY(quant(block(sample, Ff, 0, h, 0, Ff), block(sample, Ff, 0, h, r * F, F), m->stage + (size_t)h * F,
                     &su));
        sample += (uint64_t)h * Ff;
        SB_TRY(qweight_pack(m->stage, h, ly.gu.N, ly.gu.TN, F, 0, const_cast<uint4 *>(ly.gu.w), m->st));
        ly.gu.scale = sg;
        ly.gu.scale_up = su;
        SB_TRY(quant(block(sample, h, 0, Ff, 0, h), block(sample, h, r * F, F, 0, h), m->stage, &ly.down.scale));
        SB_TRY(qweight_pack(m->stage, F, h, ly.down.TN, 0, 0, const_cast<uint4 *>(ly.down.w), m->st));
        sample += (uint64_t)Ff * h;
        for (int s = 0; s < 5; s++) ly.has[s] = true;
    }
    // lm_head: target [h, V] from the [V,h] stream order (transposed)
    GenSpec gl;
    gl.K = h;
    gl.N = V;
    gl.transposed = 1;
    if (m->cfg.tie_word_embeddings) {
        gl.src = m->embed;
    } else {
        gl.base[0] = sample;
        sample += (uint64_t)V * h;
    }
    GenSpec gp = gl;
    gp.N = Vl;
    if (gl.src)
        gp.src = m->embed + (size_t)r * Vl * h;
    else
        gp.base[0] = gl.base[0] + (uint64_t)r * Vl * h;
    float scale = 0.0f;
    SB_TRY(quant(gl, gp, m->stage, &scale));
    // gen_quantize wrote [h,Vl] row-major (K x N) into stage: pack as untransposed.
    SB_TRY(qweight_pack(m->stage, h, Vl, m->lm.TN, 0, 0, const_cast<uint4 *>(m->lm.w), m->st));
    m->lm.scale = scale;
    m->has_lm = true;
    SB_CUDA_TRY(cudaStreamSynchronize(m->st));
    return SB_OK;
}

sb_status sb_llama_reset(sb_llama *m) {
    SB_CHECK(m, SB_ERR_ARG, "sb_llama_reset: null model");
    SB_CUDA_TRY(cudaMemsetAsync(m->d_pos, 0, sizeof(int) * m->B, m->st));
    SB_CUDA_TRY(cudaMemsetAsync(m->d_ngen, 0, sizeof(int) * m->B, m->st));
    SB_CUDA_TRY(cudaStreamSynchronize(m->st));
    return SB_OK;
}

sb_status sb_llama_set_trace(sb_llama *m, int enabled) {
    SB_CHECK(m, SB_ERR_ARG, "null model");
    m->trace = enabled != 0;
    return SB_OK;
}

sb_status sb_llama_get_trace(sb_llama *m, float *out) {
    SB_CHECK(m && out, SB_ERR_ARG, "null argument");
    SB_CHECK(m->trace_batch > 0, SB_ERR_STATE, "no traced step yet");
    SB_CUDA_TRY(cudaMemcpy(out, m->trace_buf, sizeof(float) * (size_t)m->L * m->trace_batch * m->h,
                           cudaMemcpyDeviceToHost));
    return SB_OK;
}

sb_status sb_llama_forward(sb_llama *m, int batch, const int32_t *tokens, const int32_t *pos, float *logits,
                           int32_t *argmax) {
    SB_CHECK(m && tokens && pos, SB_ERR_ARG, "sb_llama_forward: null argument");
    SB_CHECK(batch >= 1 && batch <= m->B, SB_ERR_SHAPE, "batch %d outside 1..%d", batch, m->B);
    for (int b = 0; b < batch; b++) {
        SB_CHECK(pos[b] >= 0 && pos[b] < m->cfg.max_seq_len, SB_ERR_SHAPE, "position %d beyond cache %d", pos[b],
                 m->cfg.max_seq_len);
        SB_CHECK(tokens[b] >= 0 && tokens[b] < m->V, SB_ERR_ARG, "token %d outside vocab %d", tokens[b], m->V);
    }
    SB_TRY(check_ready(m));
    std::vector<int32_t> zero(batch, 0);
    if (batch == 1 && m->ds_ok) {
        // token and position go to the kernel as launch arguments: no copies
        SB_TRY(ds_step(m, false, tokens[0], pos[0]));
        if (m->trace) m->trace_batch = 1;
    } else if (m->trace) {
        SB_TRY(set_state(m, batch, tokens, pos, zero.data()));
        SB_TRY(enqueue_step(m, batch, m->st, false, true));
        m->trace_batch = batch;
    } else {
        cudaGraphExec_t g = nullptr;
        SB_TRY(get_graph(m, batch, &g));
        // get_graph may have run a warm-up step: restore the inputs.
        SB_TRY(set_state(m, batch, tokens, pos, zero.data()));
        SB_CUDA_TRY(cudaGraphLaunch(g, m->st));
    }
    m->active = 0;
    if (logits && m->tp == 1)
        SB_CUDA_TRY(cudaMemcpyAsync(logits, m->logits, sizeof(float) * (size_t)batch * m->V, cudaMemcpyDeviceToHost,
                                    m->st));
    std::vector<float> lg_all;
    if (logits && m->tp > 1) {
        // every rank's vocabulary slice: [rank][row][Vl] -> host [row][V]
        SB_TRY(tp_allgather32(m->comm, m->logits, m->logits_all, (size_t)batch * m->Vl, m->st));
        lg_all.resize((size_t)batch * m->V);
        SB_CUDA_TRY(cudaMemcpyAsync(lg_all.data(), m->logits_all, sizeof(float) * lg_all.size(), cudaMemcpyDeviceToHost,
                                    m->st));
    }
    if (argmax) SB_CUDA_TRY(cudaMemcpyAsync(argmax, m->d_last, sizeof(int) * batch, cudaMemcpyDeviceToHost, m->st));
    SB_TRY(queue_error_peeks(m, batch == 1 && m->ds_ok));
    SB_CUDA_TRY(cudaStreamSynchronize(m->st));
    if (!lg_all.empty())
        for (int t = 0; t < m->tp; t++)
            for (int b = 0; b < batch; b++)
                std::memcpy(logits + (size_t)b * m->V + (size_t)t * m->Vl,
                            lg_all.data() + ((size_t)t * batch + b) * m->Vl, sizeof(float) * m->Vl);
    const unsigned *h = m->err_host;
    if (h[0] | h[1] | h[2] | h[3] | h[4]) return check_device_errors(m);  // reports and clears
    return SB_OK;
}

namespace {
// Scratch of the device sampler: [B][V] probabilities, [B] generator states, [B] tokens.
int samp_buffers(sb_llama *m) {
    if (m->samp_prob) return SB_OK;
    void *a = nullptr, *b = nullptr, *c = nullptr;
    cudaError_t e = cudaMalloc(&a, sizeof(double) * (size_t)m->B * m->V);
    if (e == cudaSuccess) m->allocs.push_back(a), e = cudaMalloc(&b, sizeof(uint64_t) * m->B);
    if (e == cudaSuccess) m->allocs.push_back(b), e = cudaMalloc(&c, sizeof(int) * m->B);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return set_error(SB_ERR_OOM, "device sampler scratch: %s", cudaGetErrorString(e));
    }
    m->allocs.push_back(c);
    m->samp_prob = static_cast<double *>(a);
    m->d_rng = static_cast<uint64_t *>(b);
    m->d_samp = static_cast<int *>(c);
    return SB_OK;
}
}  // namespace

sb_status sb_llama_set_sampling(sb_llama *m, int batch, float temperature, int top_k, float top_p, int max_draws,
                                const uint64_t *rng_state) {
    SB_CHECK(m && rng_state, SB_ERR_ARG, "sb_llama_set_sampling: null argument");
    SB_CHECK(batch >= 1 && batch <= m->B, SB_ERR_SHAPE, "batch %d outside 1..%d", batch, m->B);
    SB_CHECK(m->tp == 1, SB_ERR_UNSUPPORTED,
             "sb_llama_set_sampling: a tensor-parallel rank holds a vocabulary slice; sample on the host");
    SB_CHECK(!std::isnan(temperature) && !std::isnan(top_p) && top_k >= 0 && max_draws >= 1, SB_ERR_ARG,
             "sb_llama_set_sampling: temperature %g, top_k %d, top_p %g, max_draws %d", (double)temperature, top_k,
             (double)top_p, max_draws);
    SB_TRY(samp_buffers(m));
    SampleCfg c;
    c.temperature = temperature;
    c.top_k = top_k;
    c.top_p = top_p;
    c.max_draws = max_draws;
    if (c.temperature != m->samp.temperature || c.top_k != m->samp.top_k || c.top_p != m->samp.top_p ||
        c.max_draws != m->samp.max_draws) {
        // the sampled graphs hold the parameters: capture them again
        SB_CUDA_TRY(cudaStreamSynchronize(m->st));
        for (auto &g : m->sgraphs)
            if (g) cudaGraphExecDestroy(g), g = nullptr;
        m->samp = c;
    }
    SB_CUDA_TRY(cudaMemcpyAsync(m->d_rng, rng_state, sizeof(uint64_t) * batch, cudaMemcpyHostToDevice, m->st));
    SB_CUDA_TRY(cudaStreamSynchronize(m->st));
    m->samp_on = true;
    return SB_OK;
}

sb_status sb_llama_clear_sampling(sb_llama *m) {
    SB_CHECK(m, SB_ERR_ARG, "sb_llama_clear_sampling: null model");
    m->samp_on = false;
    return SB_OK;
}

sb_status sb_llama_get_rng(sb_llama *m, int batch, uint64_t *rng_state) {
    SB_CHECK(m && rng_state, SB_ERR_ARG, "sb_llama_get_rng: null argument");
    SB_CHECK(batch >= 1 && batch <= m->B, SB_ERR_SHAPE, "batch %d outside 1..%d", batch, m->B);
    SB_CHECK(m->d_rng, SB_ERR_STATE, "sb_llama_get_rng: the device sampler has not run");
    SB_CUDA_TRY(cudaStreamSynchronize(m->st));
    SB_TRY(check_device_errors(m));
    SB_CUDA_TRY(cudaMemcpy(rng_state, m->d_rng, sizeof(uint64_t) * batch, cudaMemcpyDeviceToHost));
    return SB_OK;
}

sb_status sb_llama_sample(sb_llama *m, int batch, float temperature, int top_k, float top_p, uint64_t *rng_state,
                          int32_t *tokens) {
    SB_CHECK(m && rng_state && tokens, SB_ERR_ARG, "sb_llama_sample: null argument");
    SB_CHECK(batch >= 1 && batch <= m->B, SB_ERR_SHAPE, "batch %d outside 1..%d", batch, m->B);
    SB_CHECK(m->tp == 1, SB_ERR_UNSUPPORTED,
             "sb_llama_sample: a tensor-parallel rank holds a vocabulary slice; gather the logits with "
             "sb_llama_forward and sample on the host");
    SB_CHECK(!std::isnan(temperature) && !std::isnan(top_p) && top_k >= 0, SB_ERR_ARG,
             "sb_llama_sample: temperature %g, top_k %d, top_p %g", (double)temperature, top_k, (double)top_p);
    SB_TRY(samp_buffers(m));
    SB_CUDA_TRY(cudaMemcpyAsync(m->d_rng, rng_state, sizeof(uint64_t) * batch, cudaMemcpyHostToDevice, m->st));
    SB_TRY(sample_rows_launch(m->logits, batch, m->V, m->Vl, temperature, top_k, top_p, m->d_rng, m->samp_prob,
                              m->d_samp, m->st));
    SB_CUDA_TRY(cudaMemcpyAsync(tokens, m->d_samp, sizeof(int) * batch, cudaMemcpyDeviceToHost, m->st));
    SB_CUDA_TRY(cudaMemcpyAsync(rng_state, m->d_rng, sizeof(uint64_t) * batch, cudaMemcpyDeviceToHost, m->st));
    SB_CUDA_TRY(cudaStreamSynchronize(m->st));
    return SB_OK;
}

sb_status sb_llama_begin(sb_llama *m, int batch, const int32_t *prompts, int n_prompt) {
    SB_CHECK(m && prompts, SB_ERR_ARG, "sb_llama_begin: null argument");
    SB_CHECK(batch >= 1 && batch <= m->B, SB_ERR_SHAPE, "batch %d outside 1..%d", batch, m->B);
    SB_CHECK(n_prompt >= 1 && n_prompt <= m->cfg.max_seq_len, SB_ERR_SHAPE, "prompt length %d", n_prompt);
    for (size_t i = 0; i < (size_t)batch * n_prompt; i++)
        SB_CHECK(prompts[i] >= 0 && prompts[i] < m->V, SB_ERR_ARG, "prompt token %d outside vocab", prompts[i]);
    SB_TRY(check_ready(m));
    if (!(batch == 1 && m->ds_ok)) {
        cudaGraphExec_t g = nullptr;
        SB_TRY(get_graph(m, batch, &g, m->samp_on ? STEP_SAMPLED : STEP_GREEDY));
    }
    for (int b = 0; b < batch; b++)
        SB_CUDA_TRY(cudaMemcpyAsync(m->d_prompt + (size_t)b * m->cfg.max_seq_len, prompts + (size_t)b * n_prompt,
                                    sizeof(int) * n_prompt, cudaMemcpyHostToDevice, m->st));
    std::vector<int32_t> tok(batch, 0), pos(batch, 0), plen(batch, n_prompt);
    SB_TRY(set_state(m, batch, tok.data(), pos.data(), plen.data()));
    SB_CUDA_TRY(cudaStreamSynchronize(m->st));
    m->active = batch;
    m->steps = 0;
    return SB_OK;
}

sb_status sb_llama_prefill(sb_llama *m, int batch, const int32_t *prompts, int n_prompt) {
    SB_CHECK(m && prompts, SB_ERR_ARG, "sb_llama_prefill: null argument");
    SB_CHECK(batch >= 1 && batch <= m->B, SB_ERR_SHAPE, "batch %d outside 1..%d", batch, m->B);
    SB_CHECK(n_prompt >= 1 && n_prompt < m->cfg.max_seq_len, SB_ERR_SHAPE, "prompt length %d", n_prompt);
    for (size_t i = 0; i < (size_t)batch * n_prompt; i++)
        SB_CHECK(prompts[i] >= 0 && prompts[i] < m->V, SB_ERR_ARG, "prompt token %d outside vocab", prompts[i]);
    SB_TRY(check_ready(m));
    const int C = m->B;  // prompt positions per batched step
    const int tail = n_prompt % C;
    // Capture every step shape used here and by the decode steps that follow
    // before any state is set: a capture's warm-up step resets the sequence state.
    cudaGraphExec_t g_full = nullptr, g_tail = nullptr, g_dec = nullptr;
    if (!(batch == 1 && m->ds_ok)) SB_TRY(get_graph(m, batch, &g_dec, m->samp_on ? STEP_SAMPLED : STEP_GREEDY));
    if (n_prompt >= C && !(C == 1 && m->ds_ok)) SB_TRY(get_graph(m, C, &g_full, STEP_PREFILL));
    if (tail > 0 && !(tail == 1 && m->ds_ok)) SB_TRY(get_graph(m, tail, &g_tail, STEP_PREFILL));
    std::vector<int> pt((size_t)m->B * m->pps);
    std::vector<int32_t> tok(C), pos(C), zero(C, 0), first(batch);
    for (int b = 0; b < batch; b++) {
        // every row is a position of sequence b: all rows use its pages
        for (int r = 0; r < m->B; r++)
            for (int i = 0; i < m->pps; i++) pt[(size_t)r * m->pps + i] = b * m->pps + i;
        SB_CUDA_TRY(cudaMemcpyAsync(m->page_table, pt.data(), sizeof(int) * pt.size(), cudaMemcpyHostToDevice, m->st));
        int M = 0;
        for (int p0 = 0; p0 < n_prompt; p0 += C) {
            M = std::min(C, n_prompt - p0);
            for (int r = 0; r < M; r++) tok[r] = prompts[(size_t)b * n_prompt + p0 + r], pos[r] = p0 + r;
            SB_TRY(set_state(m, M, tok.data(), pos.data(), zero.data()));
            if (M == 1 && m->ds_ok)
                SB_TRY(ds_step(m));
            else
                SB_CUDA_TRY(cudaGraphLaunch(M == C ? g_full : g_tail, m->st));
        }
        // the token after the last prompt position is the first generated
        // token: the argmax, or with device sampling a draw from sequence b's
        // generator on that position's logits (generate.rs:72-75)
        if (m->samp_on) {
            SB_TRY(sample_rows_launch(m->logits + (size_t)(M - 1) * m->Vl, 1, m->V, m->Vl, m->samp.temperature,
                                      m->samp.top_k, m->samp.top_p, m->d_rng + b, m->samp_prob, m->d_samp + b, m->st));
            SB_CUDA_TRY(cudaMemcpyAsync(&first[b], m->d_samp + b, sizeof(int), cudaMemcpyDeviceToHost, m->st));
        } else {
            SB_CUDA_TRY(cudaMemcpyAsync(&first[b], m->d_last + (M - 1), sizeof(int), cudaMemcpyDeviceToHost, m->st));
        }
    }
    // sequences back on their own pages, positioned after the prompt
    for (int r = 0; r < m->B; r++)
        for (int i = 0; i < m->pps; i++) pt[(size_t)r * m->pps + i] = r * m->pps + i;
    SB_CUDA_TRY(cudaMemcpyAsync(m->page_table, pt.data(), sizeof(int) * pt.size(), cudaMemcpyHostToDevice, m->st));
    SB_CUDA_TRY(cudaStreamSynchronize(m->st));
    SB_TRY(check_device_errors(m));
    std::vector<int32_t> p1(batch, n_prompt), z(batch, 0), one(batch, 1);
    SB_TRY(set_state(m, batch, first.data(), p1.data(), z.data()));
    for (int b = 0; b < batch; b++)
        SB_CUDA_TRY(cudaMemcpyAsync(m->d_out + (size_t)b * m->cfg.max_seq_len, &first[b], sizeof(int),
                                    cudaMemcpyHostToDevice, m->st));
    SB_CUDA_TRY(cudaMemcpyAsync(m->d_ngen, one.data(), sizeof(int) * batch, cudaMemcpyHostToDevice, m->st));
    SB_CUDA_TRY(cudaStreamSynchronize(m->st));
    m->active = batch;
    m->steps = n_prompt;
    return SB_OK;
}

sb_status sb_llama_forward_seq(sb_llama *m, const int32_t *tokens, int n, float *logits) {
    SB_CHECK(m && tokens && logits, SB_ERR_ARG, "sb_llama_forward_seq: null argument");
    SB_CHECK(n >= 1 && n <= m->cfg.max_seq_len, SB_ERR_SHAPE, "sb_llama_forward_seq: %d tokens, cache of %d", n,
             m->cfg.max_seq_len);
    for (int i = 0; i < n; i++)
        SB_CHECK(tokens[i] >= 0 && tokens[i] < m->V, SB_ERR_ARG, "token %d outside vocab %d", tokens[i], m->V);
    SB_TRY(check_ready(m));
    const int C = m->B;  // positions per batched step
    const int tail = n % C;
    // capture the chunk shapes first (a capture's warm-up resets the state)
    cudaGraphExec_t g_full = nullptr, g_tail = nullptr;
    if (n >= C && !(C == 1 && m->ds_ok)) SB_TRY(get_graph(m, C, &g_full, STEP_PREFILL));
    if (tail > 0 && !(tail == 1 && m->ds_ok)) SB_TRY(get_graph(m, tail, &g_tail, STEP_PREFILL));
    // every row of a chunk is a position of sequence 0: all rows use its pages
    std::vector<int> pt((size_t)m->B * m->pps);
    for (int r = 0; r < m->B; r++)
        for (int i = 0; i < m->pps; i++) pt[(size_t)r * m->pps + i] = i;
    SB_CUDA_TRY(cudaMemcpyAsync(m->page_table, pt.data(), sizeof(int) * pt.size(), cudaMemcpyHostToDevice, m->st));
    std::vector<int32_t> tok(C), pos(C), zero(C, 0);
    std::vector<float> gathered;
    int rc = SB_OK;
    for (int p0 = 0; p0 < n && rc == SB_OK; p0 += C) {
        const int M = std::min(C, n - p0);
        for (int r = 0; r < M; r++) tok[r] = tokens[p0 + r], pos[r] = p0 + r;
        rc = set_state(m, M, tok.data(), pos.data(), zero.data());
        if (rc != SB_OK) break;
        if (M == 1 && m->ds_ok) {
            rc = ds_step(m);
        } else if (cudaGraphLaunch(M == C ? g_full : g_tail, m->st) != cudaSuccess) {
            rc = set_error(SB_ERR_CUDA, "sb_llama_forward_seq: graph launch failed");
        }
        if (rc != SB_OK) break;
        if (m->tp == 1) {
            if (cudaMemcpyAsync(logits + (size_t)p0 * m->V, m->logits, sizeof(float) * (size_t)M * m->V,
                                cudaMemcpyDeviceToHost, m->st) != cudaSuccess)
                rc = set_error(SB_ERR_CUDA, "sb_llama_forward_seq: logits copy failed");
        } else {
            // every rank's vocabulary slice: [rank][row][Vl] -> host [row][V]
            rc = tp_allgather32(m->comm, m->logits, m->logits_all, (size_t)M * m->Vl, m->st);
            gathered.resize((size_t)M * m->V);
            if (rc == SB_OK && cudaMemcpyAsync(gathered.data(), m->logits_all, sizeof(float) * gathered.size(),
                                               cudaMemcpyDeviceToHost, m->st) != cudaSuccess)
                rc = set_error(SB_ERR_CUDA, "sb_llama_forward_seq: logits copy failed");
            if (rc == SB_OK && cudaStreamSynchronize(m->st) != cudaSuccess)
                rc = set_error(SB_ERR_CUDA, "sb_llama_forward_seq: synchronize failed");
            for (int t = 0; t < m->tp && rc == SB_OK; t++)
                for (int b = 0; b < M; b++)
                    std::memcpy(logits + (size_t)(p0 + b) * m->V + (size_t)t * m->Vl,
                                gathered.data() + ((size_t)t * M + b) * m->Vl, sizeof(float) * m->Vl);
        }
    }
    // sequences back on their own pages
    for (int r = 0; r < m->B; r++)
        for (int i = 0; i < m->pps; i++) pt[(size_t)r * m->pps + i] = r * m->pps + i;
    SB_CUDA_TRY(cudaMemcpyAsync(m->page_table, pt.data(), sizeof(int) * pt.size(), cudaMemcpyHostToDevice, m->st));
    SB_CUDA_TRY(cudaStreamSynchronize(m->st));
    SB_TRY(rc);
    m->active = 0;
    return check_device_errors(m);
}

sb_status sb_llama_step(sb_llama *m, int n_steps) {
    SB_CHECK(m && m->active > 0, SB_ERR_STATE, "sb_llama_step: call sb_llama_begin first");
    cudaGraphExec_t g = nullptr;
    SB_CHECK(n_steps >= 0 && (long long)m->steps + n_steps <= m->cfg.max_seq_len, SB_ERR_SHAPE,
             "sb_llama_step: %d + %d steps exceed the cache (%d positions)", m->steps, n_steps, m->cfg.max_seq_len);
    if (m->active == 1 && m->ds_ok) {
        for (int i = 0; i < n_steps; i++) SB_TRY(ds_step(m, m->samp_on));
    } else {
        SB_TRY(get_graph(m, m->active, &g, m->samp_on ? STEP_SAMPLED : STEP_GREEDY));
        for (int i = 0; i < n_steps; i++) SB_CUDA_TRY(cudaGraphLaunch(g, m->st));
    }
    m->steps += n_steps;
    return SB_OK;
}

sb_status sb_llama_tokens(sb_llama *m, int32_t *out, int max_tokens, int *n_out) {
    SB_CHECK(m && out && n_out && m->active > 0, SB_ERR_STATE, "sb_llama_tokens: no active batch");
    SB_CUDA_TRY(cudaStreamSynchronize(m->st));
    SB_TRY(check_device_errors(m));
    std::vector<int> ngen(m->active);
    SB_CUDA_TRY(cudaMemcpy(ngen.data(), m->d_ngen, sizeof(int) * m->active, cudaMemcpyDeviceToHost));
    int n = max_tokens;
    for (int b = 0; b < m->active; b++) n = std::min(n, ngen[b]);
    n = std::max(n, 0);
    for (int b = 0; b < m->active; b++)
        SB_CUDA_TRY(cudaMemcpy(out + (size_t)b * max_tokens, m->d_out + (size_t)b * m->cfg.max_seq_len,
                               sizeof(int) * n, cudaMemcpyDeviceToHost));
    *n_out = n;
    return SB_OK;
}

void *sb_llama_stream(sb_llama *m) { return m ? (void *)m->st : nullptr; }

sb_status sb_llama_generate_greedy(sb_llama *m, int batch, const int32_t *prompts, int n_prompt, int max_tokens,
                                   int32_t *out) {
    SB_CHECK(m && out, SB_ERR_ARG, "sb_llama_generate_greedy: null argument");
    SB_CHECK(max_tokens >= 1, SB_ERR_ARG, "max_tokens must be >= 1");
    SB_CHECK(n_prompt + max_tokens - 1 <= m->cfg.max_seq_len, SB_ERR_SHAPE,
             "prompt %d + %d tokens exceed the cache (%d positions)", n_prompt, max_tokens, m->cfg.max_seq_len);
    SB_TRY(sb_llama_begin(m, batch, prompts, n_prompt));
    SB_TRY(sb_llama_step(m, n_prompt + max_tokens - 1));
    int n = 0;
    SB_TRY(sb_llama_tokens(m, out, max_tokens, &n));
    SB_CHECK(n == max_tokens, SB_ERR_STATE, "generated %d of %d tokens", n, max_tokens);
    return SB_OK;
}

sb_status sb_llama_profile_step(sb_llama *m, float *gemv_ms, float *attn_ms, float *other_ms, int *launches) {
    SB_CHECK(m && m->active > 0, SB_ERR_STATE, "sb_llama_profile_step: call sb_llama_begin first");
    SB_CHECK(m->steps + 1 <= m->cfg.max_seq_len, SB_ERR_SHAPE, "sb_llama_profile_step: cache full");
    StepProfiler p;
    p.st = m->st;
    SB_TRY(enqueue_step(m, m->active, m->st, false, false, &p));
    SB_CUDA_TRY(cudaStreamSynchronize(m->st));
    SB_TRY(qgemv_check_error());
    float t[3] = {0, 0, 0};
    for (size_t i = 0; i < p.cls.size(); i++) {
        float ms = 0;
        SB_CUDA_TRY(cudaEventElapsedTime(&ms, p.ev[2 * i], p.ev[2 * i + 1]));
        t[p.cls[i]] += ms;
    }
    m->steps += 1;
    if (gemv_ms) *gemv_ms = t[0];
    if (attn_ms) *attn_ms = t[1];
    if (other_ms) *other_ms = t[2];
    if (launches) *launches = (int)p.cls.size();
    return SB_OK;
}

sb_status sb_llama_step_launches(sb_llama *m, int batch, int *launches) {
    SB_CHECK(m && launches, SB_ERR_ARG, "sb_llama_step_launches: null argument");
    SB_CHECK(batch >= 1 && batch <= m->B, SB_ERR_SHAPE, "batch %d outside 1..%d", batch, m->B);
    if (batch == 1 && m->ds_ok)
        *launches = 1;  // the persistent step kernel
    else if (batch > QG_MAX_M) {
        // the q|k|v epilogue inside the one-split tensor-map attention
        const bool fuse = m->att_tma && tma_splits(m, batch) == 1;
        if (m->tp == 1)
            // embed; per layer the q|k|v GEMM (+ its finish unless fused; the
            // planes in layer 0), attention, o planes + GEMM + row finish,
            // gate/up and down GEMM + row finish; lm_head GEMM + finish; argmax
            *launches = fuse ? 5 + 9 * m->L : 5 + 10 * m->L;
        else
            // embed, 4 linears x 3 (q|k|v x 2 when fused) + attention per layer,
            // lm_head x 3, argmax
            *launches = fuse ? 5 + 12 * m->L : 5 + 13 * m->L;
    }
    else
        *launches = 3 + 5 * m->L;  // embed, 5 per layer, lm_head, argmax
    return SB_OK;
}

sb_status sb_llama_set_timeline(sb_llama *m, int enabled) {
    SB_CHECK(m, SB_ERR_ARG, "sb_llama_set_timeline: null model");
    SB_CHECK(m->ds_ok, SB_ERR_UNSUPPORTED, "sb_llama_set_timeline: this model does not run the persistent step");
    SB_CHECK(!enabled || ds_timeline_built(), SB_ERR_UNSUPPORTED,
             "sb_llama_set_timeline: this library was built without the step timeline (build with "
             "SB_STEP_TIMELINE=1 in the environment)");
    if (enabled && !m->ds_stamps) {
        const size_t n = (size_t)(6 * m->L + 2) * ds_grid() * DS_STAMPS;
        SB_TRY(dalloc_t(m, &m->ds_stamps, n));
    }
    if (!enabled) m->ds_stamps = nullptr;  // the buffer stays in m->allocs until destroy
    return SB_OK;
}

sb_status sb_llama_get_timeline(sb_llama *m, uint64_t *out, size_t cap, int *phases, int *ctas) {
    SB_CHECK(m && phases && ctas, SB_ERR_ARG, "sb_llama_get_timeline: null argument");
    SB_CHECK(m->ds_stamps, SB_ERR_STATE, "sb_llama_get_timeline: timeline not enabled");
    *phases = 6 * m->L + 2;
    *ctas = ds_grid();
    const size_t n = (size_t)(*phases) * (*ctas) * DS_STAMPS;
    if (out) {
        SB_CHECK(cap >= n, SB_ERR_SHAPE, "sb_llama_get_timeline: %zu slots, %zu needed", cap, n);
        SB_CUDA_TRY(cudaStreamSynchronize(m->st));
        SB_CUDA_TRY(cudaMemcpy(out, m->ds_stamps, sizeof(uint64_t) * n, cudaMemcpyDeviceToHost));
    }
    return SB_OK;
}

sb_status sb_llama_attn_plan(sb_llama *m, int batch, int *splits, int *tensor_map, int *chunk) {
    SB_CHECK(m, SB_ERR_ARG, "sb_llama_attn_plan: null model");
    SB_CHECK(batch >= 1 && batch <= m->B, SB_ERR_SHAPE, "batch %d outside 1..%d", batch, m->B);
    int s = 0, tm = 0, ch = 0;
    if (batch == 1 && m->ds_ok) {
        ch = m->ds_chunk;  // KV positions per ring stage of the persistent step
    } else {
        tm = m->att_tma ? 1 : 0;
        s = m->att_tma ? tma_splits(m, batch) : m->att_splits;
        ch = m->att_tma ? 64 : 0;  // the tensor-map kernel's tile
    }
    if (splits) *splits = s;
    if (tensor_map) *tensor_map = tm;
    if (chunk) *chunk = ch;
    return SB_OK;
}

sb_status sb_llama_step_bytes(sb_llama *m, double *weight_bytes, double *kv_bytes_per_pos) {
    SB_CHECK(m, SB_ERR_ARG, "null model");
    const double h = m->h, F = m->F, V = m->V;
    const double per_layer = h * m->qkv_dim + (double)m->q_dim * h + 2.0 * h * F + F * h;
    if (weight_bytes) *weight_bytes = per_layer * m->L + V * h;  // int8 bytes (+ negligible scalar scales)
    if (kv_bytes_per_pos) *kv_bytes_per_pos = 2.0 * m->L * m->kv_dim * (m->kv_f32 ? 4.0 : 2.0);
    return SB_OK;
}

}  // extern "C"
