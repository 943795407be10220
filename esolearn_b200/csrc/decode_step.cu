// Persistent decode step for one sequence: the whole of
// LlamaModel::forward_with_llama_cache (llama.rs:744-763) for int8 weights
// plus the greedy pick of generate() (generate.rs:72-89), as ONE cooperative
// kernel with one CTA per SM.
//
// Why one kernel.  At batch 1 the step is a chain of 4 GEMVs + attention per
// layer whose inputs depend on the previous link, and each weight matrix is
// only 17-90 MB.  Launched as separate kernels, every link pays a start-up
// (fetching and quantizing its input row) and a tail, and its tile count
// never divides evenly over the 148 SMs.  Here a producer warp per CTA
// streams every byte the step reads -- all weights of all layers in order,
// and each layer's K/V rows -- through a deep ring of 16 KB shared-memory
// stages with 1-D TMA bulk copies.  None of those bytes depends on the
// step's own results (the new token's K/V row is patched in shared memory),
// so the stream never waits for computation, only for free ring slots: the
// ring keeps filling while the consumer warps wait at a phase boundary.
//
// Work split.  Each GEMV's packed weight is one linear sequence of stages
// (tile-major, 8 k-steps of a 128-column tile per stage); CTA c takes stages
// [c*U/G, (c+1)*U/G), so every SM streams the same byte count (imbalance
// below 3% for llama2-7b shapes).  Partial column sums of a tile split between
// CTAs are exact integers and meet in an int64 buffer through atomic adds,
// so the result does not depend on the split: y = (f32)(sum * 2^-shift *
// scale * rstd) is bit-identical to the per-kernel GEMV (qgemv.cu).
// Attention splits the (kv head, KV chunk) sequence the same way; each CTA
// keeps an online-softmax partial per head it touches and the next
// projection's input stage combines the partials in CTA order.
//
// Phases and ordering.  Per layer: QKV -> ATT -> O -> GU -> ACT -> DOWN, then
// LM -> ARGMAX.  A phase's consumers wait until every CTA has arrived at the
// end of the previous phase (one monotonic counter in global memory,
// release/acquire at gpu scope).  Each GEMV input stage rebuilds the input
// row from the previous phase's outputs: residual add of the previous
// projection (x + y), fused RMSNorm, SwiGLU (its own phase: the f64 SiLU is
// computed once per element, split across CTAs), attention combine.
//
// Every wait is bounded (2 s of %globaltimer).  A wait that runs out raises
// the abort flag in sync[2]; all CTAs then skip the rest of the step, wait
// (bounded) for their copies in flight, and exit; the host reports
// SB_ERR_TIMEOUT.
#include "decode_step.cuh"

#include <algorithm>

namespace sb {

// Entry points of the instantiation units (decode_step_<hd>_<kv>.cu).
int ds_limit_128_bf16(int rep, int *limit);
int ds_limit_128_f32(int rep, int *limit);
int ds_limit_64_bf16(int rep, int *limit);
int ds_limit_64_f32(int rep, int *limit);
int ds_launch_128_bf16(const DsArgs &a, int rep, cudaStream_t st);
int ds_launch_128_f32(const DsArgs &a, int rep, cudaStream_t st);
int ds_launch_64_bf16(const DsArgs &a, int rep, cudaStream_t st);
int ds_launch_64_f32(const DsArgs &a, int rep, cudaStream_t st);

bool ds_supported(int h, int F, int q_dim, int hd, int rep, int kv_f32, int page_size, int *chunk) {
    if (hd != 64 && hd != 128) return false;
    if (rep != 1 && rep != 2 && rep != 4 && rep != 8) return false;
    if (h > DS_QMAX_H * DS_CONSUMERS * 4 || q_dim > DS_QMAX_H * DS_CONSUMERS * 4) return false;
    if (F > DS_QMAX_F * DS_CONSUMERS * 4) return false;
    if (h % 4 || q_dim % 4 || F % 4) return false;  // the input stages read quads
    const int per_stage = DS_KV_HALF / (hd * (kv_f32 ? 4 : 2));
    const int ch = std::min(per_stage, page_size);
    if (ch < 1 || page_size % ch != 0) return false;
    if (chunk) *chunk = ch;
    return true;
}

int ds_plan(int ksmax, int rep, int hd, int chunk, int kv_f32, int mtab, int *nst, size_t *smem) {
    int limit = 0;
    int rc;
    if (hd == 128) rc = kv_f32 ? ds_limit_128_f32(rep, &limit) : ds_limit_128_bf16(rep, &limit);
    else rc = kv_f32 ? ds_limit_64_f32(rep, &limit) : ds_limit_64_bf16(rep, &limit);
    SB_TRY(rc);
    const size_t fixed = ds_layout(0, ksmax, rep, hd, chunk, mtab).total;
    int n = 0;
    if ((size_t)limit > fixed) n = (int)(((size_t)limit - fixed) / (DS_STAGE + 16));
    n = std::min(n, DS_MAX_NST);
    *nst = n >= 3 ? n : 0;
    *smem = *nst ? ds_layout(*nst, ksmax, rep, hd, chunk, mtab).total : 0;
    return SB_OK;
}

int ds_grid() { return device_props().sm_count; }

bool ds_timeline_built() {
#ifdef SB_STEP_TIMELINE
    return true;
#else
    return false;
#endif
}

int ds_mtab_bytes(int nh, int nkv) { return (2 * nh * (ds_grid() / nkv + 2) + nh) * 4; }

size_t ds_part_floats(int nkv, int rep, int hd) { return (size_t)nkv * ds_grid() * rep * DS_REC(hd); }

int ds_launch(const DsArgs &a, int rep, cudaStream_t st) {
    SB_CHECK(a.nst >= 3 && a.nst <= DS_MAX_NST, SB_ERR_ARG, "decode step: ring of %d stages", a.nst);
    if (a.hd == 128) return a.kv_f32 ? ds_launch_128_f32(a, rep, st) : ds_launch_128_bf16(a, rep, st);
    if (a.hd == 64) return a.kv_f32 ? ds_launch_64_f32(a, rep, st) : ds_launch_64_bf16(a, rep, st);
    return set_error(SB_ERR_UNSUPPORTED, "decode step: head_dim %d", a.hd);
}

int ds_error_peek(const unsigned *sync_dev, unsigned *host, cudaStream_t st) {
    SB_CUDA_TRY(cudaMemcpyAsync(host, sync_dev + 2, sizeof(unsigned), cudaMemcpyDeviceToHost, st));
    return SB_OK;
}

int ds_check_error(unsigned *sync_dev, cudaStream_t st) {
    unsigned f = 0;
    SB_CUDA_TRY(cudaMemcpyAsync(&f, sync_dev + 2, sizeof f, cudaMemcpyDeviceToHost, st));
    SB_CUDA_TRY(cudaStreamSynchronize(st));
    if (f) {
        SB_CUDA_TRY(cudaMemsetAsync(sync_dev, 0, 3 * sizeof(unsigned), st));
        SB_CUDA_TRY(cudaStreamSynchronize(st));
        return set_error(SB_ERR_TIMEOUT, "decode step: a bounded wait timed out; the step was abandoned");
    }
    return SB_OK;
}

}  // namespace sb
