// Decode attention for one new token per sequence.  Replaces the reference
// decode attention (llama.rs:414-456): gather_reshape_repeat_kv
// (cpu.rs:707-730) materialised n_q copies of the cache; QK^T and AV were
// strided-batched GEMVs (cpu.rs:1337-1350) and softmax a separate pass
// (cpu.rs:336-366).
//
// Here one CTA handles (sequence b, kv head g, context split s).  It reads
// each K and V row of its split once and applies it to all n_rep query
// heads of the group (q-head h uses kv-head h / n_rep, as the GQA gather
// does).  Scores are f32 dot products of the pre-scaled query with K; the
// split keeps its own max m_s, sum l_s and unnormalised output o_s.  When a
// sequence is split, the last CTA of (b, g) to finish (arrival counter in
// scratch) combines the splits in split order:
//   out = sum_s exp(m_s - M) o_s / sum_s exp(m_s - M) l_s,  M = max_s m_s,
// which equals softmax(QK^T) V.  The combine order is fixed, so results do
// not depend on CTA scheduling.
#include "attention.cuh"

#include <algorithm>

namespace sb {

constexpr int ATT_THREADS = 128;

template <typename KV>
struct KvLoad;
template <>
struct KvLoad<__nv_bfloat16> {
    static constexpr int EPL = 8;  // elements per 16-byte load
    __device__ static void load(const __nv_bfloat16 *p, float v[8]) {
        const uint4 u = *reinterpret_cast<const uint4 *>(p);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            v[2 * i] = __uint_as_float(w[i] << 16);
            v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
        }
    }
};
template <>
struct KvLoad<float> {
    static constexpr int EPL = 4;
    __device__ static void load(const float *p, float v[4]) {
        const float4 u = *reinterpret_cast<const float4 *>(p);
        v[0] = u.x, v[1] = u.y, v[2] = u.z, v[3] = u.w;
    }
};

template <int HD, int REP, typename KV>
__global__ void __launch_bounds__(ATT_THREADS) attn_decode_kernel(const AttnArgs a) {
    using LD = KvLoad<KV>;
    constexpr int EPL = LD::EPL;
    constexpr int LPP = HD / EPL;          // lanes per position row
    constexpr int PPW = 32 / LPP;          // position rows per warp pass
    constexpr int NW = ATT_THREADS / 32;
    constexpr int NPG = ATT_THREADS / LPP; // position groups in the AV pass
    static_assert(LPP <= 32 && 32 % LPP == 0, "head_dim / lanes mismatch");

    extern __shared__ __align__(16) float sm[];
    float *qs = sm;                        // [REP][HD]
    float *sc = qs + REP * HD;             // [REP][max_chunk]
    float *red = sc + REP * a.max_chunk;   // [NPG][REP][HD]
    __shared__ float s_m[REP], s_l[REP];
    __shared__ int s_last;

    const int g = blockIdx.x, s = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int qdim = a.n_heads * HD;

    pdl_launch_dependents();
    pdl_wait();

    const int cap = min(a.max_pages * a.page_size, a.max_chunk * a.n_splits);
    const int ctx = min(max(a.len_is_pos ? a.len[b] + 1 : a.len[b], 0), cap);
    const int chunk = (ctx + a.n_splits - 1) / a.n_splits;
    const int p0 = s * chunk;
    const int p1 = min(p0 + chunk, ctx);
    const int n = max(p1 - p0, 0);

    for (int i = tid; i < REP * HD; i += ATT_THREADS) qs[i] = a.q[(size_t)b * qdim + (size_t)g * REP * HD + i];
    __syncthreads();

    const KV *kc = reinterpret_cast<const KV *>(a.kc);
    const KV *vc = reinterpret_cast<const KV *>(a.vc);
    const int *ptab = a.page_table + (size_t)b * a.max_pages;
    const int sub = lane % LPP;

    // ---- scores: sc[r][p - p0] = q_r . k_p
    for (int pb = warp * PPW; pb < n; pb += NW * PPW) {
        const int pi = pb + lane / LPP;
        float dots[REP];
#pragma unroll
        for (int r = 0; r < REP; r++) dots[r] = 0.0f;
        if (pi < n) {
            const int p = p0 + pi;
            const int page = ptab[p / a.page_size], slot = p % a.page_size;
            float kv[EPL];
            LD::load(kc + (((size_t)page * a.n_kv + g) * a.page_size + slot) * HD + sub * EPL, kv);
#pragma unroll
            for (int r = 0; r < REP; r++) {
                const float *qr = qs + r * HD + sub * EPL;
#pragma unroll
                for (int e = 0; e < EPL; e++) dots[r] = fmaf(qr[e], kv[e], dots[r]);
            }
        }
#pragma unroll
        for (int r = 0; r < REP; r++) {
#pragma unroll
            for (int o = LPP / 2; o > 0; o >>= 1) dots[r] += __shfl_xor_sync(0xffffffffu, dots[r], o);
        }
        if (sub == 0 && pi < n) {
#pragma unroll
            for (int r = 0; r < REP; r++) sc[r * a.max_chunk + pi] = dots[r];
        }
    }
    __syncthreads();

    // ---- per-head max and exp / sum (softmax numerator of this split)
    for (int r = warp; r < REP; r += NW) {
        float mx = -INFINITY;
        for (int i = lane; i < n; i += 32) mx = fmaxf(mx, sc[r * a.max_chunk + i]);
        mx = warp_max_f(mx);
        float sum = 0.0f;
        for (int i = lane; i < n; i += 32) {
            const float e = expf(sc[r * a.max_chunk + i] - mx);
            sc[r * a.max_chunk + i] = e;
            sum += e;
        }
        sum = warp_sum_f(sum);
        if (lane == 0) s_m[r] = mx, s_l[r] = sum;
    }
    __syncthreads();

    // ---- AV: o[r][d] = sum_p e[r][p] v_p[d]
    {
        const int pg = tid / LPP;
        float acc[REP][EPL];
#pragma unroll
        for (int r = 0; r < REP; r++)
#pragma unroll
            for (int e = 0; e < EPL; e++) acc[r][e] = 0.0f;
        for (int pi = pg; pi < n; pi += NPG) {
            const int p = p0 + pi;
            const int page = ptab[p / a.page_size], slot = p % a.page_size;
            float vv[EPL];
            LD::load(vc + (((size_t)page * a.n_kv + g) * a.page_size + slot) * HD + sub * EPL, vv);
#pragma unroll
            for (int r = 0; r < REP; r++) {
                const float w = sc[r * a.max_chunk + pi];
#pragma unroll
                for (int e = 0; e < EPL; e++) acc[r][e] = fmaf(w, vv[e], acc[r][e]);
            }
        }
#pragma unroll
        for (int r = 0; r < REP; r++)
#pragma unroll
            for (int e = 0; e < EPL; e++) red[((size_t)pg * REP + r) * HD + sub * EPL + e] = acc[r][e];
    }
    __syncthreads();

    const size_t hbase = (size_t)b * a.n_heads + (size_t)g * REP;  // first q head of the group
    if (a.n_splits == 1) {
        for (int i = tid; i < REP * HD; i += ATT_THREADS) {
            const int r = i / HD, d = i % HD;
            float o = 0.0f;
            for (int q = 0; q < NPG; q++) o += red[((size_t)q * REP + r) * HD + d];
            a.out[(hbase + r) * HD + d] = o / s_l[r];
        }
        return;
    }

    // ---- split partials -> scratch, last CTA of (b, g) combines in order
    const int stride = HD + 2;
    for (int i = tid; i < REP * HD; i += ATT_THREADS) {
        const int r = i / HD, d = i % HD;
        float o = 0.0f;
        for (int q = 0; q < NPG; q++) o += red[((size_t)q * REP + r) * HD + d];
        a.part[((hbase + r) * a.n_splits + s) * stride + d] = o;
    }
    if (tid < REP) {
        a.part[((hbase + tid) * a.n_splits + s) * stride + HD] = (n > 0) ? s_m[tid] : -INFINITY;
        a.part[((hbase + tid) * a.n_splits + s) * stride + HD + 1] = (n > 0) ? s_l[tid] : 0.0f;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        unsigned *cnt = a.counters + (size_t)b * a.n_kv + g;
        const unsigned prev = atomicAdd(cnt, 1u);
        s_last = (prev == (unsigned)a.n_splits - 1);
        if (s_last) *cnt = 0u;  // ready for the next launch
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int i = tid; i < REP * HD; i += ATT_THREADS) {
        const int r = i / HD, d = i % HD;
        const float *pr = a.part + (hbase + r) * a.n_splits * stride;
        float M = -INFINITY;
        for (int t = 0; t < a.n_splits; t++) M = fmaxf(M, __ldcg(pr + t * stride + HD));
        float L = 0.0f, O = 0.0f;
        for (int t = 0; t < a.n_splits; t++) {
            const float mt = __ldcg(pr + t * stride + HD);
            if (mt == -INFINITY) continue;
            const float w = expf(mt - M);
            L = fmaf(__ldcg(pr + t * stride + HD + 1), w, L);
            O = fmaf(__ldcg(pr + t * stride + d), w, O);
        }
        a.out[(hbase + r) * HD + d] = O / L;
    }
}

int attn_pick_splits(int B, int n_kv, int max_ctx) {
    const int sms = device_props().sm_count;
    int splits = ceil_div(2 * sms, std::max(1, B * n_kv));
    splits = std::min(splits, ceil_div(std::max(max_ctx, 1), 16));
    return std::max(1, std::min(splits, 64));
}

size_t attn_scratch_floats(int B, int n_heads, int n_splits, int hd) {
    return (size_t)B * n_heads * n_splits * (hd + 2);
}

template <int HD, int REP, typename KV>
static int attn_inst(const AttnArgs &a, cudaStream_t st, bool pdl) {
    constexpr int EPL = KvLoad<KV>::EPL;
    constexpr int NPG = ATT_THREADS / (HD / EPL);
    const size_t smem = sizeof(float) * ((size_t)REP * HD + (size_t)REP * a.max_chunk + (size_t)NPG * REP * HD);
    auto kern = attn_decode_kernel<HD, REP, KV>;
    static int limit[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!limit[dev & 63]) SB_TRY(allow_max_dynamic_smem(kern, &limit[dev & 63]));  // once, before any capture
    SB_CHECK(smem <= (size_t)limit[dev & 63], SB_ERR_SHAPE,
             "attention: split of %d positions needs %zu B shared memory (limit %d)", a.max_chunk, smem,
             limit[dev & 63]);
    SB_CUDA_TRY(launch(kern, dim3(a.n_kv, a.n_splits, a.B), dim3(ATT_THREADS), smem, st, pdl, a));
    return SB_OK;
}

template <int HD, typename KV>
static int attn_rep(const AttnArgs &a, cudaStream_t st, bool pdl) {
    switch (a.n_heads / a.n_kv) {
    case 1: return attn_inst<HD, 1, KV>(a, st, pdl);
    case 2: return attn_inst<HD, 2, KV>(a, st, pdl);
    case 4: return attn_inst<HD, 4, KV>(a, st, pdl);
    case 8: return attn_inst<HD, 8, KV>(a, st, pdl);
    default:
        return set_error(SB_ERR_UNSUPPORTED, "attention: GQA ratio %d not in {1,2,4,8}", a.n_heads / a.n_kv);
    }
}

int attn_launch(const AttnArgs &a, cudaStream_t st, bool pdl) {
    SB_CHECK(a.n_kv > 0 && a.n_heads % a.n_kv == 0, SB_ERR_SHAPE, "attention: n_heads %% n_kv != 0");
    SB_CHECK(a.n_splits == 1 || (a.part && a.counters), SB_ERR_ARG, "attention: split without scratch");
    SB_CHECK(a.max_chunk > 0, SB_ERR_ARG, "attention: max_chunk must be positive");
    if (a.hd == 128) return a.kv_f32 ? attn_rep<128, float>(a, st, pdl) : attn_rep<128, __nv_bfloat16>(a, st, pdl);
    if (a.hd == 64) return a.kv_f32 ? attn_rep<64, float>(a, st, pdl) : attn_rep<64, __nv_bfloat16>(a, st, pdl);
    return set_error(SB_ERR_UNSUPPORTED, "attention: head_dim %d not in {64,128}", a.hd);
}

}  // namespace sb
