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

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Positions per shared-memory tile (K and V tiles of T*HD elements each,
// double buffered).
template <typename KV>
constexpr int att_tile() {
    return sizeof(KV) == 2 ? 64 : 32;
}

template <int HD, int REP, typename KV>
constexpr size_t att_smem_bytes() {
    return (size_t)4 * att_tile<KV>() * HD * sizeof(KV) + sizeof(float) * ((size_t)REP * HD + (size_t)REP * att_tile<KV>());
}

template <int HD, int REP, typename KV>
__global__ void __launch_bounds__(ATT_THREADS) attn_decode_kernel(const AttnArgs a) {
    using LD = KvLoad<KV>;
    constexpr int EPL = LD::EPL;            // elements per 16-byte chunk
    constexpr int LPP = HD / EPL;           // chunks (lanes) per position row
    constexpr int PPW = 32 / LPP;           // position rows per warp pass
    constexpr int NW = ATT_THREADS / 32;
    constexpr int NPG = ATT_THREADS / LPP;  // position groups in the AV pass
    constexpr int T = att_tile<KV>();
    constexpr int TE = T * HD;
    static_assert(LPP <= 32 && 32 % LPP == 0, "head_dim / lanes mismatch");
    static_assert((size_t)NPG * REP * HD * 4 <= (size_t)4 * TE * sizeof(KV), "reduction buffer must fit the tiles");

    extern __shared__ __align__(16) uint8_t smraw[];
    KV *kt = reinterpret_cast<KV *>(smraw);             // [2][T][HD]
    KV *vt = kt + 2 * TE;                                // [2][T][HD]
    float *qs = reinterpret_cast<float *>(vt + 2 * TE);  // [REP][HD]
    float *sc = qs + REP * HD;                           // [REP][T]
    float *red = reinterpret_cast<float *>(smraw);       // [NPG][REP][HD], reuses the tiles after the loop
    __shared__ float s_m[REP], s_l[REP], s_alpha[REP];
    __shared__ int s_last;

    const int g = blockIdx.x, s = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int qdim = a.n_heads * HD;

    pdl_launch_dependents();
    pdl_wait();

    const int cap = a.max_pages * a.page_size;
    const int ctx = min(max(a.len_is_pos ? a.len[b] + 1 : a.len[b], 0), cap);
    const int chunk = (ctx + a.n_splits - 1) / a.n_splits;
    const int p0 = min(s * chunk, ctx);
    const int p1 = min(p0 + chunk, ctx);
    const int n = p1 - p0;
    const int ntiles = (n + T - 1) / T;

    const KV *kc = reinterpret_cast<const KV *>(a.kc);
    const KV *vc = reinterpret_cast<const KV *>(a.vc);
    const int *ptab = a.page_table + (size_t)b * a.max_pages;

    // Copy K and V rows of tile t into buffer buf (16-byte async copies).
    auto issue = [&](int t, int buf) {
        const int base = p0 + t * T;
        const int cnt = min(T, p1 - base);
        for (int c = tid; c < cnt * LPP; c += ATT_THREADS) {
            const int i = c / LPP, sub = c - (c / LPP) * LPP;
            const int p = base + i;
            const int page = ptab[p / a.page_size], slot = p % a.page_size;
            const size_t off = (((size_t)page * a.n_kv + g) * a.page_size + slot) * HD + sub * EPL;
            cp_async16(kt + buf * TE + i * HD + sub * EPL, kc + off);
            cp_async16(vt + buf * TE + i * HD + sub * EPL, vc + off);
        }
        cp_async_commit();
    };
    if (ntiles > 0) issue(0, 0);

    for (int i = tid; i < REP * HD; i += ATT_THREADS) qs[i] = a.q[(size_t)b * qdim + (size_t)g * REP * HD + i];
    if (tid < REP) s_m[tid] = -INFINITY, s_l[tid] = 0.0f;

    const int sub = lane % LPP;
    const int pg = tid / LPP, asub = tid % LPP;
    float acc[REP][EPL];
#pragma unroll
    for (int r = 0; r < REP; r++)
#pragma unroll
        for (int e = 0; e < EPL; e++) acc[r][e] = 0.0f;

    for (int t = 0; t < ntiles; t++) {
        const int buf = t & 1;
        if (t + 1 < ntiles) {
            issue(t + 1, buf ^ 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncthreads();
        const int cnt = min(T, p1 - (p0 + t * T));
        const KV *kb = kt + buf * TE;
        const KV *vb = vt + buf * TE;

        // scores of this tile: sc[r][i] = q_r . k_i
        for (int pb = warp * PPW; pb < cnt; pb += NW * PPW) {
            const int pi = pb + lane / LPP;
            float dots[REP];
#pragma unroll
            for (int r = 0; r < REP; r++) dots[r] = 0.0f;
            if (pi < cnt) {
                float kv[EPL];
                LD::load(kb + pi * HD + sub * EPL, kv);
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
            if (sub == 0 && pi < cnt) {
#pragma unroll
                for (int r = 0; r < REP; r++) sc[r * T + pi] = dots[r];
            }
        }
        __syncthreads();

        // online softmax: running max / sum per head, tile probabilities in sc
        for (int r = warp; r < REP; r += NW) {
            float mx = -INFINITY;
            for (int i = lane; i < cnt; i += 32) mx = fmaxf(mx, sc[r * T + i]);
            mx = warp_max_f(mx);
            const float m_old = s_m[r];
            const float m_new = fmaxf(m_old, mx);
            float sum = 0.0f;
            for (int i = lane; i < cnt; i += 32) {
                const float e = expf(sc[r * T + i] - m_new);
                sc[r * T + i] = e;
                sum += e;
            }
            sum = warp_sum_f(sum);
            if (lane == 0) {
                const float alpha = m_old == -INFINITY ? 0.0f : expf(m_old - m_new);
                s_alpha[r] = alpha;
                s_l[r] = fmaf(s_l[r], alpha, sum);
                s_m[r] = m_new;
            }
        }
        __syncthreads();

        // AV: acc[r][e] = alpha_r * acc[r][e] + sum_i p[r][i] v_i[e]
#pragma unroll
        for (int r = 0; r < REP; r++) {
            const float al = s_alpha[r];
#pragma unroll
            for (int e = 0; e < EPL; e++) acc[r][e] *= al;
        }
        for (int pi = pg; pi < cnt; pi += NPG) {
            float vv[EPL];
            LD::load(vb + pi * HD + asub * EPL, vv);
#pragma unroll
            for (int r = 0; r < REP; r++) {
                const float w = sc[r * T + pi];
#pragma unroll
                for (int e = 0; e < EPL; e++) acc[r][e] = fmaf(w, vv[e], acc[r][e]);
            }
        }
        __syncthreads();  // the buffer may be refilled by the next issue
    }

#pragma unroll
    for (int r = 0; r < REP; r++)
#pragma unroll
        for (int e = 0; e < EPL; e++) red[((size_t)pg * REP + r) * HD + asub * EPL + e] = acc[r][e];
    __syncthreads();

    const size_t hbase = (size_t)b * a.n_heads + (size_t)g * REP;  // first q head of the group
    if (a.n_splits == 1) {
        for (int i = tid; i < REP * HD; i += ATT_THREADS) {
            const int r = i / HD, d = i % HD;
            float o = 0.0f;
            for (int q = 0; q < NPG; q++) o += red[((size_t)q * REP + r) * HD + d];
            a.out[(hbase + r) * HD + d] = s_l[r] > 0.0f ? o / s_l[r] : 0.0f;
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
        float Lsum = 0.0f, O = 0.0f;
        for (int t = 0; t < a.n_splits; t++) {
            const float mt = __ldcg(pr + t * stride + HD);
            if (mt == -INFINITY) continue;
            const float w = expf(mt - M);
            Lsum = fmaf(__ldcg(pr + t * stride + HD + 1), w, Lsum);
            O = fmaf(__ldcg(pr + t * stride + d), w, O);
        }
        a.out[(hbase + r) * HD + d] = Lsum > 0.0f ? O / Lsum : 0.0f;
    }
}

int attn_pick_splits(int B, int n_kv, int max_ctx) {
    const int sms = device_props().sm_count;
    int splits = std::max(ceil_div(2 * sms, std::max(1, B * n_kv)), ceil_div(std::max(max_ctx, 1), 256));
    splits = std::min(splits, ceil_div(std::max(max_ctx, 1), 16));
    return std::max(1, std::min(splits, 64));
}

size_t attn_scratch_floats(int B, int n_heads, int n_splits, int hd) {
    return (size_t)B * n_heads * n_splits * (hd + 2);
}

template <int HD, int REP, typename KV>
static int attn_inst(const AttnArgs &a, cudaStream_t st, bool pdl) {
    const size_t smem = att_smem_bytes<HD, REP, KV>();
    auto kern = attn_decode_kernel<HD, REP, KV>;
    static int limit[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!limit[dev & 63]) SB_TRY(allow_max_dynamic_smem(kern, &limit[dev & 63]));  // once, before any capture
    SB_CHECK(smem <= (size_t)limit[dev & 63], SB_ERR_SHAPE, "attention: needs %zu B shared memory (limit %d)", smem,
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
    if (attn_tc_supported(a)) return attn_tc_launch(a, st, pdl);
    if (a.hd == 128) return a.kv_f32 ? attn_rep<128, float>(a, st, pdl) : attn_rep<128, __nv_bfloat16>(a, st, pdl);
    if (a.hd == 64) return a.kv_f32 ? attn_rep<64, float>(a, st, pdl) : attn_rep<64, __nv_bfloat16>(a, st, pdl);
    return set_error(SB_ERR_UNSUPPORTED, "attention: head_dim %d not in {64,128}", a.hd);
}

}  // namespace sb
