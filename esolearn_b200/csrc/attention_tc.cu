// Decode attention on the tensor cores for grouped-query heads (2, 4 or 8
// query heads per KV head) over a bf16 KV cache: the batched-decode form of
// llama.rs:414-456 (the GQA gather of cpu.rs:707-730, QK^T and AV as
// strided GEMVs, cpu.rs:1337-1350, softmax cpu.rs:336-366).
//
// With n_rep query heads per KV head every K/V element takes 2 * n_rep
// multiply-adds; at 4 or 8 heads per group that is more FMA work than the SM
// can retire while HBM delivers the cache, so both products run as
// mma.sync m16n8k16 bf16 -> f32 tiles.  K and V are exact bf16 values; the
// f32 query and the f32 probabilities are each split into a bf16 high part
// and a bf16 low part (x = hi + lo to about 2^-17 relative), and both parts
// go through the same MMA as separate rows of the A operand:
//   rows h     : hi(q_h) / hi(p_h)      rows h + 8 : lo(q_h) / lo(p_h)
// so every thread holds the hi and lo partial of the same head and adds them
// in registers.  Products of bf16 values are exact in f32, so the result
// matches the f32 SIMT kernel (attention.cu) to f32 rounding.
//
// Work split: one CTA per (kv head, context split, sequence) like
// attention.cu; K/V tiles of 64 positions stream through a 3-stage cp.async
// ring into padded shared-memory rows (272 B for hd 128, conflict-free
// ldmatrix); each of the 4 warps takes 16 positions of a tile and keeps its
// own online softmax (running max, sum, unnormalised output); warps are
// combined through shared memory at the end, splits by the last CTA of a
// (sequence, kv head) in split order (deterministic).
#include "attention.cuh"
#include "mma_bf16.cuh"
#include "pipeline.cuh"

namespace sb {

namespace {

constexpr int ATC_WARPS = 4;  // consumer warps
constexpr int ATC_THREADS = ATC_WARPS * 32;

// Set by a bounded mbarrier wait of the tensor-map kernel that ran out.
__device__ unsigned atc_error_flag = 0;
constexpr int ATC_T = 64;  // positions per tile (16 per warp)
constexpr int ATC_NST = 3;

template <int HD>
constexpr int atc_row() {
    return HD + 8;  // bf16 elements per padded shared-memory row
}
template <int HD>
constexpr size_t atc_stage_bytes() {
    return (size_t)2 * ATC_T * atc_row<HD>() * 2;  // K and V
}
template <int HD, int REP>
constexpr size_t atc_smem_bytes() {
    return ATC_NST * atc_stage_bytes<HD>();
}

// Barrier of the consumer warps (a producer warp, when there is one, does not join).
__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, %0;" ::"n"(ATC_WARPS * 32) : "memory"); }

// Query fragments (A operand of S = Q K^T): row grp = hi(q), row grp+8 = lo(q).
template <int HD, int REP>
__device__ __forceinline__ void atc_load_q(const AttnArgs &a, int b, int g, int grp, int qd,
                                           uint32_t (&qa)[HD / 16][4]) {
    const float *q = a.q + (size_t)b * a.n_heads * HD + ((size_t)g * REP + grp) * HD;
    const bool live = grp < REP;
#pragma unroll
    for (int ks = 0; ks < HD / 16; ks++) {
        float x[4] = {0.f, 0.f, 0.f, 0.f};
        if (live) {
            const float2 u = *reinterpret_cast<const float2 *>(q + ks * 16 + 2 * qd);
            const float2 v = *reinterpret_cast<const float2 *>(q + ks * 16 + 8 + 2 * qd);
            x[0] = u.x, x[1] = u.y, x[2] = v.x, x[3] = v.y;
        }
        __nv_bfloat16 h[4], l[4];
#pragma unroll
        for (int i = 0; i < 4; i++) split_bf16(x[i], h[i], l[i]);
        qa[ks][0] = pack_bf16(h[0], h[1]);
        qa[ks][1] = pack_bf16(l[0], l[1]);
        qa[ks][2] = pack_bf16(h[2], h[3]);
        qa[ks][3] = pack_bf16(l[2], l[3]);
    }
}

// One warp's 16 positions [r0, r0+16) of a tile in shared memory (positions
// >= cnt masked): scores, online softmax update, P V.  kaddr(prow, c) and
// vaddr(prow, c) give the shared address of 16-byte chunk c (8 elements of
// head dim) of tile row prow in the K and V buffers.
template <int HD, typename KA, typename VA>
__device__ __forceinline__ void atc_block_impl(const uint32_t (&qa)[HD / 16][4], const KA &kaddr, const VA &vaddr,
                                               int r0, int cnt, float &m_run, float &l_run, float (&o)[HD / 8][4]) {
    constexpr int KSTEPS = HD / 16, NB = HD / 8;
    const int lane = threadIdx.x & 31, qd = lane & 3;
    const int mi = lane >> 3, ri = lane & 7;
    // S^T blocks: c[nb] = scores of positions r0 + nb*8 + (2qd, 2qd+1), hi rows + lo rows
    float c[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    {
        const int prow = r0 + (mi >> 1) * 8 + ri;  // matrices: (pos 0-7, d), (0-7, d+8), (8-15, d), (8-15, d+8)
#pragma unroll
        for (int ks = 0; ks < KSTEPS; ks++) {
            uint32_t b0, b1, b2, b3;
            ldsm_x4(kaddr(prow, 2 * ks + (mi & 1)), b0, b1, b2, b3);
            mma_bf16(c[0], qa[ks], b0, b1);
            mma_bf16(c[1], qa[ks], b2, b3);
        }
    }
    float sc[2][2];
#pragma unroll
    for (int nb = 0; nb < 2; nb++)
#pragma unroll
        for (int e = 0; e < 2; e++) {
            const int p = r0 + nb * 8 + 2 * qd + e;
            sc[nb][e] = p < cnt ? __fadd_rn(c[nb][e], c[nb][2 + e]) : -INFINITY;
        }
    float mx = fmaxf(fmaxf(sc[0][0], sc[0][1]), fmaxf(sc[1][0], sc[1][1]));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float m_new = fmaxf(m_run, mx);  // finite: the block has a valid position
    const float alpha = m_run == -INFINITY ? 0.f : expf(m_run - m_new);
    m_run = m_new;
    float p[2][2];
    float psum = 0.f;
#pragma unroll
    for (int nb = 0; nb < 2; nb++)
#pragma unroll
        for (int e = 0; e < 2; e++) {
            p[nb][e] = sc[nb][e] == -INFINITY ? 0.f : expf(sc[nb][e] - m_new);
            psum += p[nb][e];
        }
    l_run = fmaf(l_run, alpha, psum);
#pragma unroll
    for (int j = 0; j < NB; j++)
#pragma unroll
        for (int e = 0; e < 4; e++) o[j][e] *= alpha;
    // P as the A operand of O = P V: cols 2qd.. of positions 0-7 and 8-15
    uint32_t pa[4];
    {
        __nv_bfloat16 h[2][2], l[2][2];
#pragma unroll
        for (int nb = 0; nb < 2; nb++)
#pragma unroll
            for (int e = 0; e < 2; e++) split_bf16(p[nb][e], h[nb][e], l[nb][e]);
        pa[0] = pack_bf16(h[0][0], h[0][1]);
        pa[1] = pack_bf16(l[0][0], l[0][1]);
        pa[2] = pack_bf16(h[1][0], h[1][1]);
        pa[3] = pack_bf16(l[1][0], l[1][1]);
    }
    {
        // matrices: (pos 0-7, d), (pos 8-15, d), (pos 0-7, d+8), (pos 8-15, d+8)
        const int prow = r0 + (mi & 1) * 8 + ri;
#pragma unroll
        for (int j = 0; j < NB; j += 2) {
            uint32_t b0, b1, b2, b3;
            ldsm_x4_t(vaddr(prow, j + (mi >> 1)), b0, b1, b2, b3);
            mma_bf16(o[j], pa, b0, b1);
            mma_bf16(o[j + 1], pa, b2, b3);
        }
    }
}

// Combine the consumer warps' records through shared memory (wo, which may
// alias the free stages) and write the split's partial -- or, unsplit, the
// output; the last CTA of (sequence, kv head) combines the splits in split
// order.  Called by the ATC_WARPS consumer warps only.
template <int HD, int REP>
__device__ __forceinline__ void atc_finish(const AttnArgs &a, int b, int g, int s, float m_run, float l_run,
                                           const float (&o)[HD / 8][4], float *wo, float (*s_m)[REP],
                                           float (*s_l)[REP], float *s_fm, float *s_fl, int *s_last) {
    constexpr int NB = HD / 8;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int grp = lane >> 2, qd = lane & 3;
    // head grp's output d = 8j + 2qd + e is o[j][e] + o[j][2+e]
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
    if (grp < REP) {
        if (qd == 0) s_m[warp][grp] = m_run, s_l[warp][grp] = l_run;
        float *dst = wo + ((size_t)warp * REP + grp) * HD;
#pragma unroll
        for (int j = 0; j < NB; j++) {
            const int d = j * 8 + 2 * qd;
            dst[d] = __fadd_rn(o[j][0], o[j][2]);
            dst[d + 1] = __fadd_rn(o[j][1], o[j][3]);
        }
    }
    consumer_sync();
    if (tid < REP) {
        float M = -INFINITY;
        for (int w = 0; w < ATC_WARPS; w++) M = fmaxf(M, s_m[w][tid]);
        float L = 0.f;
        if (M != -INFINITY)
            for (int w = 0; w < ATC_WARPS; w++)
                if (s_m[w][tid] != -INFINITY) L = fmaf(s_l[w][tid], expf(s_m[w][tid] - M), L);
        s_fm[tid] = M, s_fl[tid] = L;
    }
    consumer_sync();
    const size_t hbase = (size_t)b * a.n_heads + (size_t)g * REP;  // first q head of the group
    const int stride = HD + 2;
    for (int i = tid; i < REP * HD; i += ATC_WARPS * 32) {
        const int r = i / HD, d = i - r * HD;
        const float M = s_fm[r];
        float O = 0.f;
        if (M != -INFINITY)
            for (int w = 0; w < ATC_WARPS; w++)
                if (s_m[w][r] != -INFINITY) O = fmaf(wo[((size_t)w * REP + r) * HD + d], expf(s_m[w][r] - M), O);
        if (a.n_splits == 1)
            a.out[(hbase + r) * HD + d] = s_fl[r] > 0.f ? O / s_fl[r] : 0.f;
        else
            a.part[((hbase + r) * a.n_splits + s) * stride + d] = O;
    }
    if (a.n_splits == 1) return;
    if (tid < REP) {
        a.part[((hbase + tid) * a.n_splits + s) * stride + HD] = s_fm[tid];
        a.part[((hbase + tid) * a.n_splits + s) * stride + HD + 1] = s_fl[tid];
    }
    __threadfence();
    consumer_sync();
    if (tid == 0) {
        unsigned *cntr = a.counters + (size_t)b * a.n_kv + g;
        const unsigned prev = atomicAdd(cntr, 1u);
        *s_last = (prev == (unsigned)a.n_splits - 1);
        if (*s_last) *cntr = 0u;  // ready for the next launch
    }
    consumer_sync();
    if (!*s_last) return;
    __threadfence();
    for (int i = tid; i < REP * HD; i += ATC_WARPS * 32) {
        const int r = i / HD, d = i - r * HD;
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

// ---- kernel A: cp.async tiles into padded rows (any page size; the op-level ABI)
template <int HD, int REP>
__global__ void __launch_bounds__(ATC_THREADS) attn_tc_kernel(const AttnArgs a) {
    static_assert(REP == 2 || REP == 4 || REP == 8, "tensor-core attention takes 2, 4 or 8 heads per group");
    constexpr int RW = atc_row<HD>();
    constexpr int NB = HD / 8;
    constexpr int CPR = HD / 8;      // 16-byte chunks per K/V row

    extern __shared__ __align__(1024) uint8_t smraw[];
    __shared__ float s_m[ATC_WARPS][REP], s_l[ATC_WARPS][REP];
    __shared__ float s_fm[REP], s_fl[REP];
    __shared__ int s_last;

    const int g = blockIdx.x, s = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int grp = lane >> 2, qd = lane & 3;

    pdl_launch_dependents();
    pdl_wait();

    const int cap = a.max_pages * a.page_size;
    const int ctx = min(max(a.len_is_pos ? a.len[b] + 1 : a.len[b], 0), cap);
    const int chunk = (ctx + a.n_splits - 1) / a.n_splits;
    const int p0 = min(s * chunk, ctx);
    const int p1 = min(p0 + chunk, ctx);
    const int ntiles = (p1 - p0 + ATC_T - 1) / ATC_T;

    const __nv_bfloat16 *kc = reinterpret_cast<const __nv_bfloat16 *>(a.kc);
    const __nv_bfloat16 *vc = reinterpret_cast<const __nv_bfloat16 *>(a.vc);
    const int *ptab = a.page_table + (size_t)b * a.max_pages;
    const uint32_t sbase = smem_u32(smraw);

    // K and V rows of tile t into stage st (16-byte async copies, padded rows).
    auto issue = [&](int t, int st) {
        const int base = p0 + t * ATC_T;
        const int cnt = min(ATC_T, p1 - base);
        const uint32_t kdst = sbase + (uint32_t)(st * atc_stage_bytes<HD>());
        const uint32_t vdst = kdst + (uint32_t)(ATC_T * RW * 2);
        for (int c = tid; c < cnt * CPR; c += ATC_THREADS) {
            const int i = c / CPR, sub = c - i * CPR;
            const int p = base + i;
            const int page = ptab[p / a.page_size], slot = p % a.page_size;
            const size_t off = (((size_t)page * a.n_kv + g) * a.page_size + slot) * HD + sub * 8;
            const uint32_t so = (uint32_t)((i * RW + sub * 8) * 2);
            cp_async16(kdst + so, kc + off);
            cp_async16(vdst + so, vc + off);
        }
        // Rows past the context are read by the MMAs (with probability 0):
        // zero them, since 0 * (stale NaN or Inf) would poison the sums.
        for (int c = cnt * CPR + tid; c < ATC_T * CPR; c += ATC_THREADS) {
            const int i = c / CPR, sub = c - i * CPR;
            const uint32_t so = (uint32_t)((i * RW + sub * 8) * 2);
            asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};" ::"r"(kdst + so), "r"(0u) : "memory");
            asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};" ::"r"(vdst + so), "r"(0u) : "memory");
        }
    };
#pragma unroll
    for (int t = 0; t < ATC_NST - 1; t++) {
        if (t < ntiles) issue(t, t);
        cp_commit();
    }

    uint32_t qa[HD / 16][4];
    atc_load_q<HD, REP>(a, b, g, grp, qd, qa);
    float o[NB][4];
#pragma unroll
    for (int j = 0; j < NB; j++) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m_run = -INFINITY, l_run = 0.f;  // per head grp (l: this lane's share)

    for (int t = 0; t < ntiles; t++) {
        cp_wait<ATC_NST - 2>();
        __syncthreads();  // tile t is in shared memory; stage (t-1) % NST is free
        if (t + ATC_NST - 1 < ntiles) issue(t + ATC_NST - 1, (t + ATC_NST - 1) % ATC_NST);
        cp_commit();
        const int st = t % ATC_NST;
        const int cnt = min(ATC_T, p1 - (p0 + t * ATC_T));
        const int r0 = warp * 16;  // this warp's 16 positions of the tile
        if (r0 >= cnt) continue;
        const uint32_t kb = sbase + (uint32_t)(st * atc_stage_bytes<HD>());
        const uint32_t vb = kb + (uint32_t)(ATC_T * RW * 2);
        auto kaddr = [&](int prow, int c) { return kb + (uint32_t)((prow * RW + c * 8) * 2); };
        auto vaddr = [&](int prow, int c) { return vb + (uint32_t)((prow * RW + c * 8) * 2); };
        atc_block_impl<HD>(qa, kaddr, vaddr, r0, cnt, m_run, l_run, o);
    }
    cp_wait<0>();
    __syncthreads();  // every warp is done with the stages: reuse them for the combine
    atc_finish<HD, REP>(a, b, g, s, m_run, l_run, o, reinterpret_cast<float *>(smraw), s_m, s_l, s_fm, s_fl,
                        &s_last);
}

// ---- kernel B: 2-D TMA tiles of whole pages, 128-byte swizzle (the engine) --------
// A producer warp loads each 64-position tile of K and of V as HD/64 boxes of
// [64 rows x 64 elements] with cp.async.bulk.tensor (no multicast) from a
// tensor map over the whole cache ([rows][head_dim], all layers); the 128-byte
// swizzle stores 16-byte chunk c of box row r at chunk c ^ (r & 7), which
// keeps the ldmatrix row reads conflict-free without padding.  Splits start
// at multiples of 64 positions and pages hold a multiple of 64 positions, so
// a tile never crosses a page.  Rows past the context in the last tile hold
// finite cache values (written rows or the zero-initialised cache) and get
// probability 0.
constexpr int ATM_NST = 3;
constexpr uint32_t ATM_BOX = 64 * 128;  // bytes of one 64 x 64 bf16 box

template <int HD>
constexpr uint32_t atm_stage_bytes() {
    return 2 * (HD / 64) * ATM_BOX;  // K and V
}
template <int HD>
constexpr size_t atm_smem_bytes() {
    return ATM_NST * atm_stage_bytes<HD>() + 1024;  // + alignment of the swizzled boxes
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, int x, int y, uint32_t bar,
                                            uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar), "l"(policy)
        : "memory");
}

// ---- the q|k|v epilogue fused into the tensor-map kernel (one split) -------
// Producer warp: the new K and V rows of kv head g for sequence b, from the
// projection's int64 sums (RoPE on K, rope_with_freqs_preloaded, cpu.rs:
// 650-661), written as bf16 to the cache at position pos when 0 <= pos <
// max_pos; their sums are cleared either way.  The stores are then made
// visible to the async proxy, so a tensor-map load issued after this sees them.
template <int HD>
__device__ __forceinline__ void atm_new_kv(const AttnArgs &a, int b, int g, int pos) {
    const int lane = threadIdx.x & 31;
    const double f = gemv_factor(a.shift[b], a.qkv_scale, a.rstd[b]);
    long long *ks = const_cast<long long *>(a.qkv_sums) + (size_t)b * a.ld_sums + (size_t)a.n_heads * HD +
                    (size_t)g * HD;
    long long *vs = ks + (size_t)a.n_kv * HD;
    const bool live = pos >= 0 && pos < a.max_pos;
    size_t row = 0;
    if (live) {
        const int page = a.page_table[(size_t)b * a.max_pages + pos / a.page_size];
        row = (((size_t)page * a.n_kv + g) * a.page_size + pos % a.page_size) * HD;
    }
    __nv_bfloat16 *kc = reinterpret_cast<__nv_bfloat16 *>(const_cast<void *>(a.kc)) + row;
    __nv_bfloat16 *vc = reinterpret_cast<__nv_bfloat16 *>(const_cast<void *>(a.vc)) + row;
    for (int d0 = 2 * lane; d0 < HD; d0 += 64) {
        const long long t0 = __ldcg(ks + d0), t1 = __ldcg(ks + d0 + 1);
        const long long u0 = __ldcg(vs + d0), u1 = __ldcg(vs + d0 + 1);
        ks[d0] = 0, ks[d0 + 1] = 0, vs[d0] = 0, vs[d0 + 1] = 0;
        if (live) {
            const float y0 = gemv_out(t0, f), y1 = gemv_out(t1, f);
            const float cs = a.rope_cos[(size_t)pos * (HD / 2) + (d0 >> 1)];
            const float sn = a.rope_sin[(size_t)pos * (HD / 2) + (d0 >> 1)];
            kc[d0] = __float2bfloat16_rn(__fsub_rn(__fmul_rn(y0, cs), __fmul_rn(y1, sn)));
            kc[d0 + 1] = __float2bfloat16_rn(__fadd_rn(__fmul_rn(y0, sn), __fmul_rn(y1, cs)));
            vc[d0] = __float2bfloat16_rn(gemv_out(u0, f));
            vc[d0 + 1] = __float2bfloat16_rn(gemv_out(u1, f));
        }
    }
    asm volatile("fence.proxy.async.global;" ::: "memory");
    __syncwarp();
}

// Consumer lanes: the query fragments of head g * REP + grp (as atc_load_q)
// from the projection's sums: y = sum * factor, RoPE at the position, times
// q_scale (the projection epilogue's arithmetic, qgemm.cu QEPI_QKV).
template <int HD, int REP>
__device__ __forceinline__ void atm_load_q_sums(const AttnArgs &a, int b, int g, int grp, int qd, int pos,
                                                uint32_t (&qa)[HD / 16][4]) {
    const bool live = grp < REP;
    const double f = gemv_factor(a.shift[b], a.qkv_scale, a.rstd[b]);
    const long long *qs = a.qkv_sums + (size_t)b * a.ld_sums + ((size_t)g * REP + grp) * HD;
    const int rp = min(max(pos, 0), a.max_pos - 1);  // outside the cache the output is unused
    const float *cr = a.rope_cos + (size_t)rp * (HD / 2), *sr = a.rope_sin + (size_t)rp * (HD / 2);
#pragma unroll
    for (int k = 0; k < HD / 16; k++) {
        float x[4] = {0.f, 0.f, 0.f, 0.f};
        if (live) {
#pragma unroll
            for (int hlf = 0; hlf < 2; hlf++) {
                const int d0 = k * 16 + 8 * hlf + 2 * qd;
                const float y0 = gemv_out(__ldcg(qs + d0), f), y1 = gemv_out(__ldcg(qs + d0 + 1), f);
                const float cs = cr[d0 >> 1], sn = sr[d0 >> 1];
                x[2 * hlf] = __fmul_rn(__fsub_rn(__fmul_rn(y0, cs), __fmul_rn(y1, sn)), a.q_scale);
                x[2 * hlf + 1] = __fmul_rn(__fadd_rn(__fmul_rn(y0, sn), __fmul_rn(y1, cs)), a.q_scale);
            }
        }
        __nv_bfloat16 h[4], l[4];
#pragma unroll
        for (int i = 0; i < 4; i++) split_bf16(x[i], h[i], l[i]);
        qa[k][0] = pack_bf16(h[0], h[1]);
        qa[k][1] = pack_bf16(l[0], l[1]);
        qa[k][2] = pack_bf16(h[2], h[3]);
        qa[k][3] = pack_bf16(l[2], l[3]);
    }
}

// FUSED: the q|k|v projection's epilogue runs here (a.qkv_sums; one split).
template <int HD, int REP, bool FUSED>
__global__ void __launch_bounds__(ATC_THREADS + 32) attn_tc_tma_kernel(const __grid_constant__ AttnArgs a) {
    static_assert(REP == 2 || REP == 4 || REP == 8, "tensor-core attention takes 2, 4 or 8 heads per group");
    static_assert(HD % 64 == 0, "head_dim is whole 64-element boxes");
    constexpr int NB = HD / 8;
    constexpr int NBOX = HD / 64;
    constexpr uint32_t KVB = NBOX * ATM_BOX;  // K (or V) bytes of a tile

    extern __shared__ __align__(1024) uint8_t smraw[];
    __shared__ __align__(8) unsigned long long bars[2 * ATM_NST];  // full, empty
    __shared__ float s_m[ATC_WARPS][REP], s_l[ATC_WARPS][REP];
    __shared__ float s_fm[REP], s_fl[REP];
    __shared__ int s_last, s_abort;

    const int g = blockIdx.x, s = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int grp = lane >> 2, qd = lane & 3;
    const uint32_t sbase = (smem_u32(smraw) + 1023u) & ~1023u;
    const uint32_t b_full = smem_u32(&bars[0]), b_empty = smem_u32(&bars[ATM_NST]);
    if (tid == 0) {
        for (int i = 0; i < ATM_NST; i++) {
            mbar_init(b_full + 8 * i, 1);
            mbar_init(b_empty + 8 * i, ATC_WARPS);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        s_abort = 0;
    }
    __syncthreads();

    pdl_launch_dependents();
    pdl_wait();

    const int cap = a.max_pages * a.page_size;
    const int ctx = min(max(a.len_is_pos ? a.len[b] + 1 : a.len[b], 0), cap);
    const int chunk = ((ctx + a.n_splits - 1) / a.n_splits + ATC_T - 1) / ATC_T * ATC_T;
    const int p0 = min(s * chunk, ctx);
    const int p1 = min(p0 + chunk, ctx);
    const int ntiles = (p1 - p0 + ATC_T - 1) / ATC_T;

    if (warp == ATC_WARPS) {
        // ---- producer: one elected lane issues every tile's boxes; with
        // FUSED the whole warp writes the new K/V row before the tile that
        // holds it is requested (ahead of tile min(its tile, NST - 1): writing
        // it once the ring is full instead measured slower)
        const int pos = FUSED ? a.len[b] : -1;
        const int t_row = (FUSED && pos >= p0 && pos < p1) ? min((pos - p0) / ATC_T, ATM_NST - 1) : -1;
        bool row_done = false;
        const uint64_t pol = l2_evict_first_policy();  // every row is read once per step
        const int *ptab = a.page_table + (size_t)b * a.max_pages;
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&a.tmk)) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&a.tmv)) : "memory");
        }
        int t = 0;
        for (; t < ntiles; t++) {
            if (FUSED && t == t_row) {
                atm_new_kv<HD>(a, b, g, pos);
                row_done = true;
            }
            const int st = t % ATM_NST;
            int stop = 0;
            if (lane == 0) {
                if (t >= ATM_NST && (s_abort || !mbar_wait(b_empty + 8 * st, ((t / ATM_NST) - 1) & 1))) {
                    atomicOr(&atc_error_flag, 1u);
                    s_abort = 1;
                    stop = 1;
                } else {
                    const int p = p0 + t * ATC_T;
                    const int pg = ptab[p / a.page_size], slot = p % a.page_size;
                    const int row = (int)(a.tm_row0 + ((long long)pg * a.n_kv + g) * a.page_size + slot);
                    const uint32_t kdst = sbase + (uint32_t)st * atm_stage_bytes<HD>();
                    mbar_expect_tx(b_full + 8 * st, 2 * KVB);
#pragma unroll
                    for (int bx = 0; bx < NBOX; bx++) {
                        tma_load_2d(kdst + bx * ATM_BOX, &a.tmk, 64 * bx, row, b_full + 8 * st, pol);
                        tma_load_2d(kdst + KVB + bx * ATM_BOX, &a.tmv, 64 * bx, row, b_full + 8 * st, pol);
                    }
                }
            }
            if (__shfl_sync(0xffffffffu, stop, 0)) break;
        }
        if (FUSED && !row_done) atm_new_kv<HD>(a, b, g, pos);  // the sums are cleared in every case
        // leave no copy in flight: the last stages issued have landed
        if (lane == 0)
            for (int u = max(0, t - ATM_NST); u < t; u++)
                if (!mbar_wait(b_full + 8 * (u % ATM_NST), (u / ATM_NST) & 1)) atomicOr(&atc_error_flag, 1u);
        return;  // the consumer warps combine and write
    }

    uint32_t qa[HD / 16][4];
    if (FUSED) {
        atm_load_q_sums<HD, REP>(a, b, g, grp, qd, a.len[b], qa);
        consumer_sync();  // every consumer warp has its query; clear its sums
        if (warp == 0) {
            long long *qs = const_cast<long long *>(a.qkv_sums) + (size_t)b * a.ld_sums + (size_t)g * REP * HD;
            for (int i = lane; i < REP * HD; i += 32) qs[i] = 0;
        }
    } else {
        atc_load_q<HD, REP>(a, b, g, grp, qd, qa);
    }
    float o[NB][4];
#pragma unroll
    for (int j = 0; j < NB; j++) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m_run = -INFINITY, l_run = 0.f;  // per head grp (l: this lane's share)

    for (int t = 0; t < ntiles; t++) {
        const int st = t % ATM_NST;
        const bool ok = !s_abort && mbar_wait(b_full + 8 * st, (t / ATM_NST) & 1);
        if (__any_sync(0xffffffffu, !ok)) {
            if (lane == 0) atomicOr(&atc_error_flag, 1u), s_abort = 1;
            break;
        }
        const int cnt = min(ATC_T, p1 - (p0 + t * ATC_T));
        const int r0 = warp * 16;  // this warp's 16 positions of the tile
        if (r0 < cnt) {
            const uint32_t kb = sbase + (uint32_t)st * atm_stage_bytes<HD>(), vb = kb + KVB;
            // chunk c of row r in box c/8: swizzled to (c & 7) ^ (r & 7)
            auto kaddr = [&](int prow, int c) {
                return kb + (uint32_t)(c >> 3) * ATM_BOX + (uint32_t)prow * 128 + (uint32_t)(((c & 7) ^ (prow & 7)) << 4);
            };
            auto vaddr = [&](int prow, int c) {
                return vb + (uint32_t)(c >> 3) * ATM_BOX + (uint32_t)prow * 128 + (uint32_t)(((c & 7) ^ (prow & 7)) << 4);
            };
            atc_block_impl<HD>(qa, kaddr, vaddr, r0, cnt, m_run, l_run, o);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(b_empty + 8 * st);  // this warp is done with the stage
    }
    // every stage's copies have landed (each consumer waited for every tile)
    consumer_sync();
    atc_finish<HD, REP>(a, b, g, s, m_run, l_run, o, reinterpret_cast<float *>(smraw + (sbase - smem_u32(smraw))), s_m,
                        s_l, s_fm, s_fl, &s_last);
}

template <int HD, int REP, bool FUSED>
int atm_inst_k(const AttnArgs &a, cudaStream_t st, bool pdl) {
    constexpr size_t smem = atm_smem_bytes<HD>();
    static_assert((size_t)ATC_WARPS * REP * HD * 4 + 1024 <= smem, "combine buffer must fit the stages");
    auto kern = attn_tc_tma_kernel<HD, REP, FUSED>;
    static int limit[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!limit[dev & 63]) SB_TRY(allow_max_dynamic_smem(kern, &limit[dev & 63]));  // once, before any capture
    SB_CHECK(smem <= (size_t)limit[dev & 63], SB_ERR_SHAPE, "attention: needs %zu B shared memory (limit %d)", smem,
             limit[dev & 63]);
    SB_CUDA_TRY(launch(kern, dim3(a.n_kv, a.n_splits, a.B), dim3(ATC_THREADS + 32), smem, st, pdl, a));
    return SB_OK;
}

template <int HD, int REP>
int atm_inst(const AttnArgs &a, cudaStream_t st, bool pdl) {
    if (a.qkv_sums) {
        SB_CHECK(a.n_splits == 1 && a.shift && a.rstd && a.rope_cos && a.rope_sin && a.max_pos > 0, SB_ERR_ARG,
                 "attention: the fused q|k|v epilogue needs one split and the projection's scratch");
        return atm_inst_k<HD, REP, true>(a, st, pdl);
    }
    return atm_inst_k<HD, REP, false>(a, st, pdl);
}

template <int HD>
int atm_rep(const AttnArgs &a, cudaStream_t st, bool pdl) {
    switch (a.n_heads / a.n_kv) {
    case 2: return atm_inst<HD, 2>(a, st, pdl);
    case 4: return atm_inst<HD, 4>(a, st, pdl);
    case 8: return atm_inst<HD, 8>(a, st, pdl);
    default: return set_error(SB_ERR_UNSUPPORTED, "tensor-core attention: GQA ratio %d", a.n_heads / a.n_kv);
    }
}

template <int HD, int REP>
int atc_inst(const AttnArgs &a, cudaStream_t st, bool pdl) {
    constexpr size_t smem = atc_smem_bytes<HD, REP>();
    static_assert((size_t)ATC_WARPS * REP * HD * 4 <= smem, "combine buffer must fit the stages");
    auto kern = attn_tc_kernel<HD, REP>;
    static int limit[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!limit[dev & 63]) SB_TRY(allow_max_dynamic_smem(kern, &limit[dev & 63]));  // once, before any capture
    SB_CHECK(smem <= (size_t)limit[dev & 63], SB_ERR_SHAPE, "attention: needs %zu B shared memory (limit %d)", smem,
             limit[dev & 63]);
    SB_CUDA_TRY(launch(kern, dim3(a.n_kv, a.n_splits, a.B), dim3(ATC_THREADS), smem, st, pdl, a));
    return SB_OK;
}

template <int HD>
int atc_rep(const AttnArgs &a, cudaStream_t st, bool pdl) {
    switch (a.n_heads / a.n_kv) {
    case 2: return atc_inst<HD, 2>(a, st, pdl);
    case 4: return atc_inst<HD, 4>(a, st, pdl);
    case 8: return atc_inst<HD, 8>(a, st, pdl);
    default: return set_error(SB_ERR_UNSUPPORTED, "tensor-core attention: GQA ratio %d", a.n_heads / a.n_kv);
    }
}

}  // namespace

bool attn_tc_supported(const AttnArgs &a) {
    const int rep = a.n_kv > 0 ? a.n_heads / a.n_kv : 0;
    return !a.kv_f32 && (a.hd == 64 || a.hd == 128) && (rep == 2 || rep == 4 || rep == 8);
}

int attn_tc_error_peek(unsigned *host, cudaStream_t st) {
    SB_CUDA_TRY(cudaMemcpyFromSymbolAsync(host, atc_error_flag, sizeof(unsigned), 0, cudaMemcpyDeviceToHost, st));
    return SB_OK;
}

int attn_tc_check_error() {
    unsigned f = 0;
    SB_CUDA_TRY(cudaMemcpyFromSymbol(&f, atc_error_flag, sizeof f));
    if (f) {
        const unsigned zero = 0;
        cudaMemcpyToSymbol(atc_error_flag, &zero, sizeof zero);
        return set_error(SB_ERR_TIMEOUT, "attention: a bounded pipeline wait timed out");
    }
    return SB_OK;
}

int attn_make_tensor_map(CUtensorMap *map, const void *base, long long rows, int hd) {
    using EncodeFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
    static EncodeFn encode = nullptr;
    if (!encode) {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        SB_CUDA_TRY(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
        SB_CHECK(fn && q == cudaDriverEntryPointSuccess, SB_ERR_UNSUPPORTED, "cuTensorMapEncodeTiled unavailable");
        encode = reinterpret_cast<EncodeFn>(fn);
    }
    SB_CHECK(hd % 64 == 0 && rows > 0 && rows < (1LL << 31), SB_ERR_SHAPE, "attention tensor map: %lld rows of %d", rows,
             hd);
    SB_CHECK((reinterpret_cast<uintptr_t>(base) & 15) == 0, SB_ERR_ARG, "attention tensor map: unaligned cache");
    const cuuint64_t dims[2] = {(cuuint64_t)hd, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)hd * 2};
    const cuuint32_t box[2] = {64, 64}, estr[2] = {1, 1};
    const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box,
                              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    SB_CHECK(r == CUDA_SUCCESS, SB_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
    return SB_OK;
}

int attn_tc_launch(const AttnArgs &a, cudaStream_t st, bool pdl) {
    if (a.tma && a.page_size % ATC_T == 0) return a.hd == 128 ? atm_rep<128>(a, st, pdl) : atm_rep<64>(a, st, pdl);
    if (a.hd == 128) return atc_rep<128>(a, st, pdl);
    return atc_rep<64>(a, st, pdl);
}

}  // namespace sb
