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
#include "pipeline.cuh"

namespace sb {

namespace {

constexpr int ATC_THREADS = 128;
constexpr int ATC_WARPS = ATC_THREADS / 32;
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

__device__ __forceinline__ void cp_async16(uint32_t dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
// D += A(16x16 bf16, row) * B(16x8 bf16, col), f32 accumulate.
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// bf16 pair (lo element in the low half) and the hi/lo split of an f32.
__device__ __forceinline__ uint32_t pack_bf16(__nv_bfloat16 lo, __nv_bfloat16 hi) {
    return (uint32_t)__bfloat16_as_ushort(lo) | ((uint32_t)__bfloat16_as_ushort(hi) << 16);
}
__device__ __forceinline__ void split_bf16(float x, __nv_bfloat16 &hi, __nv_bfloat16 &lo) {
    hi = __float2bfloat16_rn(x);
    lo = __float2bfloat16_rn(__fsub_rn(x, __bfloat162float(hi)));
}

template <int HD, int REP>
__global__ void __launch_bounds__(ATC_THREADS) attn_tc_kernel(const AttnArgs a) {
    static_assert(REP == 2 || REP == 4 || REP == 8, "tensor-core attention takes 2, 4 or 8 heads per group");
    constexpr int RW = atc_row<HD>();
    constexpr int KSTEPS = HD / 16;  // k steps of the score MMA
    constexpr int NB = HD / 8;       // 8-column output blocks of the AV MMA
    constexpr int CPR = HD / 8;      // 16-byte chunks per K/V row

    extern __shared__ __align__(16) uint8_t smraw[];
    __shared__ float s_m[ATC_WARPS][REP], s_l[ATC_WARPS][REP];
    __shared__ float s_fm[REP], s_fl[REP];
    __shared__ int s_last;

    const int g = blockIdx.x, s = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int grp = lane >> 2, qd = lane & 3;  // MMA row group (head) and column pair
    const int qdim = a.n_heads * HD;

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

    // Query fragments (A operand of S = Q K^T): row grp = hi(q), row grp+8 = lo(q).
    uint32_t qa[KSTEPS][4];
    {
        const float *q = a.q + (size_t)b * qdim + ((size_t)g * REP + grp) * HD;
        const bool live = grp < REP;
#pragma unroll
        for (int ks = 0; ks < KSTEPS; ks++) {
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

        // S^T blocks: c[nb] = scores of positions r0 + nb*8 + (2qd, 2qd+1), hi rows + lo rows
        float c[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        {
            const int mi = lane >> 3, ri = lane & 7;
            const int prow = r0 + (mi >> 1) * 8 + ri;  // matrices: (pos 0-7, d), (0-7, d+8), (8-15, d), (8-15, d+8)
            const uint32_t rowaddr = kb + (uint32_t)((prow * RW + (mi & 1) * 8) * 2);
#pragma unroll
            for (int ks = 0; ks < KSTEPS; ks++) {
                uint32_t b0, b1, b2, b3;
                ldsm_x4(rowaddr + ks * 32, b0, b1, b2, b3);
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
            const int mi = lane >> 3, ri = lane & 7;
            // matrices: (pos 0-7, d), (pos 8-15, d), (pos 0-7, d+8), (pos 8-15, d+8)
            const int prow = r0 + (mi & 1) * 8 + ri;
            const uint32_t rowaddr = vb + (uint32_t)((prow * RW + (mi >> 1) * 8) * 2);
#pragma unroll
            for (int j = 0; j < NB; j += 2) {
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(rowaddr + j * 16, b0, b1, b2, b3);
                mma_bf16(o[j], pa, b0, b1);
                mma_bf16(o[j + 1], pa, b2, b3);
            }
        }
    }
    cp_wait<0>();
    __syncthreads();  // every warp is done with the stages: reuse them for the combine

    // ---- combine the warps: head grp's output d = 8j + 2qd + e is o[j][e] + o[j][2+e]
    float *wo = reinterpret_cast<float *>(smraw);  // [ATC_WARPS][REP][HD]
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
    __syncthreads();
    if (tid < REP) {
        float M = -INFINITY;
        for (int w = 0; w < ATC_WARPS; w++) M = fmaxf(M, s_m[w][tid]);
        float L = 0.f;
        if (M != -INFINITY)
            for (int w = 0; w < ATC_WARPS; w++)
                if (s_m[w][tid] != -INFINITY) L = fmaf(s_l[w][tid], expf(s_m[w][tid] - M), L);
        s_fm[tid] = M, s_fl[tid] = L;
    }
    __syncthreads();
    const size_t hbase = (size_t)b * a.n_heads + (size_t)g * REP;  // first q head of the group
    const int stride = HD + 2;
    for (int i = tid; i < REP * HD; i += ATC_THREADS) {
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
    // ---- the last CTA of (sequence, kv head) combines the splits in split order
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        unsigned *cntr = a.counters + (size_t)b * a.n_kv + g;
        const unsigned prev = atomicAdd(cntr, 1u);
        s_last = (prev == (unsigned)a.n_splits - 1);
        if (s_last) *cntr = 0u;  // ready for the next launch
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int i = tid; i < REP * HD; i += ATC_THREADS) {
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

int attn_tc_launch(const AttnArgs &a, cudaStream_t st, bool pdl) {
    if (a.hd == 128) return atc_rep<128>(a, st, pdl);
    return atc_rep<64>(a, st, pdl);
}

}  // namespace sb
