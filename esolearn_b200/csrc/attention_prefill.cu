// Causal attention of a prefill chunk on the tensor cores: every row of the
// chunk is one prompt position of the same sequence, so each K/V tile is read
// once for all the rows that see it, instead of once per row as the decode
// attention does.  The batched form of the reference's full-sequence forward
// (llama.rs:683-700: QK^T over the prompt with the causal mask, softmax
// cpu.rs:336-366, AV), computed per position exactly as the decode step
// (llama.rs:414-456) would: row r attends to positions 0..pos[r].
//
// CTA (q head h, block of 16 rows): the 16 query rows are the A operand of
// mma.sync m16n8k16, once as bf16 high parts and once as bf16 low parts
// (q = hi + lo to about 2^-17; bf16 products are exact in f32), so
// S = hi(Q) K^T + lo(Q) K^T in f32 (the two products accumulate apart);
// P V likewise.  K/V tiles of 64 positions stream through a 3-stage cp.async
// ring into padded rows (a tile inside one page is one contiguous run of
// rows, so its addresses need a single page lookup); each of the 4 warps
// takes 16 positions of every tile and keeps its own online softmax per row
// (running max, sum, unnormalised output), and the warps are combined in
// warp order at the end.  Positions past a row's own position get
// probability 0; rows past the chunk are skipped.
#include "attention.cuh"

#include <algorithm>

#include "mma_bf16.cuh"
#include "pipeline.cuh"

namespace sb {

namespace {

constexpr int APF_T = 64;     // positions per tile (4 blocks of 16)
constexpr int APF_ROWS = 16;  // query rows per CTA
constexpr int APF_NST = 3;

template <int HD>
constexpr int apf_row() {
    return HD + 8;  // bf16 elements per padded row (conflict-free ldmatrix)
}
template <int HD>
constexpr size_t apf_stage_bytes() {
    return (size_t)2 * APF_T * apf_row<HD>() * 2;  // K and V
}
constexpr int APF_WARPS = 4;
constexpr int APF_THREADS = APF_WARPS * 32;
template <int HD>
constexpr size_t apf_smem_bytes() {
    // the ring, reused after the loop for the warps' [16][HD] outputs
    return APF_NST * apf_stage_bytes<HD>() > (size_t)APF_WARPS * APF_ROWS * HD * 4
               ? APF_NST * apf_stage_bytes<HD>()
               : (size_t)APF_WARPS * APF_ROWS * HD * 4;
}

// A fragments of the 16 query rows [r0, r0+16) of head h: hi and lo parts.
template <int HD>
__device__ __forceinline__ void apf_load_q(const PrefillAttnArgs &a, int h, int r0, uint32_t (&qh)[HD / 16][4],
                                           uint32_t (&ql)[HD / 16][4]) {
    const int lane = threadIdx.x & 31, grp = lane >> 2, qd = lane & 3;
    const int ld = a.n_heads * HD;
    const int ra = r0 + grp, rb = r0 + grp + 8;
    const float *qa = a.q + (size_t)ra * ld + (size_t)h * HD;
    const float *qb = a.q + (size_t)rb * ld + (size_t)h * HD;
    const bool va = ra < a.M, vb = rb < a.M;
#pragma unroll
    for (int ks = 0; ks < HD / 16; ks++) {
        float x[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (va) {
            const float2 u = *reinterpret_cast<const float2 *>(qa + ks * 16 + 2 * qd);
            const float2 v = *reinterpret_cast<const float2 *>(qa + ks * 16 + 8 + 2 * qd);
            x[0] = u.x, x[1] = u.y, x[4] = v.x, x[5] = v.y;
        }
        if (vb) {
            const float2 u = *reinterpret_cast<const float2 *>(qb + ks * 16 + 2 * qd);
            const float2 v = *reinterpret_cast<const float2 *>(qb + ks * 16 + 8 + 2 * qd);
            x[2] = u.x, x[3] = u.y, x[6] = v.x, x[7] = v.y;
        }
        __nv_bfloat16 hi[8], lo[8];
#pragma unroll
        for (int i = 0; i < 8; i++) split_bf16(x[i], hi[i], lo[i]);
        // a0: (row grp, k 2qd..), a1: (row grp+8, k 2qd..), a2: (grp, k 8+2qd..), a3: (grp+8, k 8+2qd..)
#pragma unroll
        for (int f = 0; f < 4; f++) {
            qh[ks][f] = pack_bf16(hi[2 * f], hi[2 * f + 1]);
            ql[ks][f] = pack_bf16(lo[2 * f], lo[2 * f + 1]);
        }
    }
}

// One warp's 16 positions [pr0, pr0+16) of the tile whose first position is
// base; the tile's K and V rows are at byte addresses ks / vs (padded rows).
// The thread's two query rows (grp, grp+8) see positions <= lim[0], lim[1].
template <int HD>
__device__ __forceinline__ void apf_block(const uint32_t (&qh)[HD / 16][4], const uint32_t (&ql)[HD / 16][4],
                                          uint32_t ks, uint32_t vs, int pr0, int base, const int (&lim)[2],
                                          float (&m_run)[2], float (&l_run)[2], float (&o)[HD / 8][4]) {
    constexpr int KSTEPS = HD / 16, NB = HD / 8, RW = apf_row<HD>();
    const int lane = threadIdx.x & 31, qd = lane & 3;
    const int mi = lane >> 3, ri = lane & 7;
    // S blocks: c[nb] = scores of positions pr0 + nb*8 + (2qd, 2qd+1), rows grp (0,1) and grp+8 (2,3);
    // the hi and lo products accumulate apart (four independent MMA chains) and are added once
    float c[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    float cl[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    {
        const int prow = pr0 + (mi >> 1) * 8 + ri;  // matrices: (pos 0-7, d), (0-7, d+8), (8-15, d), (8-15, d+8)
#pragma unroll
        for (int k = 0; k < KSTEPS; k++) {
            uint32_t b0, b1, b2, b3;
            ldsm_x4(ks + (uint32_t)((prow * RW + (2 * k + (mi & 1)) * 8) * 2), b0, b1, b2, b3);
            mma_bf16(c[0], qh[k], b0, b1);
            mma_bf16(cl[0], ql[k], b0, b1);
            mma_bf16(c[1], qh[k], b2, b3);
            mma_bf16(cl[1], ql[k], b2, b3);
        }
#pragma unroll
        for (int nb = 0; nb < 2; nb++)
#pragma unroll
            for (int e = 0; e < 4; e++) c[nb][e] = __fadd_rn(c[nb][e], cl[nb][e]);
    }
    float sc[2][2][2];  // [row][nb][e]
#pragma unroll
    for (int nb = 0; nb < 2; nb++)
#pragma unroll
        for (int e = 0; e < 2; e++) {
            const int p = base + pr0 + nb * 8 + 2 * qd + e;
            sc[0][nb][e] = p <= lim[0] ? c[nb][e] : -INFINITY;
            sc[1][nb][e] = p <= lim[1] ? c[nb][2 + e] : -INFINITY;
        }
    float alpha[2];
    float p[2][2][2];
#pragma unroll
    for (int r = 0; r < 2; r++) {
        float mx = fmaxf(fmaxf(sc[r][0][0], sc[r][0][1]), fmaxf(sc[r][1][0], sc[r][1][1]));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
        const float m_new = fmaxf(m_run[r], mx);
        alpha[r] = m_run[r] == -INFINITY ? 0.f : expf(m_run[r] - m_new);
        m_run[r] = m_new;
        float psum = 0.f;
#pragma unroll
        for (int nb = 0; nb < 2; nb++)
#pragma unroll
            for (int e = 0; e < 2; e++) {
                p[r][nb][e] = sc[r][nb][e] == -INFINITY ? 0.f : expf(sc[r][nb][e] - m_new);
                psum += p[r][nb][e];
            }
        l_run[r] = fmaf(l_run[r], alpha[r], psum);
    }
#pragma unroll
    for (int j = 0; j < NB; j++) {
        o[j][0] *= alpha[0], o[j][1] *= alpha[0];
        o[j][2] *= alpha[1], o[j][3] *= alpha[1];
    }
    // P as the A operand of O = P V (k = the 16 positions): hi and lo parts
    uint32_t ph[4], pl[4];
    {
        __nv_bfloat16 hi[2][2][2], lo[2][2][2];
#pragma unroll
        for (int r = 0; r < 2; r++)
#pragma unroll
            for (int nb = 0; nb < 2; nb++)
#pragma unroll
                for (int e = 0; e < 2; e++) split_bf16(p[r][nb][e], hi[r][nb][e], lo[r][nb][e]);
        // a0: (row grp, pos 2qd..), a1: (grp+8, 2qd..), a2: (grp, 8+2qd..), a3: (grp+8, 8+2qd..)
#pragma unroll
        for (int f = 0; f < 4; f++) {
            const int r = f & 1, nb = f >> 1;
            ph[f] = pack_bf16(hi[r][nb][0], hi[r][nb][1]);
            pl[f] = pack_bf16(lo[r][nb][0], lo[r][nb][1]);
        }
    }
    {
        // matrices: (pos 0-7, d), (pos 8-15, d), (pos 0-7, d+8), (pos 8-15, d+8)
        const int prow = pr0 + (mi & 1) * 8 + ri;
#pragma unroll
        for (int j = 0; j < NB; j += 2) {
            uint32_t b0, b1, b2, b3;
            ldsm_x4_t(vs + (uint32_t)((prow * RW + (j + (mi >> 1)) * 8) * 2), b0, b1, b2, b3);
            mma_bf16(o[j], ph, b0, b1);
            mma_bf16(o[j], pl, b0, b1);
            mma_bf16(o[j + 1], ph, b2, b3);
            mma_bf16(o[j + 1], pl, b2, b3);
        }
    }
}

template <int HD>
__global__ void __launch_bounds__(APF_THREADS) attn_prefill_kernel(const PrefillAttnArgs a) {
    constexpr int RW = apf_row<HD>();
    constexpr int NB = HD / 8;
    constexpr int CPR = HD / 8;  // 16-byte chunks per K/V row
    extern __shared__ __align__(1024) uint8_t smraw[];
    __shared__ float s_m[APF_WARPS][APF_ROWS], s_l[APF_WARPS][APF_ROWS];
    __shared__ float s_fm[APF_ROWS], s_fl[APF_ROWS];
    __shared__ int s_pos[APF_ROWS];

    const int h = blockIdx.x, r0 = blockIdx.y * APF_ROWS;
    const int g = h / (a.n_heads / a.n_kv);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int grp = lane >> 2, qd = lane & 3;

    pdl_launch_dependents();
    pdl_wait();

    // rows past the chunk, or at a position outside the cache, see nothing
    const int cap = a.max_pages * a.page_size;
    if (tid < APF_ROWS) {
        const int r = r0 + tid;
        const int p = r < a.M ? a.pos[r] : -1;
        s_pos[tid] = (p >= 0 && p < cap) ? p : -1;
    }
    __syncthreads();
    int jmax = -1;
#pragma unroll
    for (int i = 0; i < APF_ROWS; i++) jmax = max(jmax, s_pos[i]);
    const int lim[2] = {s_pos[grp], s_pos[grp + 8]};
    const int ntiles = (jmax + APF_T) / APF_T;  // positions 0..jmax

    uint32_t qh[HD / 16][4], ql[HD / 16][4];
    apf_load_q<HD>(a, h, r0, qh, ql);

    const __nv_bfloat16 *kc = reinterpret_cast<const __nv_bfloat16 *>(a.kc);
    const __nv_bfloat16 *vc = reinterpret_cast<const __nv_bfloat16 *>(a.vc);
    const uint32_t sbase = smem_u32(smraw);
    const bool aligned = a.page_size % APF_T == 0;  // every tile lies inside one page
    // K and V rows of tile t into stage st (16-byte async copies, padded rows)
    auto issue = [&](int t, int st) {
        const int base = t * APF_T;
        const int cnt = min(APF_T, jmax + 1 - base);
        const uint32_t kdst = sbase + (uint32_t)(st * apf_stage_bytes<HD>());
        const uint32_t vdst = kdst + (uint32_t)(APF_T * RW * 2);
        if (aligned) {
            const int page = a.page_table[base / a.page_size], slot0 = base % a.page_size;
            const size_t off0 = (((size_t)page * a.n_kv + g) * a.page_size + slot0) * HD;
            for (int c = tid; c < cnt * CPR; c += APF_THREADS) {
                const int i = c / CPR, sub = c % CPR;
                const size_t off = off0 + (size_t)i * HD + sub * 8;
                const uint32_t so = (uint32_t)((i * RW + sub * 8) * 2);
                cp_async16(kdst + so, kc + off);
                cp_async16(vdst + so, vc + off);
            }
        } else {
            for (int c = tid; c < cnt * CPR; c += APF_THREADS) {
                const int i = c / CPR, sub = c % CPR;
                const int p = base + i;
                const int page = a.page_table[p / a.page_size], slot = p % a.page_size;
                const size_t off = (((size_t)page * a.n_kv + g) * a.page_size + slot) * HD + sub * 8;
                const uint32_t so = (uint32_t)((i * RW + sub * 8) * 2);
                cp_async16(kdst + so, kc + off);
                cp_async16(vdst + so, vc + off);
            }
        }
        // rows past jmax are multiplied by probability 0: zero them, since
        // 0 * (stale NaN or Inf) would poison the sums
        for (int c = cnt * CPR + tid; c < APF_T * CPR; c += APF_THREADS) {
            const int i = c / CPR, sub = c % CPR;
            const uint32_t so = (uint32_t)((i * RW + sub * 8) * 2);
            asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};" ::"r"(kdst + so), "r"(0u) : "memory");
            asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};" ::"r"(vdst + so), "r"(0u) : "memory");
        }
    };

    float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
    float o[NB][4];
#pragma unroll
    for (int j = 0; j < NB; j++) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;

#pragma unroll
    for (int t = 0; t < APF_NST - 1; t++) {
        if (t < ntiles) issue(t, t);
        cp_commit();
    }
    for (int t = 0; t < ntiles; t++) {
        cp_wait<APF_NST - 2>();
        __syncthreads();  // tile t landed for every thread; stage (t-1) % NST is free
        if (t + APF_NST - 1 < ntiles) issue(t + APF_NST - 1, (t + APF_NST - 1) % APF_NST);
        cp_commit();
        const uint32_t ks = sbase + (uint32_t)((t % APF_NST) * apf_stage_bytes<HD>());
        apf_block<HD>(qh, ql, ks, ks + (uint32_t)(APF_T * RW * 2), warp * 16, t * APF_T, lim, m_run, l_run, o);
    }
    cp_wait<0>();
    __syncthreads();  // the ring becomes the warps' output rows

    // combine the warps in warp order: (m, l) per row, then the outputs
    float *wo = reinterpret_cast<float *>(smraw);  // [warp][row][HD]
#pragma unroll
    for (int r = 0; r < 2; r++) {
        l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 1);
        l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 2);
    }
    if (qd == 0) {
        s_m[warp][grp] = m_run[0], s_l[warp][grp] = l_run[0];
        s_m[warp][grp + 8] = m_run[1], s_l[warp][grp + 8] = l_run[1];
    }
#pragma unroll
    for (int j = 0; j < NB; j++) {
        const int d = j * 8 + 2 * qd;
        float *ra = wo + ((size_t)warp * APF_ROWS + grp) * HD, *rb = ra + 8 * HD;
        ra[d] = o[j][0], ra[d + 1] = o[j][1];
        rb[d] = o[j][2], rb[d + 1] = o[j][3];
    }
    __syncthreads();
    if (tid < APF_ROWS) {
        float M = -INFINITY;
        for (int w = 0; w < APF_WARPS; w++) M = fmaxf(M, s_m[w][tid]);
        float L = 0.f;
        if (M != -INFINITY)
            for (int w = 0; w < APF_WARPS; w++)
                if (s_m[w][tid] != -INFINITY) L = fmaf(s_l[w][tid], expf(s_m[w][tid] - M), L);
        s_fm[tid] = M, s_fl[tid] = L;
    }
    __syncthreads();
    const size_t ld = (size_t)a.n_heads * HD;
    for (int i = tid; i < APF_ROWS * HD; i += APF_THREADS) {
        const int r = i / HD, d = i - r * HD;
        if (s_pos[r] < 0) continue;
        const float M = s_fm[r];
        float O = 0.f;
        for (int w = 0; w < APF_WARPS; w++)
            if (s_m[w][r] != -INFINITY) O = fmaf(wo[((size_t)w * APF_ROWS + r) * HD + d], expf(s_m[w][r] - M), O);
        a.out[(size_t)(r0 + r) * ld + (size_t)h * HD + d] = s_fl[r] > 0.f ? O / s_fl[r] : 0.f;
    }
}

template <int HD>
int apf_launch(const PrefillAttnArgs &a, cudaStream_t st, bool pdl) {
    static int done[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    constexpr size_t smem = apf_smem_bytes<HD>();
    if (!done[dev & 63]) {
        SB_CUDA_TRY(cudaFuncSetAttribute(attn_prefill_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        done[dev & 63] = 1;
    }
    SB_CUDA_TRY(launch(attn_prefill_kernel<HD>, dim3(a.n_heads, ceil_div(a.M, APF_ROWS)), dim3(APF_THREADS), smem, st,
                       pdl, a));
    return SB_OK;
}

}  // namespace

bool attn_prefill_supported(int hd, int kv_f32) { return !kv_f32 && (hd == 64 || hd == 128); }

int attn_prefill_launch(const PrefillAttnArgs &a, cudaStream_t st, bool pdl) {
    SB_CHECK(attn_prefill_supported(a.hd, a.kv_f32), SB_ERR_UNSUPPORTED,
             "prefill attention: head_dim %d, %s cache", a.hd, a.kv_f32 ? "f32" : "bf16");
    SB_CHECK(a.q && a.kc && a.vc && a.page_table && a.pos && a.out && a.M >= 1 && a.n_kv >= 1 &&
                 a.n_heads % a.n_kv == 0 && a.page_size >= 1 && a.max_pages >= 1,
             SB_ERR_ARG, "prefill attention: bad arguments");
    if (a.hd == 128) return apf_launch<128>(a, st, pdl);
    return apf_launch<64>(a, st, pdl);
}

}  // namespace sb
