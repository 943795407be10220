// sample_token (generate.rs:92-165) on the device, one CTA per row of logits.
//
// The reference, per row of n logits x with temperature T, top_k, top_p:
//   T < 1e-8 -> argmax (ties -> last index), no random draw;
//   s = f64(x) / f64(T);
//   top_k in (0, n): thr = k-th largest s (with multiplicity), s < thr -> -inf;
//   e = exp(s - max s); p = e / sum(e) when sum > 0, else 1/n everywhere;
//   top_p in (0, 1): sort p descending, keep the shortest prefix whose running
//     sum reaches top_p, zero the rest, divide by their sum;
//   r = rng.f64() (fastrand wyrand); the token is the first i whose running
//     sum of p in index order exceeds r (n-1 when none does).
//
// Here:
// * the random stream is the reference's: each row keeps a 64-bit wyrand
//   state in device memory, advanced by one draw per sampled row, so the
//   draws equal the host's fastrand::Rng bit for bit;
// * top-k: f64 division by one positive T is strictly monotonic on f32
//   inputs, so the k-th largest s is the scaled k-th largest x, found by a
//   radix select over order-preserving 32-bit keys (four 8-bit passes,
//   integer histograms);
// * top-p: p >= 0, so its f64 bit pattern orders it.  A most-significant-
//   digit radix walk over those 64 bits (4 bits per pass) finds the value v
//   at which the descending running sum first reaches top_p: every pass sums
//   p per digit in per-thread registers and combines the threads in a fixed
//   order, so the cut is deterministic.  Elements above v are kept; of the
//   elements equal to v, as many as the running sum needs are kept, lowest
//   index first (the tie order of a stable descending sort);
// * sums run in a fixed tree order instead of the reference's left-to-right
//   order (and exp is CUDA's, within 1 ulp), so a token can differ from the
//   reference's only when r or top_p falls within f64 rounding of a running
//   sum.  NaN logits give an unspecified token (the reference's comparison
//   sort has no total order for them either).
//
// Scratch: one f64 per logit (the probabilities), row-major [rows][n].
#include "sampler.cuh"

namespace sb {
namespace {

constexpr int SP_THREADS = 512;
constexpr int SP_WARPS = SP_THREADS / 32;
constexpr uint64_t SP_WY0 = 0x2d358dccaa6c78a5ULL;
constexpr uint64_t SP_WY1 = 0x8bb84b93962eacc9ULL;

// fastrand::Rng::f64: advance the state by C0, mix, map the top 52 bits to [0, 1).
__device__ __forceinline__ double sp_rng_f64(uint64_t &state) {
    state += SP_WY0;
    const uint64_t t = state ^ SP_WY1;
    const uint64_t r = (state * t) ^ __umul64hi(state, t);
    return __longlong_as_double((long long)(0x3FF0000000000000ULL + (r >> 12))) - 1.0;
}

// Order-preserving key of a float (-0 and +0 compare equal, as in the reference).
__device__ __forceinline__ uint32_t sp_key(float x) {
    const uint32_t u = __float_as_uint(x == 0.f ? 0.f : x);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float sp_unkey(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

struct SpShared {
    double red[SP_WARPS + 1];
    double bin_s[SP_WARPS][16];
    unsigned bin_c[SP_WARPS][16];
    double seg[SP_THREADS];
    int ties[SP_THREADS];
    unsigned hist[256];
    float amax_v[SP_WARPS];
    int amax_i[SP_WARPS];
    unsigned long long prefix;
    double above;
    int k, chosen_count, keep_ties, token;
};

// Sum over the block in a fixed order: lane 0 of each warp holds its warp's
// shuffle tree, then thread 0 adds the warps in order.  Every thread returns it.
__device__ double sp_block_sum(double v, SpShared &sh) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int o = 16; o > 0; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
    if (lane == 0) sh.red[warp] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
        double s = 0.0;
        for (int w = 0; w < SP_WARPS; w++) s += sh.red[w];
        sh.red[SP_WARPS] = s;
    }
    __syncthreads();
    const double s = sh.red[SP_WARPS];
    __syncthreads();
    return s;
}

__device__ double sp_block_max(double v, SpShared &sh) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    for (int o = 16; o > 0; o >>= 1) v = fmax(v, __shfl_down_sync(0xffffffffu, v, o));
    if (lane == 0) sh.red[warp] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
        double s = -INFINITY;
        for (int w = 0; w < SP_WARPS; w++) s = fmax(s, sh.red[w]);
        sh.red[SP_WARPS] = s;
    }
    __syncthreads();
    const double s = sh.red[SP_WARPS];
    __syncthreads();
    return s;
}

// argmax with ties -> last index (generate.rs:167-173).
__device__ __forceinline__ void sp_amax_merge(float &v, int &i, float ov, int oi) {
    if (oi < 0) return;
    if (i < 0 || ov > v || (ov == v && oi > i)) v = ov, i = oi;
}

// One row: the token goes to *token_out (written by thread 0), the draw advances
// *rng_row.  Every thread of the CTA calls it; p is the row's scratch.
__device__ __forceinline__ void sp_sample_row(const float *__restrict__ x, int n, float temperature, int top_k,
                                              float top_p, uint64_t *__restrict__ rng_row, double *__restrict__ p,
                                              SpShared &sh, int *token_out) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

    if (temperature < 1e-8f) {  // greedy: no draw
        float v = -INFINITY;
        int idx = -1;
        for (int i = tid; i < n; i += SP_THREADS) sp_amax_merge(v, idx, x[i], i);
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, v, o);
            const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
            sp_amax_merge(v, idx, ov, oi);
        }
        if (lane == 0) sh.amax_v[warp] = v, sh.amax_i[warp] = idx;
        __syncthreads();
        if (tid == 0) {
            for (int w = 1; w < SP_WARPS; w++) sp_amax_merge(v, idx, sh.amax_v[w], sh.amax_i[w]);
            *token_out = idx < 0 ? 0 : idx;
        }
        return;
    }
    const double T = (double)temperature;

    // ---- top-k threshold: radix select of the k-th largest key
    const bool do_k = top_k > 0 && top_k < n;
    double thr = -INFINITY;
    if (do_k) {
        uint32_t prefix = 0, mask = 0;
        if (tid == 0) sh.k = top_k;
        for (int shift = 24; shift >= 0; shift -= 8) {
            for (int b = tid; b < 256; b += SP_THREADS) sh.hist[b] = 0;
            __syncthreads();
            for (int i = tid; i < n; i += SP_THREADS) {
                const uint32_t key = sp_key(x[i]);
                if ((key & mask) == prefix) atomicAdd(&sh.hist[(key >> shift) & 255u], 1u);
            }
            __syncthreads();
            if (tid == 0) {
                int k = sh.k, b = 255;
                for (; b > 0; b--) {
                    if ((int)sh.hist[b] >= k) break;
                    k -= (int)sh.hist[b];
                }
                sh.k = k;
                sh.prefix = prefix | ((uint32_t)b << shift);
            }
            __syncthreads();
            prefix = (uint32_t)sh.prefix;
            mask |= 255u << shift;
        }
        thr = (double)sp_unkey(prefix) / T;
    }

    // ---- softmax (f64): max, exp, sum, normalise
    double mx = -INFINITY;
    for (int i = tid; i < n; i += SP_THREADS) {
        double s = (double)x[i] / T;
        if (do_k && s < thr) s = -INFINITY;
        mx = fmax(mx, s);
    }
    mx = sp_block_max(mx, sh);
    double part = 0.0;
    for (int i = tid; i < n; i += SP_THREADS) {
        double s = (double)x[i] / T;
        if (do_k && s < thr) s = -INFINITY;
        const double e = exp(s - mx);
        p[i] = e;
        part += e;
    }
    const double sum = sp_block_sum(part, sh);
    const bool normal = sum > 0.0;
    const double uni = 1.0 / (double)n;
    for (int i = tid; i < n; i += SP_THREADS) p[i] = normal ? p[i] / sum : uni;
    __syncthreads();

    // contiguous index segment of this thread (index-order phases)
    const int seg = (n + SP_THREADS - 1) / SP_THREADS;
    const int i0 = min(n, tid * seg), i1 = min(n, i0 + seg);

    // ---- top-p: radix walk over the probability bits, most significant first
    if (top_p < 1.0f && top_p > 0.0f) {
        const double tp = (double)top_p;
        unsigned long long prefix = 0, mask = 0;
        double above = 0.0;  // sum of p over elements above the current bucket
        bool cut = true;
        int count = 0;       // elements in the current bucket
        for (int shift = 60; shift >= 0; shift -= 4) {
            double s16[16];
            unsigned c16[16];
#pragma unroll
            for (int b = 0; b < 16; b++) s16[b] = 0.0, c16[b] = 0;
            for (int i = tid; i < n; i += SP_THREADS) {
                const double v = p[i];
                const unsigned long long key = (unsigned long long)__double_as_longlong(v);
                if ((key & mask) == prefix) {
                    const int d = (int)((key >> shift) & 15ull);
#pragma unroll
                    for (int b = 0; b < 16; b++)
                        if (d == b) s16[b] += v, c16[b]++;
                }
            }
#pragma unroll
            for (int b = 0; b < 16; b++) {
                double s = s16[b];
                unsigned c = c16[b];
                for (int o = 16; o > 0; o >>= 1) {
                    s += __shfl_down_sync(0xffffffffu, s, o);
                    c += __shfl_down_sync(0xffffffffu, c, o);
                }
                if (lane == 0) sh.bin_s[warp][b] = s, sh.bin_c[warp][b] = c;
            }
            __syncthreads();
            if (tid == 0) {
                double S[16];
                unsigned Cn[16];
                for (int b = 0; b < 16; b++) {
                    double s = 0.0;
                    unsigned c = 0;
                    for (int w = 0; w < SP_WARPS; w++) s += sh.bin_s[w][b], c += sh.bin_c[w][b];
                    S[b] = s, Cn[b] = c;
                }
                int chosen = -1, lowest = -1;
                double lowest_above = above;
                for (int b = 15; b >= 0; b--) {
                    if (Cn[b] == 0) continue;
                    if (above + S[b] >= tp) {
                        chosen = b;
                        break;
                    }
                    lowest = b, lowest_above = above;
                    above += S[b];
                }
                if (chosen < 0) {
                    if (shift == 60) {
                        sh.chosen_count = -1;  // the running sum never reaches top_p: keep all
                    } else {
                        // the bucket reached top_p as a whole; rounding of the
                        // digit sums missed it: its last digit holds the cut
                        chosen = lowest;
                        above = lowest_above;
                    }
                }
                if (chosen >= 0) {
                    sh.prefix = prefix | ((unsigned long long)chosen << shift);
                    sh.chosen_count = (int)Cn[chosen];
                }
                sh.above = above;
            }
            __syncthreads();
            if (sh.chosen_count < 0) {
                cut = false;
                break;
            }
            prefix = sh.prefix;
            mask |= 15ull << shift;
            above = sh.above;
            count = sh.chosen_count;
            __syncthreads();
        }
        if (cut) {
            // prefix = bits of the cut value v; `count` elements equal v.
            const double v = __longlong_as_double((long long)prefix);
            if (tid == 0) {
                int j = 0;
                double cum = above;
                if (v > 0.0) {
                    const double need = floor((tp - above) / v) - 2.0;
                    if (need > 0.0) j = (int)fmin(need, (double)count);
                    cum = above + (double)j * v;
                }
                while (j < count) {
                    cum += v;
                    j++;
                    if (cum >= tp) break;
                }
                sh.keep_ties = j;
            }
            // rank of each tied element in index order
            int t = 0;
            for (int i = i0; i < i1; i++) t += (unsigned long long)__double_as_longlong(p[i]) == prefix;
            sh.ties[tid] = t;
            __syncthreads();
            if (tid == 0) {
                int run = 0;
                for (int w = 0; w < SP_THREADS; w++) {
                    const int c = sh.ties[w];
                    sh.ties[w] = run;
                    run += c;
                }
            }
            __syncthreads();
            const int keep = sh.keep_ties;
            int rank = sh.ties[tid];
            double kept = 0.0;
            for (int i = i0; i < i1; i++) {
                const double q = p[i];
                const unsigned long long key = (unsigned long long)__double_as_longlong(q);
                bool k = key > prefix;
                if (key == prefix) k = rank++ < keep;
                if (!k) p[i] = 0.0;
                else kept += q;
            }
            const double sum2 = sp_block_sum(kept, sh);
            if (sum2 > 0.0)
                for (int i = i0; i < i1; i++) p[i] = p[i] / sum2;
            __syncthreads();
        }
    }

    // ---- weighted_sample (generate.rs:175-185) in index order
    double ssum = 0.0;
    for (int i = i0; i < i1; i++) ssum += p[i];
    sh.seg[tid] = ssum;
    __syncthreads();
    if (tid == 0) {
        uint64_t st = *rng_row;
        const double r = sp_rng_f64(st);
        *rng_row = st;
        int token = n - 1;
        double cum = 0.0;
        int w = 0;
        for (; w < SP_THREADS; w++) {
            if (r < cum + sh.seg[w]) break;
            cum += sh.seg[w];
        }
        // walk from the segment where the running sum passes r
        bool found = false;
        for (int i = min(n, w * seg); i < n && !found; i++) {
            cum += p[i];
            if (r < cum) token = i, found = true;
        }
        *token_out = token;
    }
}

__global__ void __launch_bounds__(SP_THREADS) sample_rows_kernel(const float *__restrict__ logits, int n, int ld,
                                                                 float temperature, int top_k, float top_p,
                                                                 uint64_t *__restrict__ rng, double *__restrict__ prob,
                                                                 int *__restrict__ out) {
    __shared__ SpShared sh;
    const int row = blockIdx.x;
    sp_sample_row(logits + (size_t)row * ld, n, temperature, top_k, top_p, rng + row, prob + (size_t)row * n, sh,
                  out + row);
}

// The token step of a sampled decode loop (generate.rs:68-86), row b per CTA:
// while b is inside its prompt (pos < prompt_len - 1) nothing is drawn and
// the next step reads the prompt; from the last prompt position on, the
// token is sampled from this step's logits, recorded and fed to the next
// step, until max_draws tokens were drawn (later steps draw nothing and feed
// token 0).  The position always advances.
__global__ void __launch_bounds__(SP_THREADS) sample_step_kernel(const float *__restrict__ logits, int n, int ld,
                                                                 SampleCfg c, uint64_t *__restrict__ rng,
                                                                 double *__restrict__ prob, SeqState s) {
    __shared__ SpShared sh;
    __shared__ int tok;
    const int b = blockIdx.x;
    const int pos = s.pos[b], plen = s.prompt_len ? s.prompt_len[b] : 0, g = s.ngen[b];
    // uniform over the CTA; a step at position -1 (a graph capture's warm-up) draws nothing
    const bool draw = pos >= 0 && pos >= plen - 1 && g < c.max_draws;
    if (draw)
        sp_sample_row(logits + (size_t)b * ld, n, c.temperature, c.top_k, c.top_p, rng + b, prob + (size_t)b * n, sh,
                      &tok);
    __syncthreads();
    if (threadIdx.x == 0) {
        const int next = draw ? tok : 0;
        if (draw) {
            s.last[b] = next;
            if (g < s.max_gen) s.out[(size_t)b * s.max_gen + g] = next;
            s.ngen[b] = g + 1;
        }
        s.tok[b] = next;
        s.pos[b] = pos + 1;
    }
}

}  // namespace

int sample_step_launch(const float *logits, int rows, int n, int ld, const SampleCfg &c, uint64_t *rng, double *prob,
                       const SeqState &s, cudaStream_t st) {
    if (rows <= 0) return SB_OK;
    sample_step_kernel<<<rows, SP_THREADS, 0, st>>>(logits, n, ld, c, rng, prob, s);
    SB_CUDA_TRY(cudaGetLastError());
    return SB_OK;
}

int sample_rows_launch(const float *logits, int rows, int n, int ld, float temperature, int top_k, float top_p,
                       uint64_t *rng, double *prob, int *out, cudaStream_t st) {
    if (rows <= 0) return SB_OK;
    sample_rows_kernel<<<rows, SP_THREADS, 0, st>>>(logits, n, ld, temperature, top_k, top_p, rng, prob, out);
    SB_CUDA_TRY(cudaGetLastError());
    return SB_OK;
}

}  // namespace sb
