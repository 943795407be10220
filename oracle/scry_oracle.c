/*
 * scry_oracle.c -- CPU restatement of scry-llm's int8 Llama decode path.
 *
 * TEST INFRASTRUCTURE ONLY (the parity checker and the timed CPU baseline);
 * the B200 product never links it.  See scry_oracle.h for the contract.
 *
 * Build: oracle/Makefile (gcc -O3 -ffp-contract=off -fopenmp; hot loops cloned per ISA).  Contraction
 * must stay off: the reference is Rust, which rounds every f32/f64 multiply
 * and add separately.  Parallel loops split work only across independent
 * output elements, so every element is summed in the reference's order and
 * the results do not depend on the thread count.
 */
#include "scry_oracle.h"

#include <math.h>
#include <omp.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------------ */
/* fastrand 2.3.0 wyrand.  Reference use: nn/init.rs:2-14 (Rng::f64),       */
/* generate.rs:155-165 (weighted_sample).  Crate source is not vendored in   */
/* the reference; this follows the crate's published algorithm: the state    */
/* advances by a fixed odd constant and the output is the xor-fold of a      */
/* 64x64->128 multiply (wyhash v4.2 constants).                              */
/* ------------------------------------------------------------------------ */
#define WY0 0x2d358dccaa6c78a5ULL
#define WY1 0x8bb84b93962eacc9ULL

static inline uint64_t wy_mix(uint64_t s) {
    unsigned __int128 t = (unsigned __int128)s * (unsigned __int128)(s ^ WY1);
    return (uint64_t)t ^ (uint64_t)(t >> 64);
}

uint64_t orc_rng_u64(uint64_t *state) {
    uint64_t s = *state + WY0;
    *state = s;
    return wy_mix(s);
}

static inline double bits_to_unit_f64(uint64_t r) {
    /* Rng::f64: bits (1<<62)-(1<<52) + (u64 >> 12) is a float in [1,2); minus 1. */
    uint64_t bits = ((1ULL << 62) - (1ULL << 52)) + (r >> 12);
    double d;
    memcpy(&d, &bits, sizeof d);
    return d - 1.0;
}

double orc_rng_f64(uint64_t *state) { return bits_to_unit_f64(orc_rng_u64(state)); }

uint64_t orc_rng_below(uint64_t *state, uint64_t n) {
    /* Rng::gen_mod_u64: multiply-shift with rejection of the biased zone. */
    uint64_t r = orc_rng_u64(state);
    unsigned __int128 m = (unsigned __int128)r * n;
    uint64_t lo = (uint64_t)m;
    if (lo < n) {
        uint64_t t = (0 - n) % n;
        while (lo < t) {
            r = orc_rng_u64(state);
            m = (unsigned __int128)r * n;
            lo = (uint64_t)m;
        }
    }
    return (uint64_t)(m >> 64);
}

static inline float box_muller(double u1, double u2, float mean, float std) {
    /* nn/init.rs:3-9 */
    if (u1 < 1e-30) u1 = 1e-30;
    double z = sqrt(-2.0 * log(u1)) * cos(2.0 * 3.14159265358979323846 * u2);
    return (float)((double)mean + (double)std * z);
}

float orc_normal_sample(uint64_t *state, float mean, float std) {
    double u1 = orc_rng_f64(state);
    double u2 = orc_rng_f64(state);
    return box_muller(u1, u2, mean, std);
}

void orc_normal_vec(uint64_t *state, size_t n, float mean, float std, float *out) {
    for (size_t i = 0; i < n; i++) out[i] = orc_normal_sample(state, mean, std);
}

void orc_normal_vec_at(uint64_t seed, uint64_t first_draw, size_t n, float mean, float std,
                       float *out) {
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < n; i++) {
        uint64_t d1 = first_draw + 2 * (uint64_t)i + 1; /* 1-based draw index */
        uint64_t s1 = seed + d1 * WY0;
        uint64_t s2 = s1 + WY0;
        out[i] = box_muller(bits_to_unit_f64(wy_mix(s1)), bits_to_unit_f64(wy_mix(s2)), mean, std);
    }
}

/* ------------------------------------------------------------------------ */
/* quantize.rs                                                              */
/* ------------------------------------------------------------------------ */
float orc_quantize_symmetric(const float *w, size_t n, int8_t *q) {
    /* quantize.rs:17: absmax = fold(0, max(|w|)).  max is order independent. */
    float absmax = 0.0f;
#pragma omp parallel for reduction(max : absmax) schedule(static)
    for (size_t i = 0; i < n; i++) {
        float a = fabsf(w[i]);
        if (a > absmax) absmax = a;
    }
    if (absmax == 0.0f) { /* quantize.rs:19-21 */
        memset(q, 0, n);
        return 0.0f;
    }
    float scale = absmax / 127.0f;   /* :23 */
    float inv_scale = 1.0f / scale;  /* :24 */
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < n; i++) { /* :26-29 round half away from zero, clamp */
        float r = roundf(w[i] * inv_scale);
        if (r < -127.0f) r = -127.0f;
        if (r > 127.0f) r = 127.0f;
        /* f32::clamp leaves NaN as NaN and Rust's `as i8` maps NaN to 0 */
        q[i] = isnan(r) ? (int8_t)0 : (int8_t)r;
    }
    return scale;
}

void orc_dequantize(const int8_t *q, size_t n, float scale, float *out) {
    for (size_t i = 0; i < n; i++) out[i] = (float)q[i] * scale; /* quantize.rs:35-40 */
}

void orc_quantize_grouped(const float *w, int k, int n, int group, int8_t *q, float *scales) {
    int ng = (k + group - 1) / group;
#pragma omp parallel for schedule(static)
    for (int j = 0; j < n; j++) {
        for (int g = 0; g < ng; g++) {
            int p0 = g * group, p1 = p0 + group < k ? p0 + group : k;
            float absmax = 0.0f;
            for (int p = p0; p < p1; p++) {
                float a = fabsf(w[(size_t)p * n + j]);
                if (a > absmax) absmax = a;
            }
            if (absmax == 0.0f) {
                scales[(size_t)g * n + j] = 0.0f;
                for (int p = p0; p < p1; p++) q[(size_t)p * n + j] = 0;
                continue;
            }
            float scale = absmax / 127.0f, inv = 1.0f / scale;
            scales[(size_t)g * n + j] = scale;
            for (int p = p0; p < p1; p++) {
                float r = roundf(w[(size_t)p * n + j] * inv);
                if (r < -127.0f) r = -127.0f;
                if (r > 127.0f) r = 127.0f;
                q[(size_t)p * n + j] = isnan(r) ? (int8_t)0 : (int8_t)r; /* as quantize_symmetric */
            }
        }
    }
}

/* ------------------------------------------------------------------------ */
/* backend/cpu.rs                                                           */
/* ------------------------------------------------------------------------ */
#define JCHUNK 256

/* The hot loops are compiled for several instruction sets and picked at load
 * time (GCC target_clones); every variant performs the same IEEE operations
 * in the same order (-ffp-contract=off, no fast-math), only wider. */
#if defined(__GNUC__) && defined(__x86_64__) && !defined(__clang__)
#define ORC_CLONES __attribute__((target_clones("avx512f", "avx2", "default")))
#else
#define ORC_CLONES
#endif
#define IBLK 8

ORC_CLONES
void orc_matmul_i8_f32(const float *a, const int8_t *q, float scale, int m, int k, int n,
                       float *c) {
    /* cpu.rs:1129-1160.  c[i,j] accumulates, in f32, the terms
     * (f32)(f64(a[i,p]) * (f64(q[p,j]) * f64(scale))) for p = 0..k-1 in order
     * (the 32^3 tiling visits p ascending for every fixed (i,j)).  Here the
     * exact f64 product q[p,j] * scale (8 x 24 significant bits) is formed
     * once per (p, j) and shared by a block of rows; each (i,j) still sees
     * its terms in ascending p. */
    const double sd = (double)scale;
    int nchunks = (n + JCHUNK - 1) / JCHUNK;
#pragma omp parallel for schedule(dynamic, 1)
    for (int cj = 0; cj < nchunks; cj++) {
        int j0 = cj * JCHUNK, j1 = j0 + JCHUNK < n ? j0 + JCHUNK : n;
        double wd[JCHUNK];
        for (int i0 = 0; i0 < m; i0 += IBLK) {
            int i1 = i0 + IBLK < m ? i0 + IBLK : m;
            for (int i = i0; i < i1; i++)
                for (int j = j0; j < j1; j++) c[(size_t)i * n + j] = 0.0f;
            for (int p = 0; p < k; p++) {
                const int8_t *qrow = q + (size_t)p * n;
                for (int j = j0; j < j1; j++) wd[j - j0] = (double)qrow[j] * sd;
                for (int i = i0; i < i1; i++) {
                    double av = (double)a[(size_t)i * k + p];
                    float *crow = c + (size_t)i * n + j0;
                    for (int j = 0; j < j1 - j0; j++) crow[j] += (float)(av * wd[j]);
                }
            }
        }
    }
}

ORC_CLONES
void orc_matmul_i8_f32_tb(const float *a, const int8_t *q_t, float scale, int m, int k, int n,
                          float *c) {
    const double sd = (double)scale;
#pragma omp parallel for schedule(static)
    for (int j = 0; j < n; j++) {
        const int8_t *qcol = q_t + (size_t)j * k;
        for (int i = 0; i < m; i++) {
            const float *arow = a + (size_t)i * k;
            float acc = 0.0f;
            for (int p = 0; p < k; p++) acc += (float)((double)arow[p] * ((double)qcol[p] * sd));
            c[(size_t)i * n + j] = acc;
        }
    }
}

void orc_matmul_i8_f32_grouped(const float *a, const int8_t *q, const float *scales, int group,
                               int m, int k, int n, float *c) {
    int nchunks = (n + JCHUNK - 1) / JCHUNK;
#pragma omp parallel for schedule(dynamic, 1)
    for (int cj = 0; cj < nchunks; cj++) {
        int j0 = cj * JCHUNK, j1 = j0 + JCHUNK < n ? j0 + JCHUNK : n;
        for (int i = 0; i < m; i++) {
            float *crow = c + (size_t)i * n;
            for (int j = j0; j < j1; j++) crow[j] = 0.0f;
            for (int p = 0; p < k; p++) {
                double av = (double)a[(size_t)i * k + p];
                const int8_t *qrow = q + (size_t)p * n;
                const float *srow = scales + (size_t)(p / group) * n;
                for (int j = j0; j < j1; j++)
                    crow[j] += (float)(av * ((double)qrow[j] * (double)srow[j]));
            }
        }
    }
}

void orc_rmsnorm(const float *x, const float *w, int rows, int d, float eps, float *out) {
    /* cpu.rs:574-599 */
    for (int i = 0; i < rows; i++) {
        const float *s = x + (size_t)i * d;
        double sum = 0.0;
        for (int j = 0; j < d; j++) sum += (double)s[j] * (double)s[j];
        double mean_sq = sum / (double)d;
        double rstd = 1.0 / sqrt(mean_sq + (double)eps);
        for (int j = 0; j < d; j++) out[(size_t)i * d + j] = (float)((double)s[j] * rstd * (double)w[j]);
    }
}

void orc_rope(const float *x, int seq, int n_heads, int hd, int start_pos, const float *freqs,
              float *out) {
    /* cpu.rs:635-664 */
    int total = n_heads * hd;
    if (out != x) memcpy(out, x, sizeof(float) * (size_t)seq * total);
    for (int s = 0; s < seq; s++) {
        double pos = (double)(start_pos + s);
        for (int h = 0; h < n_heads; h++) {
            size_t hs = (size_t)s * total + (size_t)h * hd;
            for (int i = 0; i < hd / 2; i++) {
                double angle = pos * (double)freqs[i];
                float cv = (float)cos(angle), sv = (float)sin(angle);
                float x0 = x[hs + 2 * i], x1 = x[hs + 2 * i + 1];
                out[hs + 2 * i] = x0 * cv - x1 * sv;
                out[hs + 2 * i + 1] = x0 * sv + x1 * cv;
            }
        }
    }
}

void orc_scale(const float *x, size_t n, float s, float *out) {
    for (size_t i = 0; i < n; i++) out[i] = x[i] * s; /* cpu.rs:509-511 */
}

static inline float silu_scalar(float x) {
    double x64 = (double)x; /* cpu.rs:1119-1122 */
    return (float)(x64 / (1.0 + exp(-x64)));
}

void orc_swiglu(const float *g, const float *u, size_t n, float *out) {
    for (size_t i = 0; i < n; i++) out[i] = silu_scalar(g[i]) * u[i]; /* cpu.rs:666-678 */
}

void orc_softmax(const float *x, int rows, int cols, float *out) {
    /* cpu.rs:336-366: f32 max, f32 exp, f64 sum, f64 divide. */
    for (int r = 0; r < rows; r++) {
        const float *in = x + (size_t)r * cols;
        float *o = out + (size_t)r * cols;
        float mx = -INFINITY;
        for (int i = 0; i < cols; i++) mx = fmaxf(mx, in[i]);
        double sum = 0.0;
        for (int i = 0; i < cols; i++) {
            double e = (double)expf(in[i] - mx);
            o[i] = (float)e;
            sum += e;
        }
        for (int i = 0; i < cols; i++) o[i] = (float)((double)o[i] / sum);
    }
}

void orc_gemv_trans_b(const float *v, const float *mat_t, int k, int n, float *out) {
    /* cpu.rs:825-842 */
    int k4 = k & ~3;
    for (int j = 0; j < n; j++) {
        const float *row = mat_t + (size_t)j * k;
        float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
        for (int p = 0; p < k4; p += 4) {
            a0 += v[p] * row[p];
            a1 += v[p + 1] * row[p + 1];
            a2 += v[p + 2] * row[p + 2];
            a3 += v[p + 3] * row[p + 3];
        }
        float acc = a0 + a1 + a2 + a3;
        for (int p = k4; p < k; p++) acc += v[p] * row[p];
        out[j] = acc;
    }
}

void orc_gemv(const float *v, const float *mat, int k, int n, float *out) {
    /* cpu.rs:846-871 */
    for (int j = 0; j < n; j++) out[j] = 0.0f;
    int k4 = k & ~3;
    for (int p = 0; p < k4; p += 4) {
        float v0 = v[p], v1 = v[p + 1], v2 = v[p + 2], v3 = v[p + 3];
        const float *r0 = mat + (size_t)p * n, *r1 = r0 + n, *r2 = r1 + n, *r3 = r2 + n;
        for (int j = 0; j < n; j++) out[j] += v0 * r0[j] + v1 * r1[j] + v2 * r2[j] + v3 * r3[j];
    }
    for (int p = k4; p < k; p++) {
        float vv = v[p];
        const float *r = mat + (size_t)p * n;
        for (int j = 0; j < n; j++) out[j] += vv * r[j];
    }
}

void orc_gather_reshape_repeat_kv(const float *cache, int cached_len, int n_kv, int n_q, int hd,
                                  float *out) {
    /* cpu.rs:707-730 */
    int n_rep = n_q / n_kv, kv_dim = n_kv * hd;
    for (int qh = 0; qh < n_q; qh++) {
        int kvh = qh / n_rep;
        for (int s = 0; s < cached_len; s++)
            memcpy(out + ((size_t)qh * cached_len + s) * hd, cache + (size_t)s * kv_dim + (size_t)kvh * hd,
                   sizeof(float) * hd);
    }
}

void orc_compute_rope_freqs(int hd, float theta, const double *sc, double *out) {
    /* llama.rs:1035-1067 */
    double th = (double)theta;
    int np = hd / 2;
    for (int i = 0; i < np; i++) out[i] = 1.0 / pow(th, 2.0 * (double)i / (double)hd);
    if (sc) {
        double factor = sc[0], low = sc[1], high = sc[2], old_ctx = sc[3];
        double low_wl = old_ctx / low, high_wl = old_ctx / high;
        for (int i = 0; i < np; i++) {
            double wavelen = 2.0 * 3.14159265358979323846 / out[i];
            double sf;
            if (wavelen < high_wl) sf = 1.0;
            else if (wavelen > low_wl) sf = factor;
            else {
                double smooth = (old_ctx / wavelen - low) / (high - low);
                sf = 1.0 / ((1.0 - smooth) / factor + smooth);
            }
            out[i] /= sf;
        }
    }
}

int64_t orc_argmax(const float *x, size_t n) {
    /* generate.rs:167-173: Iterator::max_by keeps the LAST of equal maxima;
     * partial_cmp None (NaN) counts as Equal. */
    if (n == 0) return 0;
    size_t best = 0;
    for (size_t i = 1; i < n; i++) {
        float a = x[best], b = x[i];
        /* max_by(a, b): replace when b >= a, or when the comparison is NaN. */
        if (!(b < a)) best = i;
    }
    return (int64_t)best;
}

/* ------------------------------------------------------------------------ */
/* model                                                                    */
/* ------------------------------------------------------------------------ */
struct orc_llama {
    orc_config cfg;
    int hd, q_dim, kv_dim, qkv_dim;
    float *embed;      /* [V,h] */
    float *norm_in;    /* [L,h] */
    float *norm_post;  /* [L,h] */
    float *norm_final; /* [h] */
    int8_t **w;        /* [L*5] */
    float *scale;      /* [L*5] */
    int8_t *lm_head;   /* [V,h] */
    float lm_scale;
    float *freqs; /* [hd/2] f32, llama.rs:620-622 */
};

struct orc_cache {
    int max_seq, seq_len, kv_bf16, n_layers, kv_dim;
    float **k, **v; /* per layer [max_seq, kv_dim] */
};

static void wshape(const orc_llama *m, int slot, int *k, int *n) {
    int h = m->cfg.hidden_size, F = m->cfg.intermediate_size;
    switch (slot) {
    case ORC_QKV: *k = h; *n = m->qkv_dim; break;
    case ORC_O: *k = m->q_dim; *n = h; break;
    case ORC_GATE:
    case ORC_UP: *k = h; *n = F; break;
    default: *k = F; *n = h; break;
    }
}

orc_llama *orc_llama_new_empty(const orc_config *cfg) {
    orc_llama *m = (orc_llama *)calloc(1, sizeof *m);
    m->cfg = *cfg;
    int h = cfg->hidden_size, L = cfg->n_layers, V = cfg->vocab_size;
    m->hd = h / cfg->n_heads; /* llama.rs:97-99 */
    m->q_dim = cfg->n_heads * m->hd;
    m->kv_dim = cfg->n_kv_heads * m->hd;
    m->qkv_dim = m->q_dim + 2 * m->kv_dim;
    m->embed = (float *)malloc(sizeof(float) * (size_t)V * h);
    m->norm_in = (float *)malloc(sizeof(float) * (size_t)L * h);
    m->norm_post = (float *)malloc(sizeof(float) * (size_t)L * h);
    m->norm_final = (float *)malloc(sizeof(float) * (size_t)h);
    for (size_t i = 0; i < (size_t)L * h; i++) m->norm_in[i] = m->norm_post[i] = 1.0f; /* rmsnorm.rs:17-22 */
    for (int i = 0; i < h; i++) m->norm_final[i] = 1.0f;
    m->w = (int8_t **)calloc((size_t)L * 5, sizeof(int8_t *));
    m->scale = (float *)calloc((size_t)L * 5, sizeof(float));
    for (int l = 0; l < L; l++)
        for (int s = 0; s < 5; s++) {
            int k, n;
            wshape(m, s, &k, &n);
            m->w[l * 5 + s] = (int8_t *)calloc((size_t)k * n, 1);
        }
    m->lm_head = (int8_t *)calloc((size_t)V * h, 1);
    double *fr = (double *)malloc(sizeof(double) * (m->hd / 2));
    orc_compute_rope_freqs(m->hd, cfg->rope_theta, cfg->has_rope_scaling ? cfg->rope_scaling : NULL, fr);
    m->freqs = (float *)malloc(sizeof(float) * (m->hd / 2));
    for (int i = 0; i < m->hd / 2; i++) m->freqs[i] = (float)fr[i];
    free(fr);
    return m;
}

orc_llama *orc_llama_new_random(const orc_config *cfg, uint64_t seed) {
    /* LlamaModel::new (llama.rs:593-680).  Draw order: embed [V*h]; per layer
     * q [h*q], k [h*kv], v [h*kv], o [q*h], gate [h*F], up [h*F], down [F*h];
     * lm_head [V*h] when untied.  Each normal sample takes two f64 draws. */
    orc_llama *m = orc_llama_new_empty(cfg);
    int h = cfg->hidden_size, F = cfg->intermediate_size, V = cfg->vocab_size, L = cfg->n_layers;
    const float std = 0.02f;
    uint64_t draw = 0;
    size_t nemb = (size_t)V * h;
    orc_normal_vec_at(seed, draw, nemb, 0.0f, std, m->embed);
    draw += 2 * nemb;
    size_t nq = (size_t)h * m->q_dim, nkv = (size_t)h * m->kv_dim;
    float *qw = (float *)malloc(sizeof(float) * nq);
    float *kw = (float *)malloc(sizeof(float) * nkv);
    float *vw = (float *)malloc(sizeof(float) * nkv);
    size_t big = (size_t)h * F > (size_t)h * m->qkv_dim ? (size_t)h * F : (size_t)h * m->qkv_dim;
    float *tmp = (float *)malloc(sizeof(float) * big);
    for (int l = 0; l < L; l++) {
        orc_normal_vec_at(seed, draw, nq, 0.0f, std, qw);
        draw += 2 * nq;
        orc_normal_vec_at(seed, draw, nkv, 0.0f, std, kw);
        draw += 2 * nkv;
        orc_normal_vec_at(seed, draw, nkv, 0.0f, std, vw);
        draw += 2 * nkv;
        /* fuse_qkv_weights (llama.rs:1009-1029): row-wise column concat */
        for (int r = 0; r < h; r++) {
            float *dst = tmp + (size_t)r * m->qkv_dim;
            memcpy(dst, qw + (size_t)r * m->q_dim, sizeof(float) * m->q_dim);
            memcpy(dst + m->q_dim, kw + (size_t)r * m->kv_dim, sizeof(float) * m->kv_dim);
            memcpy(dst + m->q_dim + m->kv_dim, vw + (size_t)r * m->kv_dim, sizeof(float) * m->kv_dim);
        }
        m->scale[l * 5 + ORC_QKV] = orc_quantize_symmetric(tmp, (size_t)h * m->qkv_dim, m->w[l * 5 + ORC_QKV]);
        orc_normal_vec_at(seed, draw, nq, 0.0f, std, tmp);
        draw += 2 * nq;
        m->scale[l * 5 + ORC_O] = orc_quantize_symmetric(tmp, nq, m->w[l * 5 + ORC_O]);
        size_t nf = (size_t)h * F;
        for (int s = ORC_GATE; s <= ORC_DOWN; s++) {
            orc_normal_vec_at(seed, draw, nf, 0.0f, std, tmp);
            draw += 2 * nf;
            m->scale[l * 5 + s] = orc_quantize_symmetric(tmp, nf, m->w[l * 5 + s]);
        }
    }
    free(qw);
    free(kw);
    free(vw);
    free(tmp);
    if (cfg->tie_word_embeddings) {
        m->lm_scale = orc_quantize_symmetric(m->embed, nemb, m->lm_head);
    } else {
        float *lm = (float *)malloc(sizeof(float) * nemb);
        orc_normal_vec_at(seed, draw, nemb, 0.0f, std, lm);
        draw += 2 * nemb;
        m->lm_scale = orc_quantize_symmetric(lm, nemb, m->lm_head);
        free(lm);
    }
    return m;
}

static inline uint64_t orc_hash(uint64_t seed, uint64_t i) { return wy_mix(seed + (i + 1) * WY0); }

/* n int8 values in [-127, 127], eight per 64-bit hash of (seed, base + i/8). */
static void orc_fill_i8(int8_t *w, size_t n, uint64_t seed, uint64_t base) {
    size_t words = (n + 7) / 8;
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < words; i++) {
        uint64_t r = orc_hash(seed, base / 8 + i);
        for (int b = 0; b < 8 && 8 * i + b < n; b++) w[8 * i + b] = (int8_t)((int)((r >> (8 * b)) & 0xff) % 255 - 127);
    }
}

orc_llama *orc_llama_new_uniform(const orc_config *cfg, uint64_t seed) {
    /* A model of the given shape for timing the CPU path: int8 values uniform
     * in [-127, 127] from a counter-based hash, per-tensor scales of the
     * magnitude quantize_symmetric gives N(0, 0.02) weights, embeddings
     * uniform in [-0.05, 0.05].  The arithmetic of every op is independent of
     * the values, so the decode costs what a LlamaModel::new model costs,
     * without 2 x 6.7 G Box-Muller draws at the 7B shape. */
    orc_llama *m = orc_llama_new_empty(cfg);
    int h = cfg->hidden_size, V = cfg->vocab_size, L = cfg->n_layers;
    uint64_t base = 0;
    for (int l = 0; l < L; l++)
        for (int s = 0; s < 5; s++) {
            int k, n;
            wshape(m, s, &k, &n);
            size_t cnt = (size_t)k * n;
            int8_t *w = m->w[l * 5 + s];
            orc_fill_i8(w, cnt, seed, base);
            base += cnt;
            m->scale[l * 5 + s] = 0.09f / 127.0f;
        }
    size_t nemb = (size_t)V * h;
    orc_fill_i8(m->lm_head, nemb, seed, base);
#pragma omp parallel for schedule(static)
    for (size_t i = 0; i < nemb; i++)
        m->embed[i] = (float)(bits_to_unit_f64(orc_hash(seed ^ 0x5bd1e995ULL, i)) * 0.1 - 0.05);
    m->lm_scale = 0.09f / 127.0f;
    return m;
}

void orc_llama_free(orc_llama *m) {
    if (!m) return;
    for (int i = 0; i < m->cfg.n_layers * 5; i++) free(m->w[i]);
    free(m->w);
    free(m->scale);
    free(m->embed);
    free(m->norm_in);
    free(m->norm_post);
    free(m->norm_final);
    free(m->lm_head);
    free(m->freqs);
    free(m);
}

int8_t *orc_llama_weight(orc_llama *m, int layer, int slot, float *scale_out, int *k, int *n) {
    wshape(m, slot, k, n);
    if (scale_out) *scale_out = m->scale[layer * 5 + slot];
    return m->w[layer * 5 + slot];
}

int8_t *orc_llama_lm_head(orc_llama *m, float *scale_out) {
    if (scale_out) *scale_out = m->lm_scale;
    return m->lm_head;
}

float *orc_llama_embed(orc_llama *m) { return m->embed; }

float *orc_llama_norm(orc_llama *m, int layer, int which) {
    if (layer < 0) return m->norm_final;
    return (which ? m->norm_post : m->norm_in) + (size_t)layer * m->cfg.hidden_size;
}

void orc_llama_set_scale(orc_llama *m, int layer, int slot, float scale) {
    if (layer < 0) m->lm_scale = scale;
    else m->scale[layer * 5 + slot] = scale;
}

orc_cache *orc_cache_new(const orc_llama *m, int max_seq, int kv_bf16) {
    orc_cache *c = (orc_cache *)calloc(1, sizeof *c);
    c->max_seq = max_seq;
    c->kv_bf16 = kv_bf16;
    c->n_layers = m->cfg.n_layers;
    c->kv_dim = m->kv_dim;
    c->k = (float **)calloc(c->n_layers, sizeof(float *));
    c->v = (float **)calloc(c->n_layers, sizeof(float *));
    for (int l = 0; l < c->n_layers; l++) {
        c->k[l] = (float *)calloc((size_t)max_seq * m->kv_dim, sizeof(float));
        c->v[l] = (float *)calloc((size_t)max_seq * m->kv_dim, sizeof(float));
    }
    return c;
}

void orc_cache_free(orc_cache *c) {
    if (!c) return;
    for (int l = 0; l < c->n_layers; l++) {
        free(c->k[l]);
        free(c->v[l]);
    }
    free(c->k);
    free(c->v);
    free(c);
}

static inline float round_bf16(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    if ((u & 0x7f800000u) == 0x7f800000u) { /* inf / nan pass through */
        u &= 0xffff0000u;
    } else {
        u += 0x7fffu + ((u >> 16) & 1u); /* round to nearest even */
        u &= 0xffff0000u;
    }
    memcpy(&x, &u, 4);
    return x;
}

void orc_forward_with_cache(const orc_llama *m, orc_cache *c, int token, int pos, float *logits,
                            float *trace) {
    const orc_config *cfg = &m->cfg;
    int h = cfg->hidden_size, F = cfg->intermediate_size, V = cfg->vocab_size;
    int nh = cfg->n_heads, nkv = cfg->n_kv_heads, hd = m->hd;
    int q_dim = m->q_dim, kv_dim = m->kv_dim, qkv_dim = m->qkv_dim;
    float *x = (float *)malloc(sizeof(float) * h);
    float *xn = (float *)malloc(sizeof(float) * (h > F ? h : F) * 2);
    float *qkv = (float *)malloc(sizeof(float) * qkv_dim);
    float *qr = (float *)malloc(sizeof(float) * q_dim);
    float *kr = (float *)malloc(sizeof(float) * kv_dim);
    float *gate = (float *)malloc(sizeof(float) * F);
    float *up = (float *)malloc(sizeof(float) * F);
    float *proj = (float *)malloc(sizeof(float) * h);
    float *head_out = (float *)malloc(sizeof(float) * q_dim);
    int max_len = c->seq_len + 1;
    float *kexp = (float *)malloc(sizeof(float) * (size_t)nh * max_len * hd);
    float *vexp = (float *)malloc(sizeof(float) * (size_t)nh * max_len * hd);
    float *scores = (float *)malloc(sizeof(float) * (size_t)nh * max_len);
    float *attn = (float *)malloc(sizeof(float) * (size_t)nh * max_len);

    memcpy(x, m->embed + (size_t)token * h, sizeof(float) * h); /* llama.rs:753, cpu.rs:485-498 */
    float qscale = (float)(1.0 / sqrt((double)hd));             /* llama.rs:394 */
    int row = c->seq_len;
    for (int l = 0; l < cfg->n_layers; l++) {
        /* LlamaDecoderLayer::forward_with_llama_cache (llama.rs:556-569) */
        orc_rmsnorm(x, m->norm_in + (size_t)l * h, 1, h, cfg->rms_norm_eps, xn);
        /* LlamaAttention::forward_with_llama_cache (llama.rs:371-468) */
        orc_matmul_i8_f32(xn, m->w[l * 5 + ORC_QKV], m->scale[l * 5 + ORC_QKV], 1, h, qkv_dim, qkv);
        orc_rope(qkv, 1, nh, hd, pos, m->freqs, qr);
        orc_scale(qr, q_dim, qscale, qr); /* trait default, backend/mod.rs:219-230 */
        orc_rope(qkv + q_dim, 1, nkv, hd, pos, m->freqs, kr);
        float *kc = c->k[l] + (size_t)row * kv_dim, *vc = c->v[l] + (size_t)row * kv_dim;
        for (int i = 0; i < kv_dim; i++) {
            float kv_k = kr[i], kv_v = qkv[q_dim + kv_dim + i];
            kc[i] = c->kv_bf16 ? round_bf16(kv_k) : kv_k;
            vc[i] = c->kv_bf16 ? round_bf16(kv_v) : kv_v;
        }
        int cl = row + 1;
        orc_gather_reshape_repeat_kv(c->k[l], cl, nkv, nh, hd, kexp);
        orc_gather_reshape_repeat_kv(c->v[l], cl, nkv, nh, hd, vexp);
        for (int hh = 0; hh < nh; hh++) /* matmul_strided_batched M=1, cpu.rs:1337-1350 */
            orc_gemv_trans_b(qr + (size_t)hh * hd, kexp + (size_t)hh * cl * hd, hd, cl, scores + (size_t)hh * cl);
        orc_softmax(scores, nh, cl, attn);
        for (int hh = 0; hh < nh; hh++)
            orc_gemv(attn + (size_t)hh * cl, vexp + (size_t)hh * cl * hd, cl, hd, head_out + (size_t)hh * hd);
        orc_matmul_i8_f32(head_out, m->w[l * 5 + ORC_O], m->scale[l * 5 + ORC_O], 1, q_dim, h, proj);
        for (int i = 0; i < h; i++) x[i] = x[i] + proj[i]; /* llama.rs:564 */
        orc_rmsnorm(x, m->norm_post + (size_t)l * h, 1, h, cfg->rms_norm_eps, xn);
        /* LlamaMLP::forward (llama.rs:484-512) */
        orc_matmul_i8_f32(xn, m->w[l * 5 + ORC_GATE], m->scale[l * 5 + ORC_GATE], 1, h, F, gate);
        orc_matmul_i8_f32(xn, m->w[l * 5 + ORC_UP], m->scale[l * 5 + ORC_UP], 1, h, F, up);
        orc_swiglu(gate, up, F, gate);
        orc_matmul_i8_f32(gate, m->w[l * 5 + ORC_DOWN], m->scale[l * 5 + ORC_DOWN], 1, F, h, proj);
        for (int i = 0; i < h; i++) x[i] = x[i] + proj[i]; /* llama.rs:568 */
        if (trace) memcpy(trace + (size_t)l * h, x, sizeof(float) * h);
    }
    c->seq_len = row + 1;
    orc_rmsnorm(x, m->norm_final, 1, h, cfg->rms_norm_eps, xn); /* llama.rs:759 */
    orc_matmul_i8_f32_tb(xn, m->lm_head, m->lm_scale, 1, h, V, logits); /* llama.rs:761-762 */
    free(x); free(xn); free(qkv); free(qr); free(kr); free(gate); free(up); free(proj);
    free(head_out); free(kexp); free(vexp); free(scores); free(attn);
}

void orc_forward_tokens(const orc_llama *m, orc_cache *c, const int *tokens, int n, int pos0,
                        float *logits_all, float *logits_last) {
    /* n consecutive calls of orc_forward_with_cache (tokens[i] at position
     * pos0 + i, appended at rows seq_len + i), evaluated layer by layer for
     * all n tokens at once so every weight is streamed once per layer instead
     * of once per token.  Each output element is computed by the same
     * operations in the same order as in the per-token path: the int8
     * matmuls and RMSNorm act row by row (cpu.rs:1129-1160, :574-599), RoPE
     * per position (cpu.rs:635-664), and token i attends to rows
     * 0..seq_len+i of the gathered cache (llama.rs:414-456) -- so the logits
     * and the cache equal those of the token-by-token loop of generate()
     * (generate.rs:68-75) bit for bit.  Test infrastructure: it makes long
     * prompts affordable for the parity tests. */
    if (n <= 0) return;
    const orc_config *cfg = &m->cfg;
    int h = cfg->hidden_size, F = cfg->intermediate_size, V = cfg->vocab_size;
    int nh = cfg->n_heads, nkv = cfg->n_kv_heads, hd = m->hd;
    int q_dim = m->q_dim, kv_dim = m->kv_dim, qkv_dim = m->qkv_dim;
    int row0 = c->seq_len, full = row0 + n;
    size_t nn = (size_t)n;
    float *x = (float *)malloc(sizeof(float) * nn * h);
    float *xn = (float *)malloc(sizeof(float) * nn * h);
    float *qkv = (float *)malloc(sizeof(float) * nn * qkv_dim);
    float *qr = (float *)malloc(sizeof(float) * nn * q_dim);
    float *kr = (float *)malloc(sizeof(float) * nn * kv_dim);
    float *gate = (float *)malloc(sizeof(float) * nn * F);
    float *up = (float *)malloc(sizeof(float) * nn * F);
    float *proj = (float *)malloc(sizeof(float) * nn * h);
    float *head_out = (float *)malloc(sizeof(float) * nn * q_dim);
    float *kexp = (float *)malloc(sizeof(float) * (size_t)nh * full * hd);
    float *vexp = (float *)malloc(sizeof(float) * (size_t)nh * full * hd);
    float qscale = (float)(1.0 / sqrt((double)hd)); /* llama.rs:394 */
    for (int i = 0; i < n; i++) memcpy(x + (size_t)i * h, m->embed + (size_t)tokens[i] * h, sizeof(float) * h);
    for (int l = 0; l < cfg->n_layers; l++) {
        orc_rmsnorm(x, m->norm_in + (size_t)l * h, n, h, cfg->rms_norm_eps, xn);
        orc_matmul_i8_f32(xn, m->w[l * 5 + ORC_QKV], m->scale[l * 5 + ORC_QKV], n, h, qkv_dim, qkv);
        for (int i = 0; i < n; i++) {
            const float *qi = qkv + (size_t)i * qkv_dim;
            orc_rope(qi, 1, nh, hd, pos0 + i, m->freqs, qr + (size_t)i * q_dim);
            orc_scale(qr + (size_t)i * q_dim, q_dim, qscale, qr + (size_t)i * q_dim);
            orc_rope(qi + q_dim, 1, nkv, hd, pos0 + i, m->freqs, kr + (size_t)i * kv_dim);
            float *kc = c->k[l] + (size_t)(row0 + i) * kv_dim, *vc = c->v[l] + (size_t)(row0 + i) * kv_dim;
            for (int e = 0; e < kv_dim; e++) {
                float kv_k = kr[(size_t)i * kv_dim + e], kv_v = qi[q_dim + kv_dim + e];
                kc[e] = c->kv_bf16 ? round_bf16(kv_k) : kv_k;
                vc[e] = c->kv_bf16 ? round_bf16(kv_v) : kv_v;
            }
        }
        orc_gather_reshape_repeat_kv(c->k[l], full, nkv, nh, hd, kexp);
        orc_gather_reshape_repeat_kv(c->v[l], full, nkv, nh, hd, vexp);
#pragma omp parallel for schedule(dynamic, 1)
        for (int i = 0; i < n; i++) {
            int cl = row0 + i + 1;
            float *sc = (float *)malloc(sizeof(float) * (size_t)nh * cl);
            float *at = (float *)malloc(sizeof(float) * (size_t)nh * cl);
            for (int hh = 0; hh < nh; hh++)
                orc_gemv_trans_b(qr + (size_t)i * q_dim + (size_t)hh * hd, kexp + (size_t)hh * full * hd, hd, cl,
                                 sc + (size_t)hh * cl);
            orc_softmax(sc, nh, cl, at);
            for (int hh = 0; hh < nh; hh++)
                orc_gemv(at + (size_t)hh * cl, vexp + (size_t)hh * full * hd, cl, hd,
                         head_out + (size_t)i * q_dim + (size_t)hh * hd);
            free(sc);
            free(at);
        }
        orc_matmul_i8_f32(head_out, m->w[l * 5 + ORC_O], m->scale[l * 5 + ORC_O], n, q_dim, h, proj);
        for (size_t i = 0; i < nn * h; i++) x[i] = x[i] + proj[i]; /* llama.rs:564 */
        orc_rmsnorm(x, m->norm_post + (size_t)l * h, n, h, cfg->rms_norm_eps, xn);
        orc_matmul_i8_f32(xn, m->w[l * 5 + ORC_GATE], m->scale[l * 5 + ORC_GATE], n, h, F, gate);
        orc_matmul_i8_f32(xn, m->w[l * 5 + ORC_UP], m->scale[l * 5 + ORC_UP], n, h, F, up);
        orc_swiglu(gate, up, nn * F, gate);
        orc_matmul_i8_f32(gate, m->w[l * 5 + ORC_DOWN], m->scale[l * 5 + ORC_DOWN], n, F, h, proj);
        for (size_t i = 0; i < nn * h; i++) x[i] = x[i] + proj[i]; /* llama.rs:568 */
    }
    c->seq_len = full;
    if (logits_all) {
        orc_rmsnorm(x, m->norm_final, n, h, cfg->rms_norm_eps, xn);
        orc_matmul_i8_f32_tb(xn, m->lm_head, m->lm_scale, n, h, V, logits_all);
        if (logits_last) memcpy(logits_last, logits_all + (size_t)(n - 1) * V, sizeof(float) * V);
    } else if (logits_last) {
        orc_rmsnorm(x + (size_t)(n - 1) * h, m->norm_final, 1, h, cfg->rms_norm_eps, xn);
        orc_matmul_i8_f32_tb(xn, m->lm_head, m->lm_scale, 1, h, V, logits_last);
    }
    free(x); free(xn); free(qkv); free(qr); free(kr); free(gate); free(up); free(proj);
    free(head_out); free(kexp); free(vexp);
}

orc_cache *orc_cache_clone(const orc_cache *src) {
    /* Clone of LlamaKvCache (its storages are Clone; kv_cache.rs:69-79). */
    orc_cache *c = (orc_cache *)calloc(1, sizeof *c);
    *c = *src;
    c->k = (float **)calloc(c->n_layers, sizeof(float *));
    c->v = (float **)calloc(c->n_layers, sizeof(float *));
    for (int l = 0; l < c->n_layers; l++) {
        size_t b = sizeof(float) * (size_t)c->max_seq * c->kv_dim;
        c->k[l] = (float *)malloc(b);
        c->v[l] = (float *)malloc(b);
        memcpy(c->k[l], src->k[l], b);
        memcpy(c->v[l], src->v[l], b);
    }
    return c;
}

void orc_cache_truncate(orc_cache *c, int len) {
    /* Sets the pub seq_len field of every LlamaLayerKvCache (kv_cache.rs:75):
     * later appends overwrite rows from len on. */
    if (len >= 0 && len <= c->seq_len) c->seq_len = len;
}

int orc_cache_len(const orc_cache *c) { return c->seq_len; }

void orc_cache_fill(orc_cache *c, int len, uint64_t seed) {
    /* Rows 0..len-1 of every layer's K and V set to values uniform in
     * [-1, 1] (bf16-rounded for a bf16 cache), as if len positions had been
     * decoded: a context of that length for timing the CPU path. */
    if (len < 0 || len > c->max_seq) return;
    for (int l = 0; l < c->n_layers; l++) {
        size_t cnt = (size_t)len * c->kv_dim;
        uint64_t off = (uint64_t)l * 2 * (uint64_t)c->max_seq * c->kv_dim;
#pragma omp parallel for schedule(static)
        for (size_t i = 0; i < cnt; i++) {
            float kv = (float)(bits_to_unit_f64(orc_hash(seed, off + i)) * 2.0 - 1.0);
            float vv = (float)(bits_to_unit_f64(orc_hash(seed, off + cnt + i)) * 2.0 - 1.0);
            c->k[l][i] = c->kv_bf16 ? round_bf16(kv) : kv;
            c->v[l][i] = c->kv_bf16 ? round_bf16(vv) : vv;
        }
    }
    c->seq_len = len;
}

void orc_generate_greedy(const orc_llama *m, const int *prompt, int n_prompt, int max_tokens,
                         int kv_bf16, int *out_tokens) {
    /* generate.rs:51-89 with sample_token's greedy branch (:96-98). */
    orc_cache *c = orc_cache_new(m, n_prompt + max_tokens, kv_bf16);
    float *logits = (float *)malloc(sizeof(float) * m->cfg.vocab_size);
    int ng = 0;
    for (int pos = 0; pos < n_prompt; pos++) {
        orc_forward_with_cache(m, c, prompt[pos], pos, logits, NULL);
        if (pos == n_prompt - 1) out_tokens[ng++] = (int)orc_argmax(logits, m->cfg.vocab_size);
    }
    for (int i = 1; i < max_tokens; i++) {
        int last = out_tokens[ng - 1];
        orc_forward_with_cache(m, c, last, n_prompt + i - 1, logits, NULL);
        out_tokens[ng++] = (int)orc_argmax(logits, m->cfg.vocab_size);
    }
    free(logits);
    orc_cache_free(c);
}

/* ---- sample_token (generate.rs:92-165) ---------------------------------- */
typedef struct { size_t i; double v; } iv_pair;
static int cmp_desc(const void *a, const void *b) {
    const iv_pair *x = (const iv_pair *)a, *y = (const iv_pair *)b;
    if (x->v > y->v) return -1;
    if (x->v < y->v) return 1;
    return (x->i < y->i) ? -1 : (x->i > y->i);
}

int64_t orc_sample_token(const float *logits, size_t n, float temperature, size_t top_k,
                         float top_p, uint64_t *rng) {
    if (temperature < 1e-8f) return orc_argmax(logits, n);
    double *s = (double *)malloc(sizeof(double) * n);
    for (size_t i = 0; i < n; i++) s[i] = (double)logits[i] / (double)temperature;
    iv_pair *ix = (iv_pair *)malloc(sizeof(iv_pair) * n);
    if (top_k > 0 && top_k < n) {
        for (size_t i = 0; i < n; i++) { ix[i].i = i; ix[i].v = s[i]; }
        qsort(ix, n, sizeof *ix, cmp_desc);
        double thr = ix[top_k - 1].v;
        for (size_t i = 0; i < n; i++) if (s[i] < thr) s[i] = -INFINITY;
    }
    double mx = -INFINITY;
    for (size_t i = 0; i < n; i++) mx = fmax(mx, s[i]);
    double sum = 0.0;
    for (size_t i = 0; i < n; i++) { s[i] = exp(s[i] - mx); sum += s[i]; }
    if (sum > 0.0) for (size_t i = 0; i < n; i++) s[i] /= sum;
    else for (size_t i = 0; i < n; i++) s[i] = 1.0 / (double)n;
    if (top_p < 1.0f && top_p > 0.0f) {
        for (size_t i = 0; i < n; i++) { ix[i].i = i; ix[i].v = s[i]; }
        qsort(ix, n, sizeof *ix, cmp_desc);
        double cum = 0.0;
        size_t cut = n;
        for (size_t i = 0; i < n; i++) {
            cum += ix[i].v;
            if (cum >= (double)top_p) { cut = i + 1; break; }
        }
        char *keep = (char *)calloc(n, 1);
        for (size_t i = 0; i < cut; i++) keep[ix[i].i] = 1;
        for (size_t i = 0; i < n; i++) if (!keep[i]) s[i] = 0.0;
        free(keep);
        double s2 = 0.0;
        for (size_t i = 0; i < n; i++) s2 += s[i];
        if (s2 > 0.0) for (size_t i = 0; i < n; i++) s[i] /= s2;
    }
    /* weighted_sample (generate.rs:175-185) */
    double r = orc_rng_f64(rng), cum = 0.0;
    int64_t out = (int64_t)n - 1;
    for (size_t i = 0; i < n; i++) {
        cum += s[i];
        if (r < cum) { out = (int64_t)i; break; }
    }
    free(s);
    free(ix);
    return out;
}

void orc_set_threads(int n) { omp_set_num_threads(n > 0 ? n : 1); }
int orc_get_threads(void) { return omp_get_max_threads(); }
