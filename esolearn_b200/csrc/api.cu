// C-ABI entry points of libscryb200.so that are not part of the engine:
// error reporting, device selection, DeviceBackend storage, quantization,
// packed int8 weights with matmul_i8_f32, and the standalone Llama ops.
#include <cmath>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "attention.cuh"
#include "misc.cuh"
#include "qgemm.cuh"
#include "qgemv.cuh"
#include "sampler.cuh"

namespace sb {

namespace {
thread_local std::string g_err;
thread_local int g_err_code = SB_OK;
}  // namespace

int set_error(int code, const char *fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_err = buf;
    g_err_code = code;
    return code;
}

const DeviceProps &device_props() {
    static DeviceProps props[64];
    static bool init[64] = {};
    static std::mutex mu;
    int dev = 0;
    cudaGetDevice(&dev);
    dev &= 63;
    std::lock_guard<std::mutex> lock(mu);
    if (!init[dev]) {
        cudaDeviceProp p;
        if (cudaGetDeviceProperties(&p, dev) == cudaSuccess) {
            props[dev].sm_count = p.multiProcessorCount;
            props[dev].max_smem_optin = (int)p.sharedMemPerBlockOptin;
            props[dev].cc_major = p.major;
            props[dev].cc_minor = p.minor;
        } else {
            cudaGetLastError();
            props[dev].sm_count = 148;  // B200
            props[dev].max_smem_optin = 232448;
        }
        init[dev] = true;
    }
    return props[dev];
}

// Library-owned workspace for op-level calls (attention split partials).
struct Workspace {
    void *p = nullptr;
    size_t bytes = 0;
};

// kind 0: quantizer absmax word; kind 1: attention (counters first, then
// split partials).  Each kind has its own buffer per device so that one op
// never sees another op's leftovers; counters return to zero after every
// launch, so a buffer only needs zeroing when it is (re)allocated.
// WS_GEMM_SUMS only ever holds the tensor-core GEMM's int64 column sums,
// which must read zero before every call: a grown buffer is zero-filled and
// every call clears what it used.
// WS_SPLITK: the split-K GEMV's int64 sums and tile counters, zero between calls.
enum { WS_QUANT = 0, WS_ATTN = 1, WS_GEMM = 2, WS_GEMM_SUMS = 3, WS_SAMPLE = 4, WS_GROUPED = 5, WS_SPLITK = 6,
       WS_KINDS = 7 };
constexpr size_t WS_ATTN_COUNTER_BYTES = 64 * 1024;

static int workspace_get(int kind, size_t bytes, void **out, cudaStream_t st) {
    static Workspace ws[64][WS_KINDS];
    static std::mutex mu;
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lock(mu);
    Workspace &w = ws[dev & 63][kind];
    if (w.bytes < bytes) {
        if (w.p) {
            cudaStreamSynchronize(st);
            cudaFree(w.p);
            w.p = nullptr;
            w.bytes = 0;
        }
        cudaError_t e = cudaMalloc(&w.p, bytes);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return set_error(SB_ERR_OOM, "workspace cudaMalloc(%zu): %s", bytes, cudaGetErrorString(e));
        }
        SB_CUDA_TRY(cudaMemsetAsync(w.p, 0, bytes, st));
        w.bytes = bytes;
    }
    *out = w.p;
    return SB_OK;
}

}  // namespace sb

using namespace sb;

struct sb_qweight {
    QWeightDesc d;
    uint4 *buf = nullptr;
    float *gs = nullptr;
    bool loaded = false;
};

// I8Storage as the reference's backends hand it over: the int8 bytes of a
// weight with no shape (i8_from_vec(Vec<i8>), backend/mod.rs:18).  The bytes
// stay on the device as given; the first matmul_i8_f32 on the storage learns
// its [k, n] shape and packs a copy into 128-column tiles (the layout both the
// GEMV and the tensor-core GEMM stream), which later calls with that shape
// reuse.  The scale travels with every call, as in the reference trait.
struct sb_i8 {
    int8_t *raw = nullptr;
    size_t n = 0;
    std::mutex mu;             // guards the packed copy (clones share the storage)
    uint4 *packed = nullptr;   // [k, n] packed, or nullptr
    int pk = 0, pn = 0;        // its shape
    int dev = -1;              // device of the bytes
};

extern "C" {

int sb_last_error(char *buf, size_t len) {
    if (buf && len) {
        strncpy(buf, g_err.c_str(), len - 1);
        buf[len - 1] = 0;
    }
    return g_err_code;
}

int sb_abi_version(void) { return 1; }

sb_status sb_init(int device) {
    SB_CUDA_TRY(cudaSetDevice(device));
    SB_CUDA_TRY(cudaFree(nullptr));  // create the context
    const DeviceProps &p = device_props();
    SB_CHECK(p.cc_major >= 10, SB_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a", device,
             p.cc_major, p.cc_minor);
    return SB_OK;
}

sb_status sb_device_info(int *sm_count, int *cc_major, int *cc_minor, size_t *hbm_bytes) {
    const DeviceProps &p = device_props();
    if (sm_count) *sm_count = p.sm_count;
    if (cc_major) *cc_major = p.cc_major;
    if (cc_minor) *cc_minor = p.cc_minor;
    if (hbm_bytes) {
        size_t fr = 0, tot = 0;
        SB_CUDA_TRY(cudaMemGetInfo(&fr, &tot));
        *hbm_bytes = tot;
    }
    return SB_OK;
}

sb_status sb_alloc(void **dptr, size_t bytes) {
    SB_CHECK(dptr, SB_ERR_ARG, "sb_alloc: null out pointer");
    cudaError_t e = cudaMalloc(dptr, bytes ? bytes : 16);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return set_error(SB_ERR_OOM, "sb_alloc(%zu): %s", bytes, cudaGetErrorString(e));
    }
    SB_CUDA_TRY(cudaMemset(*dptr, 0, bytes ? bytes : 16));
    return SB_OK;
}

sb_status sb_free(void *dptr) {
    SB_CUDA_TRY(cudaFree(dptr));
    return SB_OK;
}

sb_status sb_memcpy_h2d(void *dst, const void *src, size_t bytes, void *stream) {
    SB_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, (cudaStream_t)stream));
    if (!stream) SB_CUDA_TRY(cudaStreamSynchronize(nullptr));
    return SB_OK;
}

sb_status sb_memcpy_d2h(void *dst, const void *src, size_t bytes, void *stream) {
    SB_CUDA_TRY(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, (cudaStream_t)stream));
    if (!stream) SB_CUDA_TRY(cudaStreamSynchronize(nullptr));
    return SB_OK;
}

sb_status sb_stream_sync(void *stream) {
    SB_CUDA_TRY(cudaStreamSynchronize((cudaStream_t)stream));
    return qgemv_check_error();
}

sb_status sb_quantize_symmetric_host(const float *w, size_t n, int8_t *q, float *scale) {
    // quantize.rs:16-32, bit-exact: f32 absmax fold, scale = absmax/127,
    // inv = 1/scale, q = round_half_away(w*inv) clamped to [-127, 127].
    SB_CHECK((w && q && scale) || n == 0, SB_ERR_ARG, "sb_quantize_symmetric_host: null argument");
    float absmax = 0.0f;
    for (size_t i = 0; i < n; i++) absmax = std::fmax(absmax, std::fabs(w[i]));
    if (absmax == 0.0f) {
        if (n) memset(q, 0, n);
        *scale = 0.0f;
        return SB_OK;
    }
    volatile float s = absmax / 127.0f;
    volatile float inv = 1.0f / s;
    for (size_t i = 0; i < n; i++) {
        volatile float prod = w[i] * inv;
        float r = std::round((float)prod);
        // f32::clamp keeps NaN and `as i8` maps it to 0 (a NaN weight, or
        // every weight once one is infinite: inv = 0 and inf * 0 = NaN)
        r = std::isnan(r) ? 0.0f : std::fmin(std::fmax(r, -127.0f), 127.0f);
        q[i] = (int8_t)r;
    }
    *scale = s;
    return SB_OK;
}

sb_status sb_quantize_symmetric(const float *w, size_t n, int8_t *q, float *scale, void *stream) {
    SB_CHECK(w && q && scale, SB_ERR_ARG, "sb_quantize_symmetric: null argument");
    void *ws = nullptr;
    SB_TRY(workspace_get(WS_QUANT, 256, &ws, (cudaStream_t)stream));
    SB_TRY(quantize_device(w, n, q, scale, reinterpret_cast<unsigned *>(ws), (cudaStream_t)stream));
    return SB_OK;
}

sb_status sb_qweight_create(int K, int N, int group, sb_qweight **out) { return sb_qweight_create_tn(K, N, group, 0, out); }

sb_status sb_qweight_create_tn(int K, int N, int group, int tile_n, sb_qweight **out) {
    SB_CHECK(out && K > 0 && N > 0, SB_ERR_ARG, "sb_qweight_create: bad argument");
    SB_CHECK(tile_n == 0 || tile_n == 16 || tile_n == 32 || tile_n == 64 || tile_n == 128 || tile_n == 256, SB_ERR_ARG,
             "sb_qweight_create_tn: tile width %d not in {0,16,32,64,128,256}", tile_n);
    SB_CHECK(group == 0 || group == 32 || group == 64, SB_ERR_UNSUPPORTED, "group %d not in {0,32,64}", group);
    SB_CHECK(group == 0 || K % group == 0, SB_ERR_SHAPE, "K=%d not a multiple of group %d", K, group);
    sb_qweight *w = new sb_qweight();
    w->d.K = K;
    w->d.N = N;
    w->d.KS = ceil_div(K, 16);
    w->d.TN = tile_n ? tile_n : qgemv_pick_tn(N, K, 16);
    w->d.ntiles = ceil_div(N, w->d.TN);
    w->d.group = group;
    cudaError_t e = cudaMalloc(&w->buf, qweight_bytes(K, N, w->d.TN));
    if (e == cudaSuccess && group > 0) e = cudaMalloc(&w->gs, sizeof(float) * qweight_scale_count(K, N, w->d.TN, group));
    if (e != cudaSuccess) {
        cudaGetLastError();
        cudaFree(w->buf);
        delete w;
        return set_error(SB_ERR_OOM, "sb_qweight_create: %s", cudaGetErrorString(e));
    }
    w->d.w = w->buf;
    w->d.gscale = w->gs;
    *out = w;
    return SB_OK;
}

sb_status sb_qweight_load(sb_qweight *w, const int8_t *q, const float *scales) {
    SB_CHECK(w && q && scales, SB_ERR_ARG, "sb_qweight_load: null argument");
    const int K = w->d.K, N = w->d.N;
    int8_t *tmp = nullptr;
    SB_CUDA_TRY(cudaMalloc(&tmp, (size_t)K * N));
    int rc = SB_OK;
    if (cudaMemcpy(tmp, q, (size_t)K * N, cudaMemcpyHostToDevice) != cudaSuccess)
        rc = set_error(SB_ERR_CUDA, "sb_qweight_load: upload failed");
    if (rc == SB_OK) rc = qweight_pack(tmp, K, N, w->d.TN, 0, 0, w->buf, nullptr);
    if (rc == SB_OK && w->d.group > 0) {
        const size_t ng = (size_t)(K / w->d.group) * N;
        float *ts = nullptr;
        if (cudaMalloc(&ts, sizeof(float) * ng) != cudaSuccess) rc = set_error(SB_ERR_OOM, "scale upload");
        if (rc == SB_OK && cudaMemcpy(ts, scales, sizeof(float) * ng, cudaMemcpyHostToDevice) != cudaSuccess)
            rc = set_error(SB_ERR_CUDA, "scale upload failed");
        if (rc == SB_OK) rc = qscale_pack(ts, K, N, w->d.TN, w->d.group, w->gs, nullptr);
        cudaDeviceSynchronize();
        cudaFree(ts);
    } else if (rc == SB_OK) {
        w->d.scale = scales[0];
    }
    cudaDeviceSynchronize();
    cudaFree(tmp);
    if (rc == SB_OK) w->loaded = true;
    return rc;
}

sb_status sb_qweight_destroy(sb_qweight *w) {
    if (!w) return SB_OK;
    cudaFree(w->buf);
    cudaFree(w->gs);
    delete w;
    return SB_OK;
}

// The packed copy of storage b for a [k, n] view, made on first use.
static sb_status i8_packed(sb_i8 *b, int k, int n, cudaStream_t st, QWeightDesc *d) {
    std::lock_guard<std::mutex> lock(b->mu);
    if (!b->packed || b->pk != k || b->pn != n) {
        const size_t bytes = qweight_bytes(k, n, 128);
        uint4 *p = nullptr;
        cudaError_t e = cudaMalloc(&p, bytes);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return set_error(SB_ERR_OOM, "matmul_i8_f32: packing a [%d, %d] weight: %s", k, n, cudaGetErrorString(e));
        }
        const int rc = qweight_pack(b->raw, k, n, 128, 0, 0, p, st);
        if (rc != SB_OK) {
            cudaFree(p);
            return rc;
        }
        if (b->packed) {
            // an earlier view of these bytes: its kernels were queued on some
            // stream before this call; let them finish before freeing
            SB_CUDA_TRY(cudaDeviceSynchronize());
            cudaFree(b->packed);
        }
        b->packed = p;
        b->pk = k;
        b->pn = n;
    }
    d->w = b->packed;
    d->K = k;
    d->N = n;
    d->KS = ceil_div(k, 16);
    d->TN = 128;
    d->ntiles = ceil_div(n, 128);
    d->group = 0;
    return SB_OK;
}

// Rows [0, M) of a through the tensor-core GEMM (5-64 rows per launch).
static sb_status qgemm_rows(const QWeightDesc &wd, const void *a, bool bf16, int M, const float *bias, float *c,
                            cudaStream_t stream) {
    // scratch = planes, column sums, row exponents
    QGemmWs ws;
    ws.ld_acc = wd.ntiles * 128;
    const size_t pb = align_up(qgemm_planes_bytes(wd.K, M), 256);
    void *base = nullptr, *sums = nullptr;
    // planes, then rstd[QGM_MAX_M] doubles, then shift[QGM_MAX_M] ints
    const size_t rb = sizeof(double) * QGM_MAX_M, sb = sizeof(int) * QGM_MAX_M;
    SB_TRY(workspace_get(WS_GEMM, pb + rb + sb, &base, stream));
    SB_TRY(workspace_get(WS_GEMM_SUMS, sizeof(long long) * (size_t)M * ws.ld_acc, &sums, stream));
    char *b = static_cast<char *>(base);
    ws.planes = reinterpret_cast<uint8_t *>(b);
    ws.acc = reinterpret_cast<long long *>(sums);
    ws.rstd = reinterpret_cast<double *>(b + pb);
    ws.shift = reinterpret_cast<int *>(b + pb + rb);
    QGemvArgs g;
    g.w = wd;
    g.M = M;
    g.x = a;
    g.ldx = wd.K;
    g.x_bf16 = bf16;
    g.out = c;
    g.ldo = wd.N;
    g.bias = bias;
    return qgemm_launch(bias ? QEPI_BIAS : QEPI_STORE, g, ws, stream, false);
}

// Rows [0, M) (5-32) of a group-scaled weight through the tensor cores.
static sb_status qgemm_grouped_rows(const QWeightDesc &wd, const void *a, bool bf16, int M, const float *bias,
                                    float *c, cudaStream_t stream) {
    QGemmWs ws;
    const size_t pb = align_up(qgemm_planes_bytes(wd.K, M), 256);
    const size_t rb = sizeof(double) * QGM_MAX_M, sb = sizeof(int) * QGM_MAX_M;
    void *base = nullptr, *part = nullptr;
    SB_TRY(workspace_get(WS_GEMM, pb + rb + sb, &base, stream));
    SB_TRY(workspace_get(WS_GROUPED, sizeof(double) * qgemm_grouped_part_doubles(wd), &part, stream));
    char *b = static_cast<char *>(base);
    ws.planes = reinterpret_cast<uint8_t *>(b);
    ws.rstd = reinterpret_cast<double *>(b + pb);
    ws.shift = reinterpret_cast<int *>(b + pb + rb);
    QGemvArgs g;
    g.w = wd;
    g.M = M;
    g.x = a;
    g.ldx = wd.K;
    g.x_bf16 = bf16;
    g.out = c;
    g.ldo = wd.N;
    g.bias = bias;
    return qgemm_grouped_launch(bias ? QEPI_BIAS : QEPI_STORE, g, ws, static_cast<double *>(part), stream, false);
}

static sb_status matmul_desc(const QWeightDesc &wd, const void *a, int a_dtype, int M, const float *bias, float *c,
                             void *stream) {
    SB_CHECK(a_dtype == SB_DTYPE_F32 || a_dtype == SB_DTYPE_BF16, SB_ERR_ARG, "bad activation dtype %d", a_dtype);
    SB_CHECK(M >= 0, SB_ERR_ARG, "M < 0");
    const size_t esz = a_dtype == SB_DTYPE_BF16 ? 2 : 4;
    const bool bf16 = a_dtype == SB_DTYPE_BF16;
    const cudaStream_t st = (cudaStream_t)stream;
    if (qgemm_supported(wd, M)) return qgemm_rows(wd, a, bf16, M, bias, c, st);
    if (M > QGM_MAX_M && qgemm_supported(wd, QGM_MAX_M)) {
        // More than 64 rows: balanced chunks of 33-64 rows, one GEMM each, in
        // stream order (each chunk's finish kernel clears the shared sums).
        // Rows are independent, so the result equals the row-wise GEMVs.
        const int nc = (M + QGM_MAX_M - 1) / QGM_MAX_M;
        for (int i = 0; i < nc; i++) {
            const int r0 = (int)((long long)M * i / nc), r1 = (int)((long long)M * (i + 1) / nc);
            SB_TRY(qgemm_rows(wd, static_cast<const char *>(a) + (size_t)r0 * wd.K * esz, bf16, r1 - r0, bias,
                              c + (size_t)r0 * wd.N, st));
        }
        return SB_OK;
    }
    if (M > QG_MAX_M && qgemm_grouped_supported(wd, std::min(M, 32))) {
        // Group-scaled weights, 5+ rows: balanced chunks of at most 32 rows on
        // the tensor cores (rows are independent).
        const int nc = (M + 31) / 32;
        for (int i = 0; i < nc; i++) {
            const int r0 = (int)((long long)M * i / nc), r1 = (int)((long long)M * (i + 1) / nc);
            SB_TRY(qgemm_grouped_rows(wd, static_cast<const char *>(a) + (size_t)r0 * wd.K * esz, bf16, r1 - r0,
                                      bias, c + (size_t)r0 * wd.N, st));
        }
        return SB_OK;
    }
    for (int r0 = 0; r0 < M; r0 += QG_MAX_M) {
        QGemvArgs g;
        g.w = wd;
        g.M = std::min(QG_MAX_M, M - r0);
        g.x = (const char *)a + (size_t)r0 * wd.K * esz;
        g.ldx = wd.K;
        g.x_bf16 = bf16;
        g.out = c + (size_t)r0 * wd.N;
        g.ldo = wd.N;
        g.bias = bias;
        if (qgemv_splitk_wanted(wd, g.M)) {
            // few 128-column tiles: split K over the SMs
            void *ws = nullptr;
            SB_TRY(workspace_get(WS_SPLITK, qgemv_splitk_ws_bytes(wd, QG_MAX_M), &ws, st));
            SB_TRY(qgemv_splitk_launch(bias ? QEPI_BIAS : QEPI_STORE, g, ws, st));
            continue;
        }
        SB_TRY(qgemv_launch(bias ? QEPI_BIAS : QEPI_STORE, g, st, false));
    }
    return SB_OK;
}

static sb_status matmul_impl(const sb_qweight *w, const void *a, int a_dtype, int M, const float *bias, float *c,
                             void *stream) {
    SB_CHECK(w && a && c, SB_ERR_ARG, "sb_matmul_i8_f32: null argument");
    SB_CHECK(w->loaded, SB_ERR_STATE, "sb_matmul_i8_f32: weight not loaded");
    return matmul_desc(w->d, a, a_dtype, M, bias, c, stream);
}

sb_status sb_matmul_i8_f32(const sb_qweight *w, const void *a, int a_dtype, int M, float *c, void *stream) {
    return matmul_impl(w, a, a_dtype, M, nullptr, c, stream);
}

sb_status sb_matmul_i8_f32_bias(const sb_qweight *w, const void *a, int a_dtype, int M, const float *bias, float *c,
                                void *stream) {
    SB_CHECK(bias, SB_ERR_ARG, "sb_matmul_i8_f32_bias: null bias");
    return matmul_impl(w, a, a_dtype, M, bias, c, stream);
}

sb_status sb_i8_from_vec(const int8_t *data, size_t n, sb_i8 **out) {
    SB_CHECK(out && (data || n == 0), SB_ERR_ARG, "sb_i8_from_vec: null argument");
    sb_i8 *b = new sb_i8();
    b->n = n;
    cudaGetDevice(&b->dev);
    cudaError_t e = cudaMalloc(&b->raw, n ? n : 16);
    if (e == cudaSuccess && n) e = cudaMemcpy(b->raw, data, n, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaGetLastError();
        cudaFree(b->raw);
        delete b;
        return set_error(SB_ERR_OOM, "sb_i8_from_vec(%zu bytes): %s", n, cudaGetErrorString(e));
    }
    *out = b;
    return SB_OK;
}

sb_status sb_i8_to_vec(const sb_i8 *b, int8_t *data, size_t n) {
    SB_CHECK(b && (data || n == 0), SB_ERR_ARG, "sb_i8_to_vec: null argument");
    SB_CHECK(n == b->n, SB_ERR_SHAPE, "sb_i8_to_vec: storage holds %zu bytes, buffer %zu", b->n, n);
    if (n) SB_CUDA_TRY(cudaMemcpy(data, b->raw, n, cudaMemcpyDeviceToHost));
    return SB_OK;
}

sb_status sb_i8_len(const sb_i8 *b, size_t *n) {
    SB_CHECK(b && n, SB_ERR_ARG, "sb_i8_len: null argument");
    *n = b->n;
    return SB_OK;
}

sb_status sb_i8_destroy(sb_i8 *b) {
    if (!b) return SB_OK;
    cudaFree(b->raw);
    cudaFree(b->packed);
    delete b;
    return SB_OK;
}

static sb_status i8_matmul(const float *a, sb_i8 *b_q, float scale, const float *bias, int m, int k, int n, float *c,
                           void *stream) {
    SB_CHECK(b_q && (a || m == 0) && (c || m == 0), SB_ERR_ARG, "matmul_i8_f32: null argument");
    SB_CHECK(m >= 0 && k > 0 && n > 0, SB_ERR_SHAPE, "matmul_i8_f32: m %d, k %d, n %d", m, k, n);
    SB_CHECK((size_t)k * (size_t)n <= b_q->n, SB_ERR_SHAPE, "matmul_i8_f32: [%d, %d] view of a %zu-byte storage", k,
             n, b_q->n);
    int dev = 0;
    SB_CUDA_TRY(cudaGetDevice(&dev));
    SB_CHECK(dev == b_q->dev, SB_ERR_STATE, "matmul_i8_f32: storage lives on device %d, current device %d", b_q->dev,
             dev);
    if (m == 0) return SB_OK;
    QWeightDesc d;
    SB_TRY(i8_packed(b_q, k, n, (cudaStream_t)stream, &d));
    d.scale = scale;
    return matmul_desc(d, a, SB_DTYPE_F32, m, bias, c, stream);
}

sb_status sb_i8_matmul_f32(const float *a, sb_i8 *b_q, float scale, int m, int k, int n, float *c, void *stream) {
    return i8_matmul(a, b_q, scale, nullptr, m, k, n, c, stream);
}

sb_status sb_i8_matmul_f32_bias(const float *a, sb_i8 *b_q, float scale, const float *bias, int m, int k, int n,
                                float *c, void *stream) {
    SB_CHECK(bias, SB_ERR_ARG, "matmul_i8_f32_bias: null bias");
    return i8_matmul(a, b_q, scale, bias, m, k, n, c, stream);
}

sb_status sb_rmsnorm(const float *x, const float *w, int rows, int d, float eps, float *out, void *stream) {
    SB_CHECK(x && w && out && rows >= 0 && d > 0, SB_ERR_ARG, "sb_rmsnorm: bad argument");
    return rmsnorm_launch(x, w, rows, d, eps, out, (cudaStream_t)stream);
}

sb_status sb_rope_with_freqs(const float *x, int seq, int n_heads, int head_dim, int start_pos, const float *freqs,
                             float scale, float *out, void *stream) {
    SB_CHECK(x && freqs && out && seq >= 0 && n_heads >= 0 && head_dim > 0 && head_dim % 2 == 0, SB_ERR_ARG,
             "sb_rope_with_freqs: bad argument");
    return rope_launch(x, seq, n_heads, head_dim, start_pos, freqs, scale, out, (cudaStream_t)stream);
}

sb_status sb_swiglu(const float *gate, const float *up, size_t n, float *out, void *stream) {
    SB_CHECK((gate && up && out) || n == 0, SB_ERR_ARG, "sb_swiglu: null argument");
    return swiglu_launch(gate, up, n, out, (cudaStream_t)stream);
}

sb_status sb_argmax_rows(const float *x, int rows, int n, int32_t *out, void *stream) {
    SB_CHECK(x && out && rows >= 0 && n > 0, SB_ERR_ARG, "sb_argmax_rows: bad argument");
    return argmax_rows_launch(x, rows, n, out, (cudaStream_t)stream);
}

sb_status sb_sample_rows(const float *logits, int rows, int n, int ld, float temperature, int top_k, float top_p,
                         uint64_t *rng_state, int32_t *out, void *stream) {
    SB_CHECK(logits && rng_state && out, SB_ERR_ARG, "sb_sample_rows: null argument");
    SB_CHECK(rows >= 0 && n >= 1 && ld >= n, SB_ERR_SHAPE, "sb_sample_rows: rows %d, n %d, ld %d", rows, n, ld);
    SB_CHECK(!std::isnan(temperature) && !std::isnan(top_p) && top_k >= 0, SB_ERR_ARG,
             "sb_sample_rows: temperature %g, top_k %d, top_p %g", (double)temperature, top_k, (double)top_p);
    if (rows == 0) return SB_OK;
    void *prob = nullptr;
    if (!(temperature < 1e-8f))
        SB_TRY(workspace_get(WS_SAMPLE, sizeof(double) * (size_t)rows * n, &prob, (cudaStream_t)stream));
    return sample_rows_launch(logits, rows, n, ld, temperature, top_k, top_p, rng_state, static_cast<double *>(prob),
                              out, (cudaStream_t)stream);
}

sb_status sb_attn_decode_paged(const float *q, const void *k_cache, const void *v_cache, int kv_dtype,
                               const int32_t *page_table, int max_pages, const int32_t *ctx_len, int B, int n_heads,
                               int n_kv, int head_dim, int page_size, int max_ctx, float *out, void *stream) {
    SB_CHECK(q && k_cache && v_cache && page_table && ctx_len && out, SB_ERR_ARG, "sb_attn_decode_paged: null argument");
    SB_CHECK(B >= 1 && n_kv >= 1 && n_heads >= n_kv && page_size >= 1 && max_pages >= 1 && max_ctx >= 1, SB_ERR_ARG,
             "sb_attn_decode_paged: bad shape");
    SB_CHECK(max_ctx <= max_pages * page_size, SB_ERR_SHAPE, "max_ctx %d beyond %d pages of %d", max_ctx, max_pages,
             page_size);
    AttnArgs a;
    a.q = q;
    a.kc = k_cache;
    a.vc = v_cache;
    a.kv_f32 = kv_dtype == SB_KV_F32;
    a.page_table = page_table;
    a.max_pages = max_pages;
    a.len = ctx_len;
    a.len_is_pos = 0;
    a.B = B;
    a.n_heads = n_heads;
    a.n_kv = n_kv;
    a.hd = head_dim;
    a.page_size = page_size;
    a.n_splits = attn_pick_splits(B, n_kv, max_ctx);
    a.out = out;
    if (a.n_splits > 1) {
        SB_CHECK((size_t)B * n_kv * sizeof(unsigned) <= WS_ATTN_COUNTER_BYTES, SB_ERR_SHAPE,
                 "sb_attn_decode_paged: B*n_kv = %d too large", B * n_kv);
        const size_t pf = attn_scratch_floats(B, n_heads, a.n_splits, head_dim);
        void *ws = nullptr;
        SB_TRY(workspace_get(WS_ATTN, WS_ATTN_COUNTER_BYTES + pf * sizeof(float), &ws, (cudaStream_t)stream));
        a.counters = reinterpret_cast<unsigned *>(ws);
        a.part = reinterpret_cast<float *>((char *)ws + WS_ATTN_COUNTER_BYTES);
    }
    return attn_launch(a, (cudaStream_t)stream, false);
}

}  // extern "C"
