// sb_attn_decode_paged_noalloc: the paged decode attention of
// sb_attn_decode_paged without any device allocation.
//
// Who needs it.  sb_attn_decode_paged keeps its split-context scratch (the
// per-split partial outputs and the arrival counters) in a workspace that
// the library cudaMalloc's on first use and grows when a larger shape comes
// along.  Some callers cannot let that happen: a host whose device memory is
// entirely handed out by its own pool allocator (an inference server that
// partitions HBM up front, a Rust backend that owns every buffer) has no
// room for an allocation it did not make, and a latency-critical decode loop
// cannot absorb the device-wide synchronisation that cudaMalloc/cudaFree
// imply in the middle of a step.  This entry point uses a fixed scratch
// array compiled into the library instead.
//
// The scratch.  g_attn_scratch below is a file-scope __device__ array of
// NOALLOC_SCRATCH_BYTES (16 KiB of counters + 1 MiB of partials).
// Every GPU that loads the library holds it until the process exits.  Host
// code cannot use the symbol as a device address, so on the first call on
// each device (with that device current) cudaGetSymbolAddress resolves it
// once; make that first call before any stream capture.  All calls on a
// device share the one array and it keeps whatever the last call left:
// each call therefore zeroes the counters it uses before launching, and two
// calls that overlap on the GPU (different streams, no ordering between
// them) race on the array and give wrong results.
#include <mutex>

#include "attention.cuh"

namespace sb {
namespace {

constexpr size_t NOALLOC_COUNTER_BYTES = 16 * 1024;        // up to 4096 (sequence, kv head) counters
constexpr size_t NOALLOC_PARTIAL_BYTES = 1024 * 1024;      // split partials, f32
constexpr size_t NOALLOC_SCRATCH_BYTES = NOALLOC_COUNTER_BYTES + NOALLOC_PARTIAL_BYTES;

static __device__ __align__(256) unsigned char g_attn_scratch[NOALLOC_SCRATCH_BYTES];

// Device address of g_attn_scratch on the current device, resolved once.
int scratch_address(void **out) {
    static void *addr[64] = {};
    static std::mutex mu;
    int dev = 0;
    SB_CUDA_TRY(cudaGetDevice(&dev));
    SB_CHECK(dev >= 0 && dev < 64, SB_ERR_ARG, "device %d out of range", dev);
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_attn_scratch);
        if (e != cudaSuccess)
            return set_error(SB_ERR_CUDA, "cudaGetSymbolAddress(attention scratch): %s", cudaGetErrorString(e));
        addr[dev] = p;
    }
    *out = addr[dev];
    return SB_OK;
}

}  // namespace
}  // namespace sb

using namespace sb;

extern "C" sb_status sb_attn_decode_paged_noalloc(const float *q, const void *k_cache, const void *v_cache,
                                                  int kv_dtype, const int32_t *page_table, int max_pages,
                                                  const int32_t *ctx_len, int B, int n_heads, int n_kv,
                                                  int head_dim, int page_size, int max_ctx, float *out,
                                                  void *stream) {
    SB_CHECK(q && k_cache && v_cache && page_table && ctx_len && out, SB_ERR_ARG,
             "sb_attn_decode_paged_noalloc: null argument");
    SB_CHECK(B >= 1 && n_kv >= 1 && n_heads >= n_kv && page_size >= 1 && max_pages >= 1 && max_ctx >= 1,
             SB_ERR_ARG, "sb_attn_decode_paged_noalloc: bad shape");
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
    a.n_splits = attn_pick_splits(B, n_kv, max_ctx);  // the same split choice as sb_attn_decode_paged
    a.out = out;
    cudaStream_t st = (cudaStream_t)stream;
    if (a.n_splits > 1) {
        const size_t counter_bytes = sizeof(unsigned) * (size_t)B * n_kv;
        const size_t partial_bytes = sizeof(float) * attn_scratch_floats(B, n_heads, a.n_splits, head_dim);
        SB_CHECK(counter_bytes <= NOALLOC_COUNTER_BYTES, SB_ERR_SHAPE,
                 "sb_attn_decode_paged_noalloc: B*n_kv = %d exceeds the fixed scratch (%zu counters)", B * n_kv,
                 NOALLOC_COUNTER_BYTES / sizeof(unsigned));
        SB_CHECK(partial_bytes <= NOALLOC_PARTIAL_BYTES, SB_ERR_SHAPE,
                 "sb_attn_decode_paged_noalloc: %d splits of B=%d x %d heads x (%d+2) floats need %zu bytes; the "
                 "fixed scratch holds %zu",
                 a.n_splits, B, n_heads, head_dim, partial_bytes, NOALLOC_PARTIAL_BYTES);
        void *base = nullptr;
        SB_TRY(scratch_address(&base));
        // The array keeps the last call's contents: start the counters at zero.
        SB_CUDA_TRY(cudaMemsetAsync(base, 0, counter_bytes, st));
        a.counters = reinterpret_cast<unsigned *>(base);
        a.part = reinterpret_cast<float *>(static_cast<unsigned char *>(base) + NOALLOC_COUNTER_BYTES);
    }
    return attn_launch(a, st, false);
}
