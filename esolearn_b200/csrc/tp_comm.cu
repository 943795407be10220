// Communication of the tensor-parallel engine: an NCCL communicator resolved
// with dlopen, and a one-shot all-reduce over NVLink peer memory for the
// small per-layer residual sums.
//
// Peer all-reduce (tp_ar_kernel).  CTA c of every rank owns slice c of the
// vector.  It writes each value of its slice, paired with the call's epoch in
// one 8-byte store, into slot [parity][rank] of every other rank's cells over
// NVLink; then it reads the other ranks' cells of slice c from its own HBM,
// waiting (bounded: 2 s of %globaltimer, then an error word) until each
// cell carries the epoch, and sums the ranks' values in rank order -- so all
// ranks get the same bits.  The value and its epoch travel in one store, so
// no fence or separate flag is needed.  Slots alternate by epoch parity: a
// rank can write call e+2 only after every rank wrote call e+1, i.e. after
// every rank finished reading call e.
#include "tp_comm.cuh"

#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cstring>
#include <vector>

#include "pipeline.cuh"
#include <mutex>
#include <thread>

namespace sb {

namespace {

struct NcclApi {
    bool ok = false;
    ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
    ncclResult_t (*init_rank_config)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *) = nullptr;
    ncclResult_t (*get_async_error)(ncclComm_t, ncclResult_t *) = nullptr;
    ncclResult_t (*finalize)(ncclComm_t) = nullptr;
    ncclResult_t (*destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*abort)(ncclComm_t) = nullptr;
    ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                               cudaStream_t) = nullptr;
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    const char *(*error_string)(ncclResult_t) = nullptr;
};

NcclApi g_api;
std::once_flag g_once;

template <typename F>
bool sym(void *h, const char *name, F &f) {
    f = reinterpret_cast<F>(dlsym(h, name));
    return f != nullptr;
}

const NcclApi &api() {
    std::call_once(g_once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) return;
        NcclApi a;
        a.ok = sym(h, "ncclGetUniqueId", a.get_unique_id) && sym(h, "ncclCommInitRankConfig", a.init_rank_config) &&
               sym(h, "ncclCommGetAsyncError", a.get_async_error) && sym(h, "ncclCommFinalize", a.finalize) &&
               sym(h, "ncclCommDestroy", a.destroy) && sym(h, "ncclCommAbort", a.abort) &&
               sym(h, "ncclAllReduce", a.all_reduce) && sym(h, "ncclAllGather", a.all_gather) &&
               sym(h, "ncclGetErrorString", a.error_string);
        g_api = a;
    });
    return g_api;
}

int nccl_fail(const char *what, ncclResult_t r) {
    const NcclApi &a = api();
    return set_error(SB_ERR_NCCL, "%s: %s", what, a.error_string ? a.error_string(r) : "nccl error");
}

// Poll a non-blocking communicator until its last call has finished.
int wait_comm(ncclComm_t comm, double timeout_s, const char *what) {
    const NcclApi &a = api();
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
        ncclResult_t st = ncclSuccess;
        ncclResult_t r = a.get_async_error(comm, &st);
        if (r != ncclSuccess) return nccl_fail(what, r);
        if (st == ncclSuccess) return SB_OK;
        if (st != ncclInProgress) return nccl_fail(what, st);
        const double el = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (el > timeout_s) return set_error(SB_ERR_TIMEOUT, "%s: no progress after %.0f s", what, timeout_s);
        std::this_thread::sleep_for(std::chrono::microseconds(200));
    }
}

// A collective on a non-blocking communicator may return ncclInProgress
// while it is being enqueued; wait (bounded) until it is.
int enqueued(const TpComm &c, ncclResult_t r, const char *what) {
    if (r == ncclSuccess) return SB_OK;
    if (r == ncclInProgress) return wait_comm((ncclComm_t)c.comm, 60.0, what);
    return nccl_fail(what, r);
}


__global__ void __launch_bounds__(256) tp_ar_kernel(float *x, int n, TpPeers P, int rank, int T) {
    pdl_launch_dependents();
    pdl_wait();
    const int c = blockIdx.x, G = gridDim.x, tid = threadIdx.x;
    const int per = (n + G - 1) / G;
    const int i0 = min(n, c * per), i1 = min(n, i0 + per);
    __shared__ unsigned s_epoch;
    if (tid == 0) s_epoch = P.epoch[c] + 1;
    __syncthreads();
    const unsigned e = s_epoch;
    const size_t par = e & 1u;
    // 1. this rank's values, with the epoch, into slot [par][rank] of every other rank
    for (int r = 0; r < T; r++) {
        if (r == rank) continue;
        uint2 *dst = P.recv[r] + (par * T + rank) * (size_t)P.cap;
        for (int i = i0 + tid; i < i1; i += blockDim.x) st_cell(dst + i, x[i], e);
    }
    // 2. every rank's value of each element, summed in rank order
    const uint2 *mine = P.recv[rank] + par * T * (size_t)P.cap;
    bool bad = false;
    for (int i = i0 + tid; i < i1; i += blockDim.x) {
        float sum = 0.f;
        for (int r = 0; r < T; r++) {
            float v;
            if (r == rank) {
                v = x[i];
            } else {
                const uint2 *cell = mine + (size_t)r * P.cap + i;
                uint2 u = ld_cell(cell);
                uint64_t t0 = 0;
                for (uint32_t it = 0; u.y != e && !bad; it++) {
                    if ((it & 63) == 0) {
                        const uint64_t t = global_ns();
                        if (it == 0) t0 = t;
                        else if (t - t0 > SB_WAIT_NS) bad = true;
                    }
                    u = ld_cell(cell);
                }
                v = __uint_as_float(u.x);
            }
            sum = r == 0 ? v : __fadd_rn(sum, v);
        }
        if (bad) break;
        x[i] = sum;
    }
    if (bad) atomicOr(P.error, 1u);
    __syncthreads();  // every thread of the CTA has read x before its epoch advances
    if (tid == 0) P.epoch[c] = e;
}

}  // namespace

namespace {
// Every rank's `local` buffer mapped into this process over CUDA IPC
// (handles exchanged with an NCCL all-gather): mapped[r] is rank r's buffer
// (mapped[rank] = local).  *ok = false, with nothing left open, when some
// peer's memory cannot be mapped.
int share_buffer(const TpComm &c, void *local, cudaStream_t st, void **mapped, bool *ok) {
    const int T = c.size;
    cudaIpcMemHandle_t mine;
    SB_CUDA_TRY(cudaIpcGetMemHandle(&mine, local));
    const size_t hb = sizeof mine;
    static_assert(sizeof(mine) % 4 == 0, "handles are gathered as 32-bit words");
    uint8_t *dev = nullptr;
    SB_CUDA_TRY(cudaMalloc(&dev, hb * (T + 1)));
    std::vector<uint8_t> all(hb * T);
    int rc = SB_OK;
    if (cudaMemcpyAsync(dev + hb * T, &mine, hb, cudaMemcpyHostToDevice, st) != cudaSuccess)
        rc = set_error(SB_ERR_CUDA, "peer all-reduce: handle upload failed");
    if (rc == SB_OK) rc = tp_allgather32(c, dev + hb * T, dev, hb / 4, st);
    if (rc == SB_OK && cudaMemcpyAsync(all.data(), dev, hb * T, cudaMemcpyDeviceToHost, st) != cudaSuccess)
        rc = set_error(SB_ERR_CUDA, "peer all-reduce: handle download failed");
    if (rc == SB_OK && cudaStreamSynchronize(st) != cudaSuccess)
        rc = set_error(SB_ERR_CUDA, "peer all-reduce: handle exchange failed");
    cudaFree(dev);
    SB_TRY(rc);
    *ok = true;
    for (int r = 0; r < T; r++) mapped[r] = r == c.rank ? local : nullptr;
    for (int r = 0; r < T && *ok; r++) {
        if (r == c.rank) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, all.data() + hb * r, hb);
        if (cudaIpcOpenMemHandle(&mapped[r], h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            cudaGetLastError();
            mapped[r] = nullptr;
            *ok = false;  // no peer access between these GPUs
        }
    }
    if (!*ok)
        for (int r = 0; r < T; r++)
            if (r != c.rank && mapped[r]) cudaIpcCloseMemHandle(mapped[r]), mapped[r] = nullptr;
    return SB_OK;
}
}  // namespace

int tp_setup_p2p(TpComm &c, int cap, cudaStream_t st) {
    const int T = c.size;
    SB_CHECK(T >= 2 && T <= TP_MAX_RANKS, SB_ERR_ARG, "peer all-reduce: %d ranks", T);
    uint2 *recv = nullptr;
    unsigned *misc = nullptr;
    const size_t rbytes = sizeof(uint2) * 2 * (size_t)T * cap;
    SB_CUDA_TRY(cudaMalloc(&recv, rbytes));
    c.own[0] = recv;
    SB_CUDA_TRY(cudaMalloc(&misc, sizeof(unsigned) * (TP_AR_CTAS + 1)));
    c.own[1] = misc;
    SB_CUDA_TRY(cudaMemsetAsync(recv, 0, rbytes, st));  // epoch 0: no call has written yet
    SB_CUDA_TRY(cudaMemsetAsync(misc, 0, sizeof(unsigned) * (TP_AR_CTAS + 1), st));
    void *mapped[TP_MAX_RANKS] = {};
    bool ok = false;
    SB_TRY(share_buffer(c, recv, st, mapped, &ok));
    TpPeers P;
    P.cap = cap;
    P.epoch = misc;
    P.error = misc + TP_AR_CTAS;
    for (int r = 0; r < T; r++) P.recv[r] = static_cast<uint2 *>(mapped[r]);
    c.peers = P;
    c.p2p = ok;  // without peer access NCCL carries the sums
    return SB_OK;
}

int tp_share_cells(TpComm &c, size_t cells, cudaStream_t st, uint2 **mapped) {
    SB_CHECK(c.size >= 2 && c.size <= TP_MAX_RANKS && c.p2p, SB_ERR_UNSUPPORTED,
             "shared cells: needs peer access between %d ranks", c.size);
    SB_CHECK(!c.own[2], SB_ERR_STATE, "shared cells: already set up");
    void *buf = nullptr;
    SB_CUDA_TRY(cudaMalloc(&buf, sizeof(uint2) * cells));
    c.own[2] = buf;
    SB_CUDA_TRY(cudaMemsetAsync(buf, 0, sizeof(uint2) * cells, st));  // epoch 0: nothing written yet
    void *m[TP_MAX_RANKS] = {};
    bool ok = false;
    SB_TRY(share_buffer(c, buf, st, m, &ok));
    SB_CHECK(ok, SB_ERR_UNSUPPORTED, "shared cells: a peer's memory cannot be mapped");
    for (int r = 0; r < c.size; r++) c.cells[r] = mapped[r] = static_cast<uint2 *>(m[r]);
    return SB_OK;
}

int tp_probe_timeout(int *timed_out, double *seconds) {
    // Two ranks on this device; the cells of "rank 1" are never written, so
    // rank 0's wait for them must give up after the bound and raise the error
    // word -- no fault, no trap, the context stays usable.
    const int T = 2, cap = 1024;
    uint2 *recv = nullptr;
    unsigned *misc = nullptr;
    float *x = nullptr;
    int rc = SB_OK;
    const size_t rbytes = sizeof(uint2) * 2 * (size_t)T * cap;
    if (cudaMalloc(&recv, 2 * rbytes) != cudaSuccess || cudaMalloc(&misc, sizeof(unsigned) * (TP_AR_CTAS + 1)) !=
        cudaSuccess || cudaMalloc(&x, sizeof(float) * cap) != cudaSuccess)
        rc = set_error(SB_ERR_OOM, "peer all-reduce probe: allocation failed");
    if (rc == SB_OK && (cudaMemset(recv, 0, 2 * rbytes) != cudaSuccess ||
                        cudaMemset(misc, 0, sizeof(unsigned) * (TP_AR_CTAS + 1)) != cudaSuccess ||
                        cudaMemset(x, 0, sizeof(float) * cap) != cudaSuccess))
        rc = set_error(SB_ERR_CUDA, "peer all-reduce probe: memset failed");
    unsigned err = 0;
    if (rc == SB_OK) {
        TpPeers P;
        P.cap = cap;
        P.recv[0] = recv;                       // this rank's cells
        P.recv[1] = recv + 2 * (size_t)T * cap;  // stands for rank 1's: nothing answers
        P.epoch = misc;
        P.error = misc + TP_AR_CTAS;
        const auto t0 = std::chrono::steady_clock::now();
        tp_ar_kernel<<<1, 256>>>(x, cap, P, 0, T);
        cudaError_t e = cudaGetLastError();
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        *seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (e != cudaSuccess) rc = set_error(SB_ERR_CUDA, "peer all-reduce probe: %s", cudaGetErrorString(e));
        if (rc == SB_OK && cudaMemcpy(&err, P.error, sizeof err, cudaMemcpyDeviceToHost) != cudaSuccess)
            rc = set_error(SB_ERR_CUDA, "peer all-reduce probe: readback failed");
    }
    cudaFree(recv);
    cudaFree(misc);
    cudaFree(x);
    *timed_out = err != 0;
    return rc;
}

int tp_error_peek(const TpComm &c, unsigned *host, cudaStream_t st) {
    if (!c.p2p) {
        *host = 0;
        return SB_OK;
    }
    SB_CUDA_TRY(cudaMemcpyAsync(host, c.peers.error, sizeof(unsigned), cudaMemcpyDeviceToHost, st));
    return SB_OK;
}

int tp_check_error(const TpComm &c) {
    if (!c.p2p) return SB_OK;
    unsigned f = 0;
    SB_CUDA_TRY(cudaMemcpy(&f, c.peers.error, sizeof f, cudaMemcpyDeviceToHost));
    if (f) {
        cudaMemset(c.peers.error, 0, sizeof f);
        return set_error(SB_ERR_TIMEOUT, "peer all-reduce: a rank did not deliver its partial sums within 2 s");
    }
    return SB_OK;
}

int tp_unique_id(uint8_t *id) {
    const NcclApi &a = api();
    SB_CHECK(a.ok, SB_ERR_UNSUPPORTED, "tensor parallelism needs libnccl.so.2 (not found or incomplete)");
    ncclUniqueId u;
    ncclResult_t r = a.get_unique_id(&u);
    if (r != ncclSuccess) return nccl_fail("ncclGetUniqueId", r);
    static_assert(sizeof(u) == SB_TP_ID_BYTES, "ncclUniqueId size (sb_api.h SB_TP_ID_BYTES)");
    std::memcpy(id, &u, sizeof u);
    return SB_OK;
}

int tp_init(TpComm &c, const uint8_t *id, int rank, int size, double timeout_s) {
    const NcclApi &a = api();
    SB_CHECK(a.ok, SB_ERR_UNSUPPORTED, "tensor parallelism needs libnccl.so.2 (not found or incomplete)");
    ncclUniqueId u;
    std::memcpy(&u, id, sizeof u);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclComm_t comm = nullptr;
    ncclResult_t r = a.init_rank_config(&comm, size, u, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) return nccl_fail("ncclCommInitRankConfig", r);
    int rc = wait_comm(comm, timeout_s, "ncclCommInitRankConfig");
    if (rc != SB_OK) {
        if (comm) a.abort(comm);
        return rc;
    }
    c.comm = comm;
    c.rank = rank;
    c.size = size;
    return SB_OK;
}

void tp_destroy(TpComm &c) {
    if (c.p2p)
        for (int r = 0; r < c.size; r++)
            if (r != c.rank) cudaIpcCloseMemHandle(c.peers.recv[r]);
    for (int r = 0; r < c.size; r++)
        if (r != c.rank && c.cells[r]) cudaIpcCloseMemHandle(c.cells[r]);
    for (uint2 *&p : c.cells) p = nullptr;
    c.p2p = false;
    for (void *&p : c.own)
        if (p) cudaFree(p), p = nullptr;
    if (!c.comm) return;
    const NcclApi &a = api();
    ncclComm_t comm = (ncclComm_t)c.comm;
    ncclResult_t r = a.finalize(comm);
    if ((r == ncclSuccess || r == ncclInProgress) && wait_comm(comm, 30.0, "ncclCommFinalize") == SB_OK)
        a.destroy(comm);
    else
        a.abort(comm);
    c.comm = nullptr;
}

int tp_allreduce_f32(const TpComm &c, float *buf, size_t count, cudaStream_t st) {
    if (c.p2p && count <= (size_t)c.peers.cap) {
        // Always all TP_AR_CTAS CTAs, whatever the count: every CTA index then
        // advances its epoch on every call, so all epochs stay equal and a cell
        // left by an earlier call (possibly of another count, hence another
        // slice map) never carries the epoch a reader of this call waits for.
        SB_CUDA_TRY(launch(tp_ar_kernel, dim3(TP_AR_CTAS), dim3(256), 0, st, true, buf, (int)count, c.peers, c.rank,
                           c.size));
        return SB_OK;
    }
    const NcclApi &a = api();
    return enqueued(c, a.all_reduce(buf, buf, count, ncclFloat32, ncclSum, (ncclComm_t)c.comm, st), "ncclAllReduce");
}

int tp_allgather32(const TpComm &c, const void *send, void *recv, size_t count, cudaStream_t st) {
    const NcclApi &a = api();
    return enqueued(c, a.all_gather(send, recv, count, ncclFloat32, (ncclComm_t)c.comm, st), "ncclAllGather");
}

}  // namespace sb
