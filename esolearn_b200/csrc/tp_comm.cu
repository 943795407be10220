// NCCL communicator of the tensor-parallel engine, resolved with dlopen.
#include "tp_comm.cuh"

#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
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

}  // namespace

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
    const NcclApi &a = api();
    return enqueued(c, a.all_reduce(buf, buf, count, ncclFloat32, ncclSum, (ncclComm_t)c.comm, st), "ncclAllReduce");
}

int tp_allgather32(const TpComm &c, const void *send, void *recv, size_t count, cudaStream_t st) {
    const NcclApi &a = api();
    return enqueued(c, a.all_gather(send, recv, count, ncclFloat32, (ncclComm_t)c.comm, st), "ncclAllGather");
}

}  // namespace sb
