// Tensor-parallel communicator of the engine: an NCCL communicator over the
// GPUs of one node (NVLink / NVSwitch), loaded at run time.
//
// libscryb200.so does not link NCCL: the first tensor-parallel call opens
// libnccl.so.2 with dlopen (the copy a host process such as torch already
// loaded, else the system one) and resolves the handful of entry points it
// uses.  Communicators are created non-blocking and every wait on them is
// bounded, so a rank that never joins turns into SB_ERR_TIMEOUT (and an
// aborted communicator) instead of a hang.
#pragma once

#include "sb_common.cuh"

namespace sb {

constexpr int TP_MAX_RANKS = 8;
constexpr int TP_AR_CTAS = 32;  // CTAs (and flag slots per source rank) of the peer all-reduce

// Peer-memory all-reduce state.  Every rank owns recv[2][T][cap] 8-byte
// cells (value bits, epoch) in its own HBM; the other ranks write into them
// over NVLink through IPC mappings.  epoch[TP_AR_CTAS] counts the calls each
// CTA index has made on this rank (the same on every rank, since all ranks
// make the same calls).
struct TpPeers {
    uint2 *recv[TP_MAX_RANKS] = {};  // rank r's receive cells, mapped here
    unsigned *epoch = nullptr;       // local
    unsigned *error = nullptr;       // local: a wait that ran out
    int cap = 0;                     // cells per (parity, source) slot
};

struct TpComm {
    void *comm = nullptr;  // ncclComm_t
    int rank = 0, size = 1;
    TpPeers peers;
    bool p2p = false;                    // peer all-reduce usable
    void *own[3] = {};                   // local allocations (recv, epoch+error, shared cells)
    uint2 *cells[TP_MAX_RANKS] = {};     // tp_share_cells: rank r's cells, mapped here
};

// A cell is one aligned 64-bit word (epoch << 32 | value bits): scalar 64-bit
// accesses are single-copy atomic, so a reader sees a value only together
// with the epoch it was written for.
__device__ __forceinline__ void st_cell(uint2 *p, float v, unsigned e) {
    const unsigned long long w = ((unsigned long long)e << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ void st_cell_u(uint2 *p, unsigned v, unsigned e) {
    const unsigned long long w = ((unsigned long long)e << 32) | v;
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ uint2 ld_cell(const uint2 *p) {
    unsigned long long w;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return make_uint2((unsigned)w, (unsigned)(w >> 32));
}

// Fresh unique id for a new communicator (rank 0 makes it, the caller sends
// it to the other ranks).
int tp_unique_id(uint8_t *id);
// Join the communicator of `size` ranks; gives up after timeout_s seconds.
int tp_init(TpComm &c, const uint8_t *id, int rank, int size, double timeout_s);
void tp_destroy(TpComm &c);
// Sum of `count` f32 values over the ranks, in place, on `st` (capturable):
// the peer all-reduce when it is set up and count fits, else NCCL.  Every
// rank receives the same sum (added in rank order).
int tp_allreduce_f32(const TpComm &c, float *buf, size_t count, cudaStream_t st);
// Map every rank's all-reduce buffers (cap floats per slot) into this
// process over CUDA IPC (handles exchanged with an NCCL all-gather).  Leaves
// p2p off (NCCL only) when the GPUs cannot reach each other's memory.
int tp_setup_p2p(TpComm &c, int cap, cudaStream_t st);
// `cells` zeroed 8-byte cells in this rank's memory, mapped into every rank:
// afterwards c.cells[r] (= mapped[r]) is rank r's array.  Needs peer access
// (tp_setup_p2p found it); SB_ERR_UNSUPPORTED otherwise.  Once per comm.
int tp_share_cells(TpComm &c, size_t cells, cudaStream_t st, uint2 **mapped);
// Queues a copy of the peer exchanges' error word into *host (pinned) on st.
int tp_error_peek(const TpComm &c, unsigned *host, cudaStream_t st);
// Reports (and clears) a timed-out flag wait of the peer all-reduce.
int tp_check_error(const TpComm &c);
// Runs the peer all-reduce against a peer that never writes (one device);
// *timed_out = 1 when its bounded wait gave up and raised the error word.
int tp_probe_timeout(int *timed_out, double *seconds);
// recv[r * count + i] = send_r[i], on `st` (capturable); elem_bytes 4.
int tp_allgather32(const TpComm &c, const void *send, void *recv, size_t count, cudaStream_t st);

}  // namespace sb
