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

struct TpComm {
    void *comm = nullptr;  // ncclComm_t
    int rank = 0, size = 1;
};

// Fresh unique id for a new communicator (rank 0 makes it, the caller sends
// it to the other ranks).
int tp_unique_id(uint8_t *id);
// Join the communicator of `size` ranks; gives up after timeout_s seconds.
int tp_init(TpComm &c, const uint8_t *id, int rank, int size, double timeout_s);
void tp_destroy(TpComm &c);
// Sum of `count` f32 values over the ranks, in place, on `st` (capturable).
int tp_allreduce_f32(const TpComm &c, float *buf, size_t count, cudaStream_t st);
// recv[r * count + i] = send_r[i], on `st` (capturable); elem_bytes 4.
int tp_allgather32(const TpComm &c, const void *send, void *recv, size_t count, cudaStream_t st);

}  // namespace sb
