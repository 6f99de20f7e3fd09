// comm.h -- NCCL plumbing of the engine (row-sharded data parallelism).
//
// NCCL is loaded at run time (dlopen of libnccl.so.2, reusing a copy the
// process already holds, e.g. PyTorch's), so single-GPU use needs no NCCL.
// The communicator is non-blocking: creation and every wait poll with a
// time limit, and a limit that runs out aborts the communicator and returns
// GBM_ERR_TIMEOUT instead of hanging the process.
#pragma once
#include <cuda_runtime.h>
#include <cstdint>
#include <string>

struct gbm_comm;

int gbm_comm_unique_id(void *uid_out);
int gbm_comm_create(gbm_comm **out, const void *uid, int nranks, int rank, int timeout_ms, std::string &err);
void gbm_comm_destroy(gbm_comm *c);
// In-place sums on `st`; they only enqueue (plus bounded polling while NCCL
// reports the call in progress).
int gbm_comm_allreduce_i64(gbm_comm *c, long long *buf, int64_t count, cudaStream_t st, int timeout_ms,
                           std::string &err);
int gbm_comm_allreduce_f64(gbm_comm *c, double *buf, int64_t count, cudaStream_t st, int timeout_ms,
                           std::string &err);
// Bounded stream synchronisation that also watches the communicator.
int gbm_comm_sync(gbm_comm *c, cudaStream_t st, int timeout_ms, std::string &err);
// The same for one event (c may be NULL: a bounded wait only).
int gbm_comm_wait_event(gbm_comm *c, cudaEvent_t ev, int timeout_ms, std::string &err);
int gbm_comm_check_alive(gbm_comm *c, int timeout_ms, std::string &err);
int gbm_comm_rank(const gbm_comm *c);
int gbm_comm_size(const gbm_comm *c);
