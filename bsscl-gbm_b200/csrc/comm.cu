// comm.cu -- see comm.h.
#include "comm.h"

#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <thread>

#include "../../include/gbm_b200.h"

namespace {

struct NcclApi {
    void *h = nullptr;
    ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
    ncclResult_t (*CommInitRankConfig)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*AllReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    const char *(*GetErrorString)(ncclResult_t) = nullptr;
    bool ok = false;
};

NcclApi &api() {
    static NcclApi a;
    static std::once_flag once;
    std::call_once(once, [] {
        const char *names[] = {"libnccl.so.2", "libnccl.so"};
        for (const char *nm : names) {
            a.h = dlopen(nm, RTLD_NOW | RTLD_NOLOAD);
            if (a.h) break;
        }
        for (const char *nm : names) {
            if (a.h) break;
            a.h = dlopen(nm, RTLD_NOW | RTLD_GLOBAL);
        }
        if (!a.h) return;
        a.GetUniqueId = (decltype(a.GetUniqueId))dlsym(a.h, "ncclGetUniqueId");
        a.CommInitRankConfig = (decltype(a.CommInitRankConfig))dlsym(a.h, "ncclCommInitRankConfig");
        a.CommGetAsyncError = (decltype(a.CommGetAsyncError))dlsym(a.h, "ncclCommGetAsyncError");
        a.CommAbort = (decltype(a.CommAbort))dlsym(a.h, "ncclCommAbort");
        a.CommDestroy = (decltype(a.CommDestroy))dlsym(a.h, "ncclCommDestroy");
        a.AllReduce = (decltype(a.AllReduce))dlsym(a.h, "ncclAllReduce");
        a.GetErrorString = (decltype(a.GetErrorString))dlsym(a.h, "ncclGetErrorString");
        a.ok = a.GetUniqueId && a.CommInitRankConfig && a.CommGetAsyncError && a.CommAbort &&
               a.CommDestroy && a.AllReduce && a.GetErrorString;
    });
    return a;
}

using clk = std::chrono::steady_clock;

}  // namespace

struct gbm_comm {
    ncclComm_t comm = nullptr;
    int nranks = 1, rank = 0;
    bool broken = false;
};

static int comm_fail(gbm_comm *c, std::string &err, int code, const char *what, ncclResult_t r) {
    char buf[256];
    snprintf(buf, sizeof buf, "%s: %s", what, api().ok ? api().GetErrorString(r) : "nccl unavailable");
    err = buf;
    if (c && c->comm && !c->broken) {
        api().CommAbort(c->comm);
        c->broken = true;
    }
    return code;
}

// Poll until NCCL no longer reports ncclInProgress for this communicator:
// spinning for the first 2 ms (an enqueue normally completes in
// microseconds), then every 50 us, up to the time limit.
static int wait_ready(gbm_comm *c, int timeout_ms, std::string &err, const char *what) {
    auto t0 = clk::now();
    for (int it = 0;; it++) {
        ncclResult_t st = ncclSuccess;
        ncclResult_t r = api().CommGetAsyncError(c->comm, &st);
        if (r != ncclSuccess) return comm_fail(c, err, GBM_ERR_COMM, what, r);
        if (st == ncclSuccess) return GBM_OK;
        if (st != ncclInProgress) return comm_fail(c, err, GBM_ERR_COMM, what, st);
        const auto us = std::chrono::duration_cast<std::chrono::microseconds>(clk::now() - t0).count();
        if (us > (long long)timeout_ms * 1000) return comm_fail(c, err, GBM_ERR_TIMEOUT, what, ncclInProgress);
        if (us > 2000) std::this_thread::sleep_for(std::chrono::microseconds(50));
        else std::this_thread::yield();
    }
}

int gbm_comm_unique_id(void *uid_out) {
    if (!uid_out) return GBM_ERR_ARG;
    if (!api().ok) return GBM_ERR_COMM;
    ncclUniqueId id;
    if (api().GetUniqueId(&id) != ncclSuccess) return GBM_ERR_COMM;
    static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId size");
    std::memcpy(uid_out, &id, sizeof id);
    return GBM_OK;
}

int gbm_comm_create(gbm_comm **out, const void *uid, int nranks, int rank, int timeout_ms, std::string &err) {
    *out = nullptr;
    if (!api().ok) {
        err = "libnccl.so.2 could not be loaded";
        return GBM_ERR_COMM;
    }
    gbm_comm *c = new gbm_comm();
    c->nranks = nranks;
    c->rank = rank;
    ncclUniqueId id;
    std::memcpy(&id, uid, sizeof id);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclResult_t r = api().CommInitRankConfig(&c->comm, nranks, id, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) {
        int rc = comm_fail(c, err, GBM_ERR_COMM, "ncclCommInitRankConfig", r);
        delete c;
        return rc;
    }
    int rc = wait_ready(c, timeout_ms, err, "ncclCommInitRankConfig");
    if (rc != GBM_OK) {
        delete c;
        return rc;
    }
    *out = c;
    return GBM_OK;
}

void gbm_comm_destroy(gbm_comm *c) {
    if (!c) return;
    if (c->comm) {
        if (c->broken) {
            // already aborted
        } else {
            api().CommDestroy(c->comm);
        }
    }
    delete c;
}

static int allreduce(gbm_comm *c, void *buf, int64_t count, ncclDataType_t t, cudaStream_t st, int timeout_ms,
                     std::string &err) {
    if (c->broken) {
        err = "communicator was aborted by an earlier error";
        return GBM_ERR_COMM;
    }
    ncclResult_t r = api().AllReduce(buf, buf, (size_t)count, t, ncclSum, c->comm, st);
    if (r == ncclSuccess) return GBM_OK;   // enqueued
    if (r != ncclInProgress) return comm_fail(c, err, GBM_ERR_COMM, "ncclAllReduce", r);
    return wait_ready(c, timeout_ms, err, "ncclAllReduce");
}

int gbm_comm_allreduce_i64(gbm_comm *c, long long *buf, int64_t count, cudaStream_t st, int timeout_ms,
                           std::string &err) {
    return allreduce(c, buf, count, ncclInt64, st, timeout_ms, err);
}

int gbm_comm_allreduce_f64(gbm_comm *c, double *buf, int64_t count, cudaStream_t st, int timeout_ms,
                           std::string &err) {
    return allreduce(c, buf, count, ncclFloat64, st, timeout_ms, err);
}

int gbm_comm_sync(gbm_comm *c, cudaStream_t st, int timeout_ms, std::string &err) {
    auto t0 = clk::now();
    for (;;) {
        cudaError_t e = cudaStreamQuery(st);
        if (e == cudaSuccess) return GBM_OK;
        if (e != cudaErrorNotReady) {
            err = std::string("stream error: ") + cudaGetErrorString(e);
            return GBM_ERR_CUDA;
        }
        if (c) {
            ncclResult_t s = ncclSuccess;
            if (api().CommGetAsyncError(c->comm, &s) == ncclSuccess && s != ncclSuccess && s != ncclInProgress)
                return comm_fail(c, err, GBM_ERR_COMM, "collective", s);
        }
        if (std::chrono::duration_cast<std::chrono::milliseconds>(clk::now() - t0).count() > timeout_ms) {
            if (c) return comm_fail(c, err, GBM_ERR_TIMEOUT, "stream wait (a peer may have left)", ncclInProgress);
            err = "stream wait timed out";
            return GBM_ERR_TIMEOUT;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}

int gbm_comm_wait_event(gbm_comm *c, cudaEvent_t ev, int timeout_ms, std::string &err) {
    auto t0 = clk::now();
    for (;;) {
        cudaError_t e = cudaEventQuery(ev);
        if (e == cudaSuccess) return GBM_OK;
        if (e != cudaErrorNotReady) {
            err = std::string("stream error: ") + cudaGetErrorString(e);
            return GBM_ERR_CUDA;
        }
        if (c) {
            ncclResult_t s = ncclSuccess;
            if (api().CommGetAsyncError(c->comm, &s) == ncclSuccess && s != ncclSuccess && s != ncclInProgress)
                return comm_fail(c, err, GBM_ERR_COMM, "collective", s);
        }
        if (std::chrono::duration_cast<std::chrono::milliseconds>(clk::now() - t0).count() > timeout_ms) {
            if (c) return comm_fail(c, err, GBM_ERR_TIMEOUT, "event wait (a peer may have left)", ncclInProgress);
            err = "event wait timed out";
            return GBM_ERR_TIMEOUT;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(c ? 20 : 5));
    }
}

int gbm_comm_check_alive(gbm_comm *c, int timeout_ms, std::string &err) {
    if (!c) return GBM_OK;
    if (c->broken) {
        err = "communicator was aborted by an earlier error";
        return GBM_ERR_COMM;
    }
    return wait_ready(c, timeout_ms, err, "communicator state");
}

int gbm_comm_rank(const gbm_comm *c) { return c ? c->rank : 0; }
int gbm_comm_size(const gbm_comm *c) { return c ? c->nranks : 1; }
