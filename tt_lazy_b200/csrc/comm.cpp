// comm.cpp -- the one collective of row-sharded data parallelism: the sum of
// per-shard partial reductions across ranks (one process per GPU).
//
// NCCL communicator created non-blocking (ncclConfig_t.blocking = 0). Every
// wait -- communicator set-up, enqueue, completion on the stream -- polls
// against a host deadline; an expired deadline aborts the communicator and
// returns TTC_ERR_TIMEOUT, so a rank that died or never joined turns into an
// error status instead of a hang. No reference counterpart: the reference is
// single-process and has no collectives.
#include <cuda_runtime.h>

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <thread>

#include "tt_cuda.h"

namespace ttc {
int set_error(int code, const char* fmt, ...);
}

namespace {
// Host-side fault injection for the failure-handling tests: with
// TTC_COMM_FAULT=init (or allreduce) set, that call fails with TTC_ERR_NCCL
// before it touches NCCL or the GPU, as a failing library call would.
bool inject_fault(const char* call) {
    const char* e = std::getenv("TTC_COMM_FAULT");
    return e && std::strcmp(e, call) == 0;
}
}  // namespace

#if TTC_HAVE_NCCL
#include <nccl.h>

namespace {
ncclComm_t g_comm = nullptr;

using Clock = std::chrono::steady_clock;

// Polls the communicator's async state until it leaves ncclInProgress.
int wait_comm(int timeout_ms, const char* what) {
    const auto deadline = Clock::now() + std::chrono::milliseconds(timeout_ms);
    for (;;) {
        ncclResult_t st = ncclSuccess;
        ncclResult_t r = ncclCommGetAsyncError(g_comm, &st);
        if (r != ncclSuccess) st = r;
        if (st == ncclSuccess) return TTC_OK;
        if (st != ncclInProgress) {
            ncclCommAbort(g_comm);
            g_comm = nullptr;
            return ttc::set_error(TTC_ERR_NCCL, "tt_cuda: %s failed: %s", what, ncclGetErrorString(st));
        }
        if (Clock::now() > deadline) {
            ncclCommAbort(g_comm);
            g_comm = nullptr;
            return ttc::set_error(TTC_ERR_TIMEOUT, "tt_cuda: %s did not complete within %d ms; communicator aborted",
                                  what, timeout_ms);
        }
        std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}
}  // namespace

extern "C" {

int ttc_comm_unique_id(uint8_t out[TTC_UNIQUE_ID_BYTES]) {
    static_assert(sizeof(ncclUniqueId) == TTC_UNIQUE_ID_BYTES, "ncclUniqueId size");
    ncclUniqueId id;
    ncclResult_t r = ncclGetUniqueId(&id);
    if (r != ncclSuccess) return ttc::set_error(TTC_ERR_NCCL, "tt_cuda: ncclGetUniqueId: %s", ncclGetErrorString(r));
    std::memcpy(out, &id, sizeof id);
    return TTC_OK;
}

int ttc_comm_init(int nranks, int rank, const uint8_t id[TTC_UNIQUE_ID_BYTES], int timeout_ms) {
    if (inject_fault("init")) return ttc::set_error(TTC_ERR_NCCL, "tt_cuda: injected communicator init fault");
    if (g_comm) return ttc::set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: communicator already initialised");
    if (nranks < 1 || rank < 0 || rank >= nranks || !id || timeout_ms <= 0)
        return ttc::set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: comm_init(nranks=%d, rank=%d, timeout=%d)", nranks,
                              rank, timeout_ms);
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof uid);
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;
    ncclResult_t r = ncclCommInitRankConfig(&g_comm, nranks, uid, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) {
        g_comm = nullptr;
        return ttc::set_error(TTC_ERR_NCCL, "tt_cuda: ncclCommInitRankConfig: %s", ncclGetErrorString(r));
    }
    return wait_comm(timeout_ms, "communicator initialisation");
}

int ttc_allreduce_sum(float* buf, size_t count, int timeout_ms) {
    if (inject_fault("allreduce")) return ttc::set_error(TTC_ERR_NCCL, "tt_cuda: injected all-reduce fault");
    if (!g_comm) return ttc::set_error(TTC_ERR_NOT_INITIALIZED, "tt_cuda: ttc_comm_init() not called");
    if (!buf && count) return ttc::set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: allreduce buffer is NULL");
    cudaStream_t st = (cudaStream_t)ttc_get_stream();
    ncclResult_t r = ncclAllReduce(buf, buf, count, ncclFloat32, ncclSum, g_comm, st);
    if (r != ncclSuccess && r != ncclInProgress) {
        ncclCommAbort(g_comm);
        g_comm = nullptr;
        return ttc::set_error(TTC_ERR_NCCL, "tt_cuda: ncclAllReduce: %s", ncclGetErrorString(r));
    }
    if (int rc = wait_comm(timeout_ms, "all-reduce enqueue")) return rc;
    // Completion on the stream, bounded by the same deadline.
    const auto deadline = Clock::now() + std::chrono::milliseconds(timeout_ms);
    for (;;) {
        cudaError_t e = cudaStreamQuery(st);
        if (e == cudaSuccess) break;
        if (e != cudaErrorNotReady)
            return ttc::set_error(TTC_ERR_CUDA, "tt_cuda: all-reduce stream: %s", cudaGetErrorString(e));
        ncclResult_t async = ncclSuccess;
        ncclCommGetAsyncError(g_comm, &async);
        if (async != ncclSuccess && async != ncclInProgress) {
            ncclCommAbort(g_comm);
            g_comm = nullptr;
            return ttc::set_error(TTC_ERR_NCCL, "tt_cuda: all-reduce failed: %s", ncclGetErrorString(async));
        }
        if (Clock::now() > deadline) {
            ncclCommAbort(g_comm);
            g_comm = nullptr;
            return ttc::set_error(TTC_ERR_TIMEOUT, "tt_cuda: all-reduce did not complete within %d ms; aborted",
                                  timeout_ms);
        }
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
    return TTC_OK;
}

int ttc_comm_destroy(void) {
    if (!g_comm) return TTC_OK;
    ncclResult_t r = ncclCommFinalize(g_comm);
    if (r == ncclSuccess || r == ncclInProgress) {
        const auto deadline = Clock::now() + std::chrono::milliseconds(10000);
        ncclResult_t st = ncclInProgress;
        while (st == ncclInProgress && Clock::now() < deadline) {
            ncclCommGetAsyncError(g_comm, &st);
            if (st == ncclInProgress) std::this_thread::sleep_for(std::chrono::microseconds(100));
        }
        if (st == ncclSuccess) {
            ncclCommDestroy(g_comm);
            g_comm = nullptr;
            return TTC_OK;
        }
    }
    ncclCommAbort(g_comm);
    g_comm = nullptr;
    return TTC_OK;
}

}  // extern "C"

#else  // built without NCCL headers

extern "C" {
int ttc_comm_unique_id(uint8_t*) { return ttc::set_error(TTC_ERR_UNSUPPORTED, "tt_cuda: built without NCCL"); }
int ttc_comm_init(int, int, const uint8_t*, int) {
    return ttc::set_error(TTC_ERR_UNSUPPORTED, "tt_cuda: built without NCCL");
}
int ttc_allreduce_sum(float*, size_t, int) { return ttc::set_error(TTC_ERR_UNSUPPORTED, "tt_cuda: built without NCCL"); }
int ttc_comm_destroy(void) { return TTC_OK; }
}
#endif
