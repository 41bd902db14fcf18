// comm.cpp -- the one collective of row-sharded data parallelism: the sum of
// per-shard partial reductions across ranks (one process per GPU).
//
// NCCL communicator created non-blocking (ncclConfig_t.blocking = 0).
// ttc_allreduce_sum enqueues the collective on the library stream and
// returns once NCCL has accepted it: the host does not wait for it, so the
// next step's work is enqueued while this step's collective runs. Every wait
// polls against a host deadline -- communicator set-up, enqueue, and the
// completion of an outstanding collective, which the library's
// synchronisation points (sync_stream_bounded: ttc_synchronize, device ->
// host copies, the next all-reduce's enqueue check) poll for instead of
// blocking in cudaStreamSynchronize. An expired deadline or an asynchronous
// NCCL error aborts the communicator and returns TTC_ERR_TIMEOUT /
// TTC_ERR_NCCL, so a rank that died or never joined turns into an error
// status instead of a hang. No reference counterpart: the reference is
// single-process and has no collectives.
#include <cuda_runtime.h>

#include <atomic>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <thread>

#include "tt_cuda.h"

namespace ttc {
int set_error(int code, const char* fmt, ...);
int sync_stream_bounded(cudaStream_t st);
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

// An all-reduce enqueued and not yet seen complete: an event recorded right
// after the latest one (completions are in stream order, so it covers the
// earlier ones) and its host deadline (its enqueue time + its timeout).
std::atomic<bool> g_outstanding{false};
cudaEvent_t g_done = nullptr;
Clock::time_point g_deadline;
int g_timeout_ms = 0;

void abort_comm() {
    ncclCommAbort(g_comm);
    g_comm = nullptr;
    g_outstanding = false;
}

// Polls the latest all-reduce's completion against its deadline and the
// communicator's asynchronous error. TTC_OK once it completed (or when none
// is outstanding).
int wait_outstanding() {
    while (g_comm && g_outstanding) {
        const cudaError_t e = cudaEventQuery(g_done);
        if (e == cudaSuccess) {
            g_outstanding = false;
            return TTC_OK;
        }
        if (e != cudaErrorNotReady)
            return ttc::set_error(TTC_ERR_CUDA, "tt_cuda: all-reduce completion: %s", cudaGetErrorString(e));
        ncclResult_t async = ncclSuccess;
        ncclCommGetAsyncError(g_comm, &async);
        if (async != ncclSuccess && async != ncclInProgress) {
            abort_comm();
            return ttc::set_error(TTC_ERR_NCCL, "tt_cuda: all-reduce failed: %s", ncclGetErrorString(async));
        }
        if (Clock::now() > g_deadline) {
            abort_comm();
            return ttc::set_error(TTC_ERR_TIMEOUT, "tt_cuda: all-reduce did not complete within %d ms; aborted",
                                  g_timeout_ms);
        }
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
    return TTC_OK;
}

// Polls the communicator's async state until it leaves ncclInProgress.
int wait_comm(int timeout_ms, const char* what) {
    const auto deadline = Clock::now() + std::chrono::milliseconds(timeout_ms);
    for (;;) {
        ncclResult_t st = ncclSuccess;
        ncclResult_t r = ncclCommGetAsyncError(g_comm, &st);
        if (r != ncclSuccess) st = r;
        if (st == ncclSuccess) return TTC_OK;
        if (st != ncclInProgress) {
            abort_comm();
            return ttc::set_error(TTC_ERR_NCCL, "tt_cuda: %s failed: %s", what, ncclGetErrorString(st));
        }
        if (Clock::now() > deadline) {
            abort_comm();
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
    if (int rc = wait_comm(timeout_ms, "communicator initialisation")) return rc;
    if (!g_done && cudaEventCreateWithFlags(&g_done, cudaEventDisableTiming) != cudaSuccess) {
        abort_comm();
        return ttc::set_error(TTC_ERR_CUDA, "tt_cuda: all-reduce completion event could not be created");
    }
    return TTC_OK;
}

int ttc_allreduce_sum(float* buf, size_t count, int timeout_ms) {
    if (inject_fault("allreduce")) return ttc::set_error(TTC_ERR_NCCL, "tt_cuda: injected all-reduce fault");
    if (!g_comm) return ttc::set_error(TTC_ERR_NOT_INITIALIZED, "tt_cuda: ttc_comm_init() not called");
    if (!buf && count) return ttc::set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: allreduce buffer is NULL");
    if (timeout_ms <= 0) return ttc::set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: all-reduce timeout %d ms", timeout_ms);
    // an earlier collective that failed asynchronously is reported here,
    // before another one is queued behind it
    ncclResult_t async = ncclSuccess;
    ncclCommGetAsyncError(g_comm, &async);
    if (async != ncclSuccess && async != ncclInProgress) {
        abort_comm();
        return ttc::set_error(TTC_ERR_NCCL, "tt_cuda: an earlier all-reduce failed: %s", ncclGetErrorString(async));
    }
    if (g_outstanding && cudaEventQuery(g_done) == cudaErrorNotReady && Clock::now() > g_deadline) {
        abort_comm();
        return ttc::set_error(TTC_ERR_TIMEOUT, "tt_cuda: an earlier all-reduce did not complete within %d ms; aborted",
                              g_timeout_ms);
    }
    cudaStream_t st = (cudaStream_t)ttc_get_stream();
    ncclResult_t r = ncclAllReduce(buf, buf, count, ncclFloat32, ncclSum, g_comm, st);
    if (r != ncclSuccess && r != ncclInProgress) {
        abort_comm();
        return ttc::set_error(TTC_ERR_NCCL, "tt_cuda: ncclAllReduce: %s", ncclGetErrorString(r));
    }
    if (int rc = wait_comm(timeout_ms, "all-reduce enqueue")) return rc;
    // Not waited for here: the next synchronisation point polls for it
    // against this deadline (sync_stream_bounded).
    if (cudaEventRecord(g_done, st) != cudaSuccess) {
        abort_comm();
        return ttc::set_error(TTC_ERR_CUDA, "tt_cuda: all-reduce completion event record failed");
    }
    g_timeout_ms = timeout_ms;
    g_deadline = Clock::now() + std::chrono::milliseconds(timeout_ms);
    g_outstanding = true;
    return TTC_OK;
}

int ttc_comm_destroy(void) {
    if (!g_comm) return TTC_OK;
    if (wait_outstanding() != TTC_OK) return TTC_OK;  // a queued collective that never finished: aborted
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
    abort_comm();
    return TTC_OK;
}

}  // extern "C"

namespace ttc {
// Waits for the work queued on `st`. An outstanding all-reduce is waited for
// first, by polling its completion event against its host deadline and the
// communicator's asynchronous error (a peer that died leaves the collective
// spinning on this GPU; the abort releases it); everything else on the stream
// then finishes on its own.
int sync_stream_bounded(cudaStream_t st) {
    if (int rc = wait_outstanding()) return rc;  // the only work here that can wait on another rank
    const cudaError_t e = cudaStreamSynchronize(st);
    if (e != cudaSuccess)
        return set_error(TTC_ERR_CUDA, "tt_cuda: cudaStreamSynchronize failed: %s", cudaGetErrorString(e));
    return TTC_OK;
}
}  // namespace ttc

#else  // built without NCCL headers

extern "C" {
int ttc_comm_unique_id(uint8_t*) { return ttc::set_error(TTC_ERR_UNSUPPORTED, "tt_cuda: built without NCCL"); }
int ttc_comm_init(int, int, const uint8_t*, int) {
    return ttc::set_error(TTC_ERR_UNSUPPORTED, "tt_cuda: built without NCCL");
}
int ttc_allreduce_sum(float*, size_t, int) { return ttc::set_error(TTC_ERR_UNSUPPORTED, "tt_cuda: built without NCCL"); }
int ttc_comm_destroy(void) { return TTC_OK; }
}
namespace ttc {
int sync_stream_bounded(cudaStream_t st) {
    const cudaError_t e = cudaStreamSynchronize(st);
    if (e != cudaSuccess)
        return set_error(TTC_ERR_CUDA, "tt_cuda: cudaStreamSynchronize failed: %s", cudaGetErrorString(e));
    return TTC_OK;
}
}  // namespace ttc
#endif
