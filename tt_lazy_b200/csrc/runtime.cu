// runtime.cu -- tt_cuda_lib runtime: error state, device/stream selection,
// stream-ordered device memory (the replacement of the reference's host
// MemoryPool, src/core/MemoryManager.cpp:46-133), copies, the internal
// workspace, and decoding of element-wise programs.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <unordered_map>

#include <nvtx3/nvToolsExt.h>

#include "tma_util.cuh"

namespace ttc {

namespace {
thread_local std::string g_last_error;
Runtime g_rt;
std::unordered_map<void*, size_t> g_sizes;  // live ttc_malloc blocks (stats)
}  // namespace

Runtime& rt() { return g_rt; }

int set_error(int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

void clear_error() { g_last_error.clear(); }

int check_cuda(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return TTC_OK;
    const int code = (e == cudaErrorMemoryAllocation) ? TTC_ERR_OUT_OF_MEMORY : TTC_ERR_CUDA;
    return set_error(code, "tt_cuda: %s failed: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

int workspace(size_t bytes, void** out) {
    Runtime& r = rt();
    if (bytes > r.workspace_bytes) {
        if (r.workspace) {
            // The old buffer may still be read by queued kernels: free in stream order.
            TTC_CUDA(cudaFreeAsync(r.workspace, r.stream));
            r.workspace = nullptr;
            r.workspace_bytes = 0;
        }
        size_t want = bytes < (1u << 20) ? (1u << 20) : bytes;
        TTC_CUDA(cudaMallocAsync(&r.workspace, want, r.stream));
        r.workspace_bytes = want;
    }
    *out = r.workspace;
    return TTC_OK;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int encode_tensor_map_f32(CUtensorMap* map, const void* ptr, int rank, const unsigned long long* dims,
                          const unsigned long long* strides_elems, const unsigned* box, CUtensorMapSwizzle swizzle) {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiledFn)p;
        else
            cudaGetLastError();
        if (!fn) return set_error(TTC_ERR_CUDA, "tt_cuda: cuTensorMapEncodeTiled is unavailable");
    }
    if (rank < 1 || rank > 5) return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: tensor map rank %d", rank);
    cuuint64_t d[5], s[4];
    cuuint32_t b[5], e[5];
    for (int i = 0; i < rank; ++i) {
        d[i] = dims[i];
        b[i] = box[i];
        e[i] = 1;
        if (i + 1 < rank) s[i] = strides_elems[i] * 4;
    }
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, (cuuint32_t)rank, const_cast<void*>(ptr), d, s, b, e,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS)
        return set_error(TTC_ERR_CUDA, "tt_cuda: cuTensorMapEncodeTiled failed (%d): rank %d, dims %llu x %llu", (int)r,
                         rank, (unsigned long long)d[0], rank > 1 ? (unsigned long long)d[1] : 1ull);
    return TTC_OK;
}

// A host-mapped status word that kernels with bounded waits set when a wait
// expires. The host reads it after every synchronisation.
namespace {
int* g_status_host = nullptr;
int* g_status_dev = nullptr;
}  // namespace

int device_status_ptr(int** dptr) {
    if (!g_status_host) {
        TTC_CUDA(cudaHostAlloc((void**)&g_status_host, sizeof(int), cudaHostAllocMapped));
        *g_status_host = 0;
        TTC_CUDA(cudaHostGetDevicePointer((void**)&g_status_dev, g_status_host, 0));
    }
    *dptr = g_status_dev;
    return TTC_OK;
}

bool stall_test(const char* family) {
    const char* e = getenv("TTC_TEST_STALL");
    return e && std::strcmp(e, family) == 0;
}

// After a synchronisation: turn a recorded device-side wait expiry into an error.
int check_device_status() {
    if (g_status_host && *(volatile int*)g_status_host) {
        *(volatile int*)g_status_host = 0;
        return set_error(TTC_ERR_TIMEOUT,
                         "tt_cuda: a kernel's bounded wait expired (pipeline stalled); its output is invalid");
    }
    return TTC_OK;
}

FastDiv make_fastdiv(unsigned d) {
    FastDiv f{d, 0, 0};
    unsigned s = 0;
    while ((1ull << s) < d) ++s;
    f.s = s;
    f.m = (unsigned)((((1ull << 32) * ((1ull << s) - d)) / d) + 1);
    return f;
}

int decode_program(const ttc_chain_desc& d, bool acc_preloaded, DProgram* out) {
    std::memset(out, 0, sizeof *out);
    if (d.n_instr < 0 || d.n_instr > TTC_CHAIN_MAX_INSTR)
        return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: program length %d outside [0, %d]", d.n_instr,
                         TTC_CHAIN_MAX_INSTR);
    if (d.n_inputs < 0 || d.n_inputs > TTC_CHAIN_MAX_INPUTS || d.n_outputs < 0 ||
        d.n_outputs > TTC_CHAIN_MAX_OUTPUTS)
        return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: %d inputs / %d outputs exceed %d / %d", d.n_inputs,
                         d.n_outputs, TTC_CHAIN_MAX_INPUTS, TTC_CHAIN_MAX_OUTPUTS);
    out->n_instr = d.n_instr;
    out->n_in = d.n_inputs;
    out->n_out = d.n_outputs;
    for (int i = 0; i < d.n_inputs; ++i) {
        const ttc_in_view& v = d.inputs[i];
        if (!v.ptr) return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: input %d is NULL", i);
        if (v.col_stride != 0 && v.col_stride != 1)
            return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: input %d col_stride %lld not 0 or 1", i,
                             (long long)v.col_stride);
        if (v.row_stride < 0 || v.seg_stride < 0)
            return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: input %d has a negative stride", i);
        out->in[i] = DInView{v.ptr, v.row_stride, v.col_stride, v.seg_stride};
    }
    for (int i = 0; i < d.n_outputs; ++i) {
        const ttc_out_view& v = d.outputs[i];
        if (!v.ptr) return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: output %d is NULL", i);
        if (v.row_stride < 0 || v.seg_stride < 0)
            return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: output %d has a negative stride", i);
        out->out[i] = DOutView{v.ptr, v.row_stride, v.seg_stride};
    }
    bool acc_defined = acc_preloaded;
    bool slot_defined[TTC_CHAIN_SLOTS] = {false, false, false, false};
    for (int pc = 0; pc < d.n_instr; ++pc) {
        const ttc_instr& in = d.program[pc];
        uint8_t op = 0, arg = 0;
        auto need_acc = [&]() -> int {
            if (!acc_defined)
                return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: step %d reads acc before any LOAD", pc);
            return TTC_OK;
        };
        switch (in.op) {
            case TTC_OP_LOAD:
                if (in.src == TTC_SRC_SLOT) {
                    if (in.idx >= TTC_CHAIN_SLOTS || !slot_defined[in.idx])
                        return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: step %d loads unset slot %d", pc,
                                         in.idx);
                    op = (uint8_t)(D_LOAD_S0 + in.idx);
                    acc_defined = true;
                    break;
                }
                if (in.idx >= d.n_inputs)
                    return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: step %d loads input %d of %d", pc, in.idx,
                                     d.n_inputs);
                op = D_LOAD;
                arg = in.idx;
                acc_defined = true;
                break;
            case TTC_OP_RELU:
            case TTC_OP_SIGMOID:
                if (int rc = need_acc()) return rc;
                op = in.op == TTC_OP_RELU ? D_RELU : D_SIGMOID;
                if (op == D_SIGMOID) out->has_sigmoid = 1;
                break;
            case TTC_OP_ADD:
            case TTC_OP_MUL: {
                if (int rc = need_acc()) return rc;
                const bool add = in.op == TTC_OP_ADD;
                if (in.src == TTC_SRC_ACC) {
                    op = add ? D_ADD_ACC : D_MUL_ACC;
                } else if (in.src == TTC_SRC_INPUT) {
                    if (in.idx >= d.n_inputs)
                        return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: step %d reads input %d of %d", pc,
                                         in.idx, d.n_inputs);
                    op = add ? D_ADD_IN : D_MUL_IN;
                    arg = in.idx;
                } else if (in.src == TTC_SRC_SLOT) {
                    if (in.idx >= TTC_CHAIN_SLOTS || !slot_defined[in.idx])
                        return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: step %d reads unset slot %d", pc,
                                         in.idx);
                    op = (uint8_t)((add ? D_ADD_S0 : D_MUL_S0) + in.idx);
                } else {
                    return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: step %d has source kind %d", pc, in.src);
                }
                break;
            }
            case TTC_OP_SAVE:
                if (int rc = need_acc()) return rc;
                if (in.idx >= TTC_CHAIN_SLOTS)
                    return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: step %d saves to slot %d", pc, in.idx);
                op = (uint8_t)(D_SAVE0 + in.idx);
                slot_defined[in.idx] = true;
                if (in.idx + 1 > out->n_slots) out->n_slots = in.idx + 1;
                break;
            case TTC_OP_STORE:
                if (int rc = need_acc()) return rc;
                if (in.idx >= d.n_outputs)
                    return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: step %d stores to output %d of %d", pc,
                                     in.idx, d.n_outputs);
                op = D_STORE;
                arg = in.idx;
                break;
            default:
                return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: step %d has unknown opcode %d", pc, in.op);
        }
        out->op[pc] = op;
        out->arg[pc] = arg;
    }
    if (!acc_defined && d.reduce != TTC_REDUCE_NONE)
        return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: reduction of a program that never loads");
    return TTC_OK;
}

}  // namespace ttc

using namespace ttc;

extern "C" {

const char* ttc_last_error(void) { return g_last_error.c_str(); }

int ttc_version(void) { return (0 << 16) | 1; }

int ttc_device_count(int* count) {
    if (!count) return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: count is NULL");
    cudaError_t e = cudaGetDeviceCount(count);
    if (e != cudaSuccess) {
        *count = 0;
        cudaGetLastError();
        return check_cuda(e, "cudaGetDeviceCount");
    }
    return TTC_OK;
}

int ttc_init(int device) {
    Runtime& r = rt();
    if (r.initialized) {
        if (r.device == device) return TTC_OK;
        return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: already initialised on device %d (asked %d)",
                         r.device, device);
    }
    int n = 0;
    TTC_CUDA(cudaGetDeviceCount(&n));
    if (device < 0 || device >= n)
        return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: device %d outside [0, %d)", device, n);
    TTC_CUDA(cudaSetDevice(device));
    cudaDeviceProp prop;
    TTC_CUDA(cudaGetDeviceProperties(&prop, device));
    if (prop.major != 10)
        return set_error(TTC_ERR_UNSUPPORTED, "tt_cuda: device %d is sm_%d%d; this build targets sm_100a (B200)",
                         device, prop.major, prop.minor);
    r.sm_count = prop.multiProcessorCount;
    TTC_CUDA(cudaStreamCreateWithFlags(&r.own_stream, cudaStreamNonBlocking));
    r.stream = r.own_stream;
    // Keep freed pool memory cached in the process: the tape frees and
    // re-allocates the same sizes every evaluation.
    cudaMemPool_t pool;
    TTC_CUDA(cudaDeviceGetDefaultMemPool(&pool, device));
    uint64_t threshold = UINT64_MAX;
    TTC_CUDA(cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &threshold));
    r.device = device;
    r.initialized = true;
    return TTC_OK;
}

int ttc_shutdown(void) {
    Runtime& r = rt();
    if (!r.initialized) return TTC_OK;
    sync_stream_bounded(r.stream);  // an outstanding all-reduce is waited for against its deadline
    if (r.copy_stream) {
        cudaStreamSynchronize(r.copy_stream);
        for (auto& e : r.tickets)
            if (e) cudaEventDestroy(e), e = nullptr;
        cudaStreamDestroy(r.copy_stream);
        r.copy_stream = nullptr;
    }
    if (r.workspace) cudaFree(r.workspace);
    r.workspace = nullptr;
    r.workspace_bytes = 0;
    if (r.own_stream) cudaStreamDestroy(r.own_stream);
    r.own_stream = r.stream = nullptr;
    r.initialized = false;
    r.device = -1;
    return TTC_OK;
}

void* ttc_get_stream(void) { return (void*)rt().stream; }

int ttc_set_stream(void* s) {
    TTC_REQUIRE_INIT();
    rt().stream = s ? (cudaStream_t)s : rt().own_stream;
    return TTC_OK;
}

int ttc_synchronize(void) {
    TTC_REQUIRE_INIT();
    if (int rc = sync_stream_bounded(rt().stream)) return rc;
    return check_device_status();
}

int ttc_malloc(size_t bytes, void** dptr) {
    TTC_REQUIRE_INIT();
    if (!dptr) return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: dptr is NULL");
    *dptr = nullptr;
    if (bytes == 0) return TTC_OK;
    // Round to 256 B so every buffer is TMA- and float4-aligned.
    size_t sz = (bytes + 255) & ~(size_t)255;
    cudaError_t e = cudaMallocAsync(dptr, sz, rt().stream);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return set_error(e == cudaErrorMemoryAllocation ? TTC_ERR_OUT_OF_MEMORY : TTC_ERR_CUDA,
                         "tt_cuda: cannot allocate %zu bytes of device memory: %s", bytes, cudaGetErrorString(e));
    }
    Runtime& r = rt();
    g_sizes[*dptr] = sz;
    r.bytes_in_use += sz;
    if (r.bytes_in_use > r.peak_bytes) r.peak_bytes = r.bytes_in_use;
    return TTC_OK;
}

int ttc_free(void* dptr) {
    TTC_REQUIRE_INIT();
    if (!dptr) return TTC_OK;
    auto it = g_sizes.find(dptr);
    if (it == g_sizes.end())
        return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: ttc_free of %p, which ttc_malloc did not return", dptr);
    TTC_CUDA(cudaFreeAsync(dptr, rt().stream));
    rt().bytes_in_use -= it->second;
    g_sizes.erase(it);
    return TTC_OK;
}

int ttc_memcpy_h2d(void* dst, const void* src, size_t bytes) {
    TTC_REQUIRE_INIT();
    if (bytes == 0) return TTC_OK;
    TTC_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, rt().stream));
    return TTC_OK;
}

// Copies on a second stream so that they overlap kernels on the library
// stream. The copy stream first waits for everything already enqueued on the
// library stream, so a prefetch never overwrites a buffer that earlier
// kernels still read; ttc_wait_ticket then orders later kernels after it.
int ttc_h2d_prefetch(void* dst, const void* src, size_t bytes, int* ticket) {
    TTC_REQUIRE_INIT();
    if (!ticket || (!dst && bytes) || (!src && bytes))
        return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: h2d_prefetch: null argument");
    Runtime& r = rt();
    if (!r.copy_stream) {
        TTC_CUDA(cudaStreamCreateWithFlags(&r.copy_stream, cudaStreamNonBlocking));
        for (auto& e : r.tickets) TTC_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    }
    const unsigned t = r.next_ticket++ % 256u;
    TTC_CUDA(cudaEventRecord(r.tickets[t], r.stream));
    TTC_CUDA(cudaStreamWaitEvent(r.copy_stream, r.tickets[t], 0));
    if (bytes) TTC_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, r.copy_stream));
    TTC_CUDA(cudaEventRecord(r.tickets[t], r.copy_stream));
    *ticket = (int)t;
    return TTC_OK;
}

int ttc_wait_ticket(int ticket) {
    TTC_REQUIRE_INIT();
    Runtime& r = rt();
    if (ticket < 0 || ticket >= 256 || !r.copy_stream)
        return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: wait_ticket: no prefetch %d", ticket);
    TTC_CUDA(cudaStreamWaitEvent(r.stream, r.tickets[ticket], 0));
    return TTC_OK;
}

// ------------------------------------------------------------ tracing
// NVTX ranges (visible to any attached profiler; no-ops otherwise) and
// CUDA-event marks on the library stream, from a ring of 4096 events.
namespace {
cudaEvent_t g_marks[4096] = {};
unsigned g_next_mark = 0;
}  // namespace

int ttc_range_push(const char* name) {
    nvtxRangePushA(name ? name : "");
    return TTC_OK;
}

int ttc_range_pop(void) {
    nvtxRangePop();
    return TTC_OK;
}

int ttc_timer_mark(int* mark) {
    TTC_REQUIRE_INIT();
    if (!mark) return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: timer_mark: mark is NULL");
    const unsigned i = g_next_mark++ % 4096u;
    if (!g_marks[i]) TTC_CUDA(cudaEventCreate(&g_marks[i]));
    TTC_CUDA(cudaEventRecord(g_marks[i], rt().stream));
    *mark = (int)i;
    return TTC_OK;
}

int ttc_timer_elapsed(int from, int to, float* ms) {
    TTC_REQUIRE_INIT();
    if (!ms || from < 0 || to < 0 || from >= 4096 || to >= 4096 || !g_marks[from] || !g_marks[to])
        return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: timer_elapsed: unknown mark");
    if (cudaEventQuery(g_marks[to]) != cudaSuccess) {
        if (int rc = sync_stream_bounded(rt().stream)) return rc;  // bounded when an all-reduce is queued
    }
    TTC_CUDA(cudaEventSynchronize(g_marks[to]));
    TTC_CUDA(cudaEventElapsedTime(ms, g_marks[from], g_marks[to]));
    return TTC_OK;
}

int ttc_capture_begin(void) {
    TTC_REQUIRE_INIT();
    TTC_CUDA(cudaStreamBeginCapture(rt().stream, cudaStreamCaptureModeThreadLocal));
    return TTC_OK;
}

int ttc_capture_end(void** graph_exec) {
    TTC_REQUIRE_INIT();
    if (!graph_exec) return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: capture_end: graph_exec is NULL");
    *graph_exec = nullptr;
    cudaGraph_t g = nullptr;
    TTC_CUDA(cudaStreamEndCapture(rt().stream, &g));
    cudaGraphExec_t exec = nullptr;
    const cudaError_t e = cudaGraphInstantiateWithFlags(&exec, g, cudaGraphInstantiateFlagAutoFreeOnLaunch);
    cudaGraphDestroy(g);
    TTC_CUDA(e);
    *graph_exec = (void*)exec;
    return TTC_OK;
}

int ttc_graph_launch(void* graph_exec) {
    TTC_REQUIRE_INIT();
    if (!graph_exec) return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: graph_launch: NULL graph");
    TTC_CUDA(cudaGraphLaunch((cudaGraphExec_t)graph_exec, rt().stream));
    return TTC_OK;
}

int ttc_graph_destroy(void* graph_exec) {
    if (graph_exec) cudaGraphExecDestroy((cudaGraphExec_t)graph_exec);
    return TTC_OK;
}

int ttc_memcpy_d2h(void* dst, const void* src, size_t bytes) {
    TTC_REQUIRE_INIT();
    if (bytes == 0) return TTC_OK;
    TTC_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, rt().stream));
    if (int rc = sync_stream_bounded(rt().stream)) return rc;
    return check_device_status();
}

int ttc_memcpy_d2d(void* dst, const void* src, size_t bytes) {
    TTC_REQUIRE_INIT();
    if (bytes == 0) return TTC_OK;
    TTC_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, rt().stream));
    return TTC_OK;
}

int ttc_memset_zero(void* dst, size_t bytes) {
    TTC_REQUIRE_INIT();
    if (bytes == 0) return TTC_OK;
    TTC_CUDA(cudaMemsetAsync(dst, 0, bytes, rt().stream));
    return TTC_OK;
}

int ttc_host_alloc(size_t bytes, void** hptr) {
    TTC_REQUIRE_INIT();
    if (!hptr) return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: hptr is NULL");
    TTC_CUDA(cudaHostAlloc(hptr, bytes, cudaHostAllocDefault));
    return TTC_OK;
}

int ttc_host_free(void* hptr) {
    TTC_REQUIRE_INIT();
    if (hptr) TTC_CUDA(cudaFreeHost(hptr));
    return TTC_OK;
}

int ttc_get_memory_stats(ttc_memory_stats* out) {
    if (!out) return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: out is NULL");
    Runtime& r = rt();
    out->bytes_in_use = r.bytes_in_use;
    out->peak_bytes = r.peak_bytes;
    out->workspace_bytes = r.workspace_bytes;
    out->kernels_launched = r.kernels;
    return TTC_OK;
}

}  // extern "C"
