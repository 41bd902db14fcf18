/*
 * tt_cuda.h -- C-ABI of tt_cuda_lib, the B200 (sm_100a) execution backend
 * for tt_lazy.
 *
 * It replaces the reference's CPU backend `namespace math`
 * (src/backend/cpu/math_operations.hpp:6-31, library tt_math_lib linked
 * PRIVATE into tt_lazy_tape at CMakeLists.txt:264-270). The reference seam is
 * C++ (`Tensor math::relu(const Tensor&)`, errors thrown as
 * std::runtime_error); this seam is plain C: device pointers, sizes and
 * strides in, an int status out, no C++ exception ever crosses it. The C++
 * operation handlers (tt_lazy_b200/host/Executor.cpp) turn a non-zero
 * status back into std::runtime_error(ttc_last_error()), which keeps the
 * reference's error behaviour for tt_lazy users.
 *
 * Data: fp32 only, row-major, rank <= 4 -- the reference's only dtype and
 * rank limit (src/core/Tensor.hpp:111-114).
 *
 * Threading: one process drives one GPU; calls come from one host thread
 * (the reference's Context/EvaluationManager are unsynchronised singletons,
 * src/core/Context.hpp:91-94). Kernels run in order on the library stream
 * (ttc_get_stream / ttc_set_stream).
 */
#ifndef TT_CUDA_H
#define TT_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status */
typedef enum {
    TTC_OK = 0,
    TTC_ERR_INVALID_ARGUMENT = 1, /* shape / pointer / descriptor error      */
    TTC_ERR_CUDA = 2,             /* a CUDA runtime or driver call failed     */
    TTC_ERR_OUT_OF_MEMORY = 3,
    TTC_ERR_UNSUPPORTED = 4,      /* valid request this build does not run   */
    TTC_ERR_NOT_INITIALIZED = 5,
    TTC_ERR_NCCL = 6,
    TTC_ERR_TIMEOUT = 7           /* a bounded wait (device or host) expired */
} ttc_status;

/* Text of the last error on this thread ("" when none). Mirrors the
 * std::runtime_error messages of the reference where one exists. */
const char* ttc_last_error(void);

/* ----------------------------------------------------------------- runtime */
/* Select `device`, create the library stream and the device arena. Must be
 * called once per process before any other call (except ttc_last_error,
 * ttc_device_count and ttc_version). Idempotent for the same device. */
int ttc_init(int device);
int ttc_shutdown(void);
int ttc_device_count(int* count);
int ttc_version(void); /* (major << 16) | minor */

/* The library stream (a cudaStream_t). ttc_set_stream(NULL) restores the
 * library's own stream. All launches and async copies go to this stream. */
void* ttc_get_stream(void);
int ttc_set_stream(void* cuda_stream);
int ttc_synchronize(void);

/* ----------------------------------------------------------- device memory
 * Replaces the host pool of src/core/MemoryManager.{hpp,cpp} (MemoryPool,
 * first-fit malloc pool, MemoryManager.cpp:46-61) with stream-ordered device
 * HBM. The host front end carves per-tape arenas out of these allocations. */
int ttc_malloc(size_t bytes, void** dptr);
int ttc_free(void* dptr);
/* host -> device, async on the library stream (src may be pageable or pinned) */
int ttc_memcpy_h2d(void* dst, const void* src, size_t bytes);
/* device -> host, synchronous: the single materialisation copy that stands in
 * for the memcpy of Tensor::eval_impl (src/core/Tensor.cpp:572). */
int ttc_memcpy_d2h(void* dst, const void* src, size_t bytes);
/* Host -> device prefetch on the library's copy stream (no reference
 * counterpart: it lets the upload of one batch chunk overlap the kernels of
 * the previous one). The copy starts after all work already enqueued on the
 * library stream; *ticket names it for ttc_wait_ticket, which makes later
 * work on the library stream wait for the copy. src should be pinned
 * (ttc_host_alloc) for the copy to run asynchronously. Up to 256 prefetches
 * may be outstanding. */
int ttc_h2d_prefetch(void* dst, const void* src, size_t bytes, int* ticket);
int ttc_wait_ticket(int ticket);
/* CUDA-graph capture of the library stream (no reference counterpart: a
 * compiled tape replayed with one launch instead of one per kernel). Between
 * ttc_capture_begin and ttc_capture_end the library's calls are recorded,
 * not run; they must not synchronise with the host (no ttc_memcpy_d2h, no
 * all-reduce). ttc_capture_end instantiates the recording into an opaque
 * executable graph, ttc_graph_launch replays it on the library stream. */
int ttc_capture_begin(void);
int ttc_capture_end(void** graph_exec);
int ttc_graph_launch(void* graph_exec);
int ttc_graph_destroy(void* graph_exec);
/* Tracing (no reference counterpart; the reference only logs): NVTX ranges
 * around tape operations for an attached profiler, and CUDA-event marks on
 * the library stream. ttc_timer_elapsed waits for mark `to` and returns the
 * device time between the two marks. Marks come from a ring of 4096. */
int ttc_range_push(const char* name);
int ttc_range_pop(void);
int ttc_timer_mark(int* mark);
int ttc_timer_elapsed(int from, int to, float* ms);
int ttc_memcpy_d2d(void* dst, const void* src, size_t bytes);
int ttc_memset_zero(void* dst, size_t bytes);
/* Pinned host memory for staging (cudaHostAlloc). */
int ttc_host_alloc(size_t bytes, void** hptr);
int ttc_host_free(void* hptr);

typedef struct {
    size_t bytes_in_use;      /* live ttc_malloc bytes                     */
    size_t peak_bytes;        /* high-water mark of bytes_in_use           */
    size_t workspace_bytes;   /* internal scratch (reduction partials)     */
    uint64_t kernels_launched; /* kernels this library launched so far      */
} ttc_memory_stats;
int ttc_get_memory_stats(ttc_memory_stats* out);

/* ------------------------------------------------------ element-wise chain
 * One kernel evaluates a whole element-wise chain over a 2-D iteration space
 * [rows, cols] (repeated over `nseg` segments), optionally followed by a
 * reduction of the chain's final value. It replaces a run of
 * math::relu / math::add / math::multiply (src/backend/cpu/eltwise.cpp:8-111)
 * and the README's sigmoid (README.md:332), each of which the reference runs
 * as a separate pass with a freshly allocated Tensor, plus math::reduce_sum
 * (src/backend/cpu/reduce_sum.cpp:9-62) when a reduction ends the chain.
 *
 * The program is an accumulator machine: `acc` holds the current value,
 * four save slots hold intermediates.
 *   LOAD  k      acc = input[k]       (src = SLOT: acc = slot[k])
 *   RELU         acc = (0.0f < acc) ? acc : 0.0f         (std::max(0.0f, x))
 *   SIGMOID      acc = 1.0f / (1.0f + expf(-acc))
 *   ADD  src     acc = acc + src     src = ACC | INPUT k | SLOT s
 *   MUL  src     acc = acc * src
 *   SAVE s       slot[s] = acc
 *   STORE k      output[k] = acc
 * Every step is one IEEE single operation (no FMA contraction), so results
 * are bit-identical to the reference's separate passes; SIGMOID rounds a
 * table-driven e^-x (relative error below 2^-44) once, then adds and takes
 * the IEEE reciprocal, so it equals the CPU's 1/(1+expf(-x)) on nearly every
 * input and stays within 2 ulp of it everywhere.
 *
 * Views: element (r, c) of segment g of input k is
 *   ptr[g*seg_stride + r*row_stride + c*col_stride]
 * with col_stride 1 (contiguous) or 0 (column-broadcast [R,1]) and
 * row_stride >= 0 (0 = row-broadcast [1,C], the bias case of
 * eltwise.cpp:62-76). Outputs use col_stride 1.
 * Transposed and split operands are views too (transpose.cpp:14-30 and
 * split.cpp:17-37 become stride/offset arithmetic; nothing is copied).
 */
#define TTC_CHAIN_MAX_INPUTS 6
#define TTC_CHAIN_MAX_OUTPUTS 4
#define TTC_CHAIN_MAX_INSTR 32
#define TTC_CHAIN_SLOTS 4

typedef enum {
    TTC_OP_LOAD = 1,
    TTC_OP_RELU = 2,
    TTC_OP_SIGMOID = 3,
    TTC_OP_ADD = 4,
    TTC_OP_MUL = 5,
    TTC_OP_SAVE = 6,
    TTC_OP_STORE = 7
} ttc_opcode;

typedef enum { TTC_SRC_ACC = 0, TTC_SRC_INPUT = 1, TTC_SRC_SLOT = 2 } ttc_src_kind;

typedef struct {
    uint8_t op;   /* ttc_opcode                                           */
    uint8_t src;  /* ttc_src_kind (ADD / MUL only)                        */
    uint8_t idx;  /* input / slot / output index                          */
    uint8_t pad;
} ttc_instr;

typedef struct {
    const float* ptr;
    int64_t row_stride;
    int64_t col_stride; /* 1 or 0 */
    int64_t seg_stride;
} ttc_in_view;

typedef struct {
    float* ptr;
    int64_t row_stride;
    int64_t seg_stride;
} ttc_out_view;

typedef enum {
    TTC_REDUCE_NONE = 0,
    TTC_REDUCE_ALL = 1,  /* every element of a segment -> reduce_out[g]        */
    TTC_REDUCE_ROWS = 2, /* over cols: reduce_out[g*seg + r]  (sum along dim 1) */
    TTC_REDUCE_COLS = 3  /* over rows: reduce_out[g*seg + c]  (sum along dim 0) */
} ttc_reduce_mode;

typedef struct {
    int32_t rows, cols, nseg;
    int32_t n_inputs, n_outputs, n_instr;
    ttc_in_view inputs[TTC_CHAIN_MAX_INPUTS];
    ttc_out_view outputs[TTC_CHAIN_MAX_OUTPUTS];
    ttc_instr program[TTC_CHAIN_MAX_INSTR];
    int32_t reduce;        /* ttc_reduce_mode                                  */
    int32_t reduce_mean;   /* divide each sum by its term count                */
    float* reduce_out;
    int64_t reduce_seg_stride;
} ttc_chain_desc;

int ttc_eltwise_chain(const ttc_chain_desc* desc);

/* Same computation as ttc_eltwise_chain, for callers that must not allocate
 * device memory while they run: a serving or real-time loop that reserves
 * all its memory at start-up (a cudaMalloc mid-request can stall on a device
 * synchronisation or fail under memory pressure), or a host framework that
 * owns every device allocation through its own pool, where a library
 * allocating behind its back breaks the pool's accounting and limits. No
 * counterpart in the reference (its backend runs on the CPU and allocates a
 * Tensor per op).
 *
 * It calls no cudaMalloc, cudaFree or allocating library routine: the
 * per-block partial sums of a reduction go to a fixed 1 MiB device array
 * compiled into the library (every GPU that loads the library holds it until
 * the process exits). The launch sizes its grid so the partials fit: a full
 * sum uses at most 262144 / nseg blocks per segment, a column sum at most
 * 262144 / (nseg x cols) row bands (one band needs no partials), so every
 * descriptor ttc_eltwise_chain accepts runs here too, with fewer blocks when
 * the array is the limit. A launch whose partials would still not fit
 * returns TTC_ERR_INVALID_ARGUMENT with both sizes in ttc_last_error(). The
 * first call on a device looks up that array's device address (with the
 * library's device current; first calls from several threads wait for one
 * lookup); make that first call before any stream capture.
 * All calls share the one array and it keeps the last call's contents (the
 * kernels overwrite every partial they read, nothing needs clearing), so
 * calls that overlap on the GPU -- on different streams, or from different
 * threads -- race: serialise them. It always uses the register-path kernels
 * (the TMA-staged path is not taken), so results agree with
 * ttc_eltwise_chain to rounding, not bit for bit, when a reduction is fused. */
int ttc_eltwise_chain_noalloc(const ttc_chain_desc* desc);

/* Diagnostics (no reference counterpart): the CUDA source text that the
 * program-specialised chain kernel for `desc` is compiled from (NVRTC, at
 * first use). Writes at most cap - 1 characters and a terminating NUL to
 * `out` (may be NULL to query the length) and the full length to *len.
 * Needs no device and no ttc_init. */
int ttc_chain_jit_source(const ttc_chain_desc* desc, char* out, size_t cap, size_t* len);

/* ------------------------------------------------------------ reductions
 * math::reduce_sum (src/backend/cpu/reduce_sum.cpp:9-62) and the MEAN type
 * of ReduceArgs (src/frontend/operations.hpp:13-14) over any set of dims of a
 * contiguous rank<=4 tensor (ndims == 0: all dims). `out` holds the reduced
 * elements in row-major order (keepdim only changes the shape). Sums are
 * deterministic tree reductions (fp32 partials, fp64 final combine). */
int ttc_reduce(const float* in, const uint32_t* shape, int rank, const int32_t* dims, int ndims, int mean,
               float* out);

/* --------------------------------------------------------------- transpose
 * math::transpose (src/backend/cpu/transpose.cpp:7-36): swaps the last two
 * dims of a contiguous [batch, rows, cols] tensor into [batch, cols, rows].
 * Shared-memory tiled, bank-conflict-free, both sides coalesced. */
int ttc_transpose(const float* in, float* out, int64_t batch, int64_t rows, int64_t cols);

/* ---------------------------------------------------------- strided copy
 * Materialises a view (a split chunk, split.cpp:17-37, or any 2-D strided
 * window) into a dense buffer: out[r*out_ld + c] = in[r*in_ld + c]. */
int ttc_copy2d(const float* in, int64_t in_ld, float* out, int64_t out_ld, int64_t rows, int64_t cols);

/* -------------------------------------------------------------------- GEMM
 * math::matmul (src/backend/cpu/matmul.cpp:36-85) and math::fused_mlp
 * (src/backend/cpu/fused_ops.cpp:8-64): C[M,N] = op(A)[M,K] . op(B)[K,N],
 * op = transpose when trans_a / trans_b (matmul.cpp:47-48), with the
 * epilogue program run on the accumulator before anything is written.
 *
 * The epilogue is a ttc_chain_desc over the [M, N] output space whose `acc`
 * starts as the product (no LOAD needed): e.g. ADD INPUT 0 (bias view with
 * row_stride 0), RELU, STORE 0 is the fused MLP layer. rows/cols/nseg of the
 * epilogue are ignored (M, N, 1 are used). An epilogue with n_instr == 0
 * means STORE to `c` (or nothing when `c` is NULL and a reduction is set).
 * The epilogue's `reduce` may be TTC_REDUCE_COLS: reduce_out[n] = the sum
 * (mean with reduce_mean) over the M rows of the epilogue's final value, the
 * batch-dim reduce_sum of the reference's handle_reduce on the GEMM result
 * (reduce_sum.cpp:9-62) without writing that [M, N] value anywhere. The TF32
 * kernels sum each 32-row group in the epilogue (deterministic, no atomics)
 * and combine the groups in fp64; the FFMA path reduces a scratch copy.
 *
 * path: TTC_GEMM_FFMA -- fp32 CUDA-core FMA (norm-wise rel. error ~1e-6,
 *                         the 1e-5 bound);
 *       TTC_GEMM_TF32 -- tcgen05.mma kind::tf32, TMEM accumulators, TMA
 *                         operand loads (the 2e-3 bound); a CTA pair
 *                         (cta_group::2, 256x256 tiles) when those tiles
 *                         number at least half the SMs, else one CTA per
 *                         128x256 tile (split along K when tiles are few);
 *       TTC_GEMM_AUTO -- TF32 when the shape suits the tensor-core kernel,
 *                         else FFMA;
 *       TTC_GEMM_TF32X3 -- fp32-accurate products on the tensor cores: each
 *                         operand split into a TF32 part and a TF32 remainder
 *                         (x = big + small), three kind::tf32 MMAs per step
 *                         (big*big + big*small + small*big) into fp32 TMEM
 *                         accumulators (the 1e-5 bound, ~1e-6 measured);
 *                         shapes the tensor-core kernel does not take run on
 *                         the FFMA path. An output tile whose rows of A or
 *                         columns of B hold an infinity or NaN takes the
 *                         big*big product alone (an infinity times a zero
 *                         remainder would make NaN where fp32 gives +-inf):
 *                         infinities and NaN come out where fp32 gives them,
 *                         and that tile's finite values have TF32 accuracy.
 */
typedef enum { TTC_GEMM_AUTO = 0, TTC_GEMM_FFMA = 1, TTC_GEMM_TF32 = 2, TTC_GEMM_TF32X3 = 3 } ttc_gemm_path;

typedef struct {
    int32_t M, N, K;
    const float* a; int64_t lda; int32_t trans_a; /* stored [M,K] or [K,M] when trans_a */
    const float* b; int64_t ldb; int32_t trans_b; /* stored [K,N] or [N,K] when trans_b */
    float* c; int64_t ldc;                        /* default output (epilogue n_instr == 0) */
    int32_t path;                                 /* ttc_gemm_path */
    ttc_chain_desc epilogue;
} ttc_gemm_desc;

int ttc_gemm(const ttc_gemm_desc* desc);
/* Which path ttc_gemm would take for this descriptor (TTC_GEMM_FFMA/TF32/TF32X3). */
int ttc_gemm_select_path(const ttc_gemm_desc* desc);

/* ------------------------------------------------ collective (multi-GPU)
 * Row-sharded data parallelism: every rank holds the same weights and a
 * slice of the batch; the only exchange is the sum of per-shard partial
 * reductions. NCCL communicator, created non-blocking; every wait is bounded
 * by timeout_ms and an expired wait aborts the communicator and returns
 * TTC_ERR_TIMEOUT instead of hanging. ttc_allreduce_sum enqueues the
 * collective on the library stream and returns without waiting for it; the
 * next synchronisation (ttc_synchronize, a ttc_memcpy_d2h, the next
 * ttc_allreduce_sum, ttc_comm_destroy) polls for its completion against the
 * deadline and the communicator's asynchronous error, and reports a failure
 * there. No reference counterpart (the reference is single-process). */
#define TTC_UNIQUE_ID_BYTES 128
int ttc_comm_unique_id(uint8_t out[TTC_UNIQUE_ID_BYTES]);
int ttc_comm_init(int nranks, int rank, const uint8_t id[TTC_UNIQUE_ID_BYTES], int timeout_ms);
int ttc_allreduce_sum(float* buf, size_t count, int timeout_ms);
int ttc_comm_destroy(void);

#ifdef __cplusplus
}
#endif
#endif /* TT_CUDA_H */
