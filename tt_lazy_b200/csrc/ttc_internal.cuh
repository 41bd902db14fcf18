// ttc_internal.cuh -- shared internals of tt_cuda_lib: error plumbing, the
// runtime state, and the element-wise program interpreter that the chain
// kernel and every GEMM epilogue run.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/tt_cuda.h"
#ifdef __CUDACC__
#include "expf_ref.cuh"
#endif

// ------------------------------------------------------------------ errors
namespace ttc {

int set_error(int code, const char* fmt, ...);
int check_cuda(cudaError_t e, const char* what);
void clear_error();

struct Runtime {
    bool initialized = false;
    int device = -1;
    int sm_count = 0;
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;
    void* workspace = nullptr;  // grow-only internal scratch (reduction partials)
    size_t workspace_bytes = 0;
    size_t bytes_in_use = 0, peak_bytes = 0;
    unsigned long long kernels = 0;
    cudaStream_t copy_stream = nullptr;  // host-to-device prefetch (ttc_h2d_prefetch)
    cudaEvent_t tickets[256] = {};       // completion events of prefetches, a ring
    unsigned next_ticket = 0;
};
Runtime& rt();
// Waits for the work queued on `st`; with an all-reduce outstanding, polls
// against its deadline instead of blocking (comm.cpp).
int sync_stream_bounded(cudaStream_t st);
// One-time per-device set-up (kernel attributes, occupancy, loaded modules)
// is cached in arrays indexed by the device ordinal: function attributes and
// modules belong to a device's context, so a ttc_shutdown / ttc_init on
// another device must not reuse the first device's.
constexpr int kMaxDevices = 64;
// Scratch of at least `bytes`, valid until the next call that asks for more.
int workspace(size_t bytes, void** out);
inline void count_launch(unsigned n = 1) { rt().kernels += n; }

}  // namespace ttc

#define TTC_REQUIRE_INIT()                                                                  \
    do {                                                                                    \
        if (!ttc::rt().initialized)                                                        \
            return ttc::set_error(TTC_ERR_NOT_INITIALIZED, "tt_cuda: ttc_init() not called"); \
    } while (0)

#define TTC_CUDA(call)                                                  \
    do {                                                                \
        cudaError_t _e = (call);                                        \
        if (_e != cudaSuccess) return ttc::check_cuda(_e, #call);        \
    } while (0)

// ------------------------------------------------ device program (decoded)
// The C-ABI program (ttc_instr: op, src, idx) is decoded on the host into a
// flat opcode per step so that each step is one warp-uniform switch case
// working on compile-time registers (no runtime-indexed register arrays,
// which would spill to local memory).
namespace ttc {

enum DOp : uint8_t {
    D_LOAD = 0,
    D_RELU,
    D_SIGMOID,
    D_ADD_ACC,
    D_ADD_IN,
    D_ADD_S0,
    D_ADD_S1,
    D_ADD_S2,
    D_ADD_S3,
    D_MUL_ACC,
    D_MUL_IN,
    D_MUL_S0,
    D_MUL_S1,
    D_MUL_S2,
    D_MUL_S3,
    D_SAVE0,
    D_SAVE1,
    D_SAVE2,
    D_SAVE3,
    D_STORE,
    D_LOAD_S0,
    D_LOAD_S1,
    D_LOAD_S2,
    D_LOAD_S3,
    D_NUM_OPS
};

struct DInView {
    const float* ptr;
    long long sr, sc, sseg;
};
struct DOutView {
    float* ptr;
    long long sr, sseg;
};

struct DProgram {
    int n_instr;
    int n_in, n_out;
    int has_sigmoid;  // kernels fill the exp table only when a step needs it
    int n_slots;      // 1 + highest save slot the program uses (0 if none)
    uint8_t op[TTC_CHAIN_MAX_INSTR];
    uint8_t arg[TTC_CHAIN_MAX_INSTR];
    DInView in[TTC_CHAIN_MAX_INPUTS];
    DOutView out[TTC_CHAIN_MAX_OUTPUTS];
};

// Validates and decodes `d` (the shape part is checked by the caller).
// `acc_preloaded`: the GEMM epilogue case -- acc holds the product at entry.
int decode_program(const ttc_chain_desc& d, bool acc_preloaded, DProgram* out);

// 32-bit unsigned division by an invariant divisor (Granlund & Montgomery,
// "Division by invariant integers using multiplication", PLDI 1994, sec. 4):
// q = (umulhi(n, m) + n) >> s, exact for n < 2^31.
struct FastDiv {
    unsigned d, m, s;
};
FastDiv make_fastdiv(unsigned d);

#ifdef __CUDACC__
__device__ __forceinline__ unsigned fdiv(unsigned n, const FastDiv& f) {
    return (__umulhi(n, f.m) + n) >> f.s;
}

// --------------------------------------------------------------------------
// Interpreter. A thread evaluates G groups of W consecutive columns (W = 4:
// one 128-bit access per operand per group; W = 1: scalar path). Group g
// sits at (seg, row[g], col[g]); invalid groups skip every memory access.
// Every arithmetic step is a single IEEE op; the translation units that use
// this are compiled with -fmad=false so no multiply-add pair is contracted.
template <int W>
__device__ __forceinline__ void load_group(const DInView& v, long long seg, long long row, long long col,
                                           float (&dst)[W]) {
    const float* p = v.ptr + seg * v.sseg + row * v.sr;
    if constexpr (W == 4) {
        if (v.sc == 0) {
            const float s = __ldg(p);
            dst[0] = dst[1] = dst[2] = dst[3] = s;
        } else {
            const float4 q = __ldg(reinterpret_cast<const float4*>(p + col));
            dst[0] = q.x;
            dst[1] = q.y;
            dst[2] = q.z;
            dst[3] = q.w;
        }
    } else {
        dst[0] = __ldg(p + col * v.sc);
    }
}

template <int W>
__device__ __forceinline__ void store_group(const DOutView& v, long long seg, long long row, long long col,
                                            const float (&src)[W]) {
    float* p = v.ptr + seg * v.sseg + row * v.sr + col;
    if constexpr (W == 4) {
        *reinterpret_cast<float4*>(p) = make_float4(src[0], src[1], src[2], src[3]);
    } else {
        p[0] = src[0];
    }
}

__device__ __forceinline__ float op_relu(float x) { return (0.0f < x) ? x : 0.0f; }

// sigmoid = 1 / (1 + e^-x) with the exp of expf_ref.cuh; its 32-entry table
// lives in shared memory (exp2_table_init_block fills it at kernel start,
// before a __syncthreads).
static __shared__ ExpTable s_exp_tab;

__device__ __forceinline__ void exp2_table_init_block() { exp_table_init(s_exp_tab); }

// Applies f(g, w) to every element. Arithmetic runs on all groups (invalid
// groups compute on zeros and are never stored or summed).
template <int G, int W, class F>
__device__ __forceinline__ void each(F&& f) {
#pragma unroll
    for (int g = 0; g < G; ++g)
#pragma unroll
        for (int w = 0; w < W; ++w) f(g, w);
}

// Memory policy of the interpreter: operands come straight from global
// memory through the program's views. Other kernels supply their own policy
// (the staged chain kernel reads full operands from shared memory).
template <int G, int W>
struct GlobalIO {
    const DProgram& P;
    long long seg;
    const long long (&row)[G];
    const long long (&col)[G];
    const bool (&valid)[G];
    __device__ __forceinline__ bool ok(int g) const { return valid[g]; }
    __device__ __forceinline__ void load(int k, int g, float (&dst)[W]) const {
        load_group<W>(P.in[k], seg, row[g], col[g], dst);
    }
    __device__ __forceinline__ void store(int j, int g, const float (&src)[W]) const {
        store_group<W>(P.out[j], seg, row[g], col[g], src);
    }
};

// Runs the program on acc. NS = save slots the caller's programs may use
// (slots >= NS never occur: the host picks the instantiation from the
// decoded program), so unused slots cost no registers.
template <int G, int W, int NS, class IO>
__device__ __forceinline__ void run_program_io(const DProgram& P, float (&acc)[G][W], const IO& io) {
    float s[NS][G][W];
#pragma unroll
    for (int k = 0; k < NS; ++k) each<G, W>([&](int g, int w) { s[k][g][w] = 0.0f; });

    for (int pc = 0; pc < P.n_instr; ++pc) {
        const int a = P.arg[pc];
        switch (P.op[pc]) {
            case D_LOAD:
#pragma unroll
                for (int g = 0; g < G; ++g)
                    if (io.ok(g)) io.load(a, g, acc[g]);
                break;
            case D_RELU: each<G, W>([&](int g, int w) { acc[g][w] = op_relu(acc[g][w]); }); break;
            case D_SIGMOID:
#pragma unroll
                for (int g = 0; g < G; ++g) sigmoid_ref_n<W>(acc[g], s_exp_tab);
                break;
            case D_ADD_ACC: each<G, W>([&](int g, int w) { acc[g][w] = acc[g][w] + acc[g][w]; }); break;
            case D_MUL_ACC: each<G, W>([&](int g, int w) { acc[g][w] = acc[g][w] * acc[g][w]; }); break;
            case D_ADD_IN:
            case D_MUL_IN: {
                float t[G][W];
                each<G, W>([&](int g, int w) { t[g][w] = 0.0f; });
#pragma unroll
                for (int g = 0; g < G; ++g)
                    if (io.ok(g)) io.load(a, g, t[g]);
                if (P.op[pc] == D_ADD_IN)
                    each<G, W>([&](int g, int w) { acc[g][w] = acc[g][w] + t[g][w]; });
                else
                    each<G, W>([&](int g, int w) { acc[g][w] = acc[g][w] * t[g][w]; });
                break;
            }
#define TTC_SLOT_CASES(K)                                                                                 \
    case D_ADD_S0 + K:                                                                                    \
        if constexpr (NS > K) each<G, W>([&](int g, int w) { acc[g][w] = acc[g][w] + s[K % NS][g][w]; }); \
        break;                                                                                            \
    case D_MUL_S0 + K:                                                                                    \
        if constexpr (NS > K) each<G, W>([&](int g, int w) { acc[g][w] = acc[g][w] * s[K % NS][g][w]; }); \
        break;                                                                                            \
    case D_SAVE0 + K:                                                                                     \
        if constexpr (NS > K) each<G, W>([&](int g, int w) { s[K % NS][g][w] = acc[g][w]; });             \
        break;                                                                                            \
    case D_LOAD_S0 + K:                                                                                   \
        if constexpr (NS > K) each<G, W>([&](int g, int w) { acc[g][w] = s[K % NS][g][w]; });             \
        break;
                TTC_SLOT_CASES(0)
                TTC_SLOT_CASES(1)
                TTC_SLOT_CASES(2)
                TTC_SLOT_CASES(3)
#undef TTC_SLOT_CASES
            case D_STORE:
#pragma unroll
                for (int g = 0; g < G; ++g)
                    if (io.ok(g)) io.store(a, g, acc[g]);
                break;
            default:
                break;
        }
    }
}

template <int G, int W, int NS = 4>
__device__ __forceinline__ void run_program(const DProgram& P, float (&acc)[G][W], long long seg,
                                            const long long (&row)[G], const long long (&col)[G],
                                            const bool (&valid)[G]) {
    const GlobalIO<G, W> io{P, seg, row, col, valid};
    run_program_io<G, W, NS>(P, acc, io);
}

// Warp / block sums used by the reductions (fixed shuffle order: the result
// does not depend on scheduling, so reductions are run-to-run deterministic).
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
#endif  // __CUDACC__

}  // namespace ttc
