// chain.cu -- the fused element-wise chain kernel (+ optional tail
// reduction), and the reductions / strided copies built on it.
//
// Replaces src/backend/cpu/eltwise.cpp:8-111 (relu, add, multiply, each a
// separate single-threaded pass with a fresh Tensor), the README's sigmoid
// (README.md:332) and src/backend/cpu/reduce_sum.cpp:9-62.
//
// HBM-bound: every input element is read once with a 128-bit load, every
// stored element written once with a 128-bit store; intermediates live in
// registers. Grids are sized to the resident capacity of the 148 SMs and
// iterate grid-stride. Compiled with -fmad=false: each step is a single IEEE
// op, as in the reference's separate passes.
#include <algorithm>
#include <cstdlib>
#include <atomic>
#include <cstring>
#include <mutex>

#include "tma_util.cuh"

namespace ttc {

// Staged (TMA-fed) variant, chain_tma.cu: launches when the layout allows it.
int launch_chain_tma(const ttc_chain_desc& d, const DProgram& prog, bool* launched);
// Program-specialised variant, chain_jit.cu: launches when compiled.
int launch_chain_jit(const ttc_chain_desc& d, const DProgram& prog, bool* launched);

namespace {

constexpr int kThreads = 256;
constexpr int kGroups = 2;  // 128-bit groups per thread per program pass

struct ChainParams {
    DProgram prog;
    int rows, cols, nseg;
    unsigned cpr;  // column chunks (of W) per row
    FastDiv cpr_div;
    unsigned total;  // rows * cpr  (< 2^31)
    float* red_out;
    long long red_sseg;
    float* partials;
    int nsplit, rows_per_split;
    int mean;
    double count;
};

template <int W, bool REDUCE_ALL>
__global__ void __launch_bounds__(kThreads) chain_flat_kernel(const __grid_constant__ ChainParams p) {
    constexpr int G = kGroups;
    if (p.prog.has_sigmoid) {
        exp2_table_init_block();
        __syncthreads();
    }
    const long long seg = blockIdx.y;
    float sum = 0.0f;
    for (unsigned blk = blockIdx.x; (unsigned long long)blk * (kThreads * G) < p.total; blk += gridDim.x) {
        const unsigned q0 = blk * (kThreads * G) + threadIdx.x;
        long long row[G], col[G];
        bool valid[G];
#pragma unroll
        for (int g = 0; g < G; ++g) {
            const unsigned q = q0 + g * kThreads;
            valid[g] = q < p.total;
            const unsigned r = fdiv(q, p.cpr_div);
            row[g] = r;
            col[g] = (long long)(q - r * p.cpr) * W;
        }
        float acc[G][W];
        each<G, W>([&](int g, int w) { acc[g][w] = 0.0f; });
        run_program<G, W>(p.prog, acc, seg, row, col, valid);
        if (REDUCE_ALL) {
#pragma unroll
            for (int g = 0; g < G; ++g)
                if (valid[g])
#pragma unroll
                    for (int w = 0; w < W; ++w) sum += acc[g][w];
        }
    }
    if (REDUCE_ALL) {
        __shared__ float red[kThreads / 32];
        sum = warp_sum(sum);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sum;
        __syncthreads();
        if (threadIdx.x < 32) {
            float v = threadIdx.x < kThreads / 32 ? red[threadIdx.x] : 0.0f;
            v = warp_sum(v);
            if (threadIdx.x == 0) p.partials[seg * gridDim.x + blockIdx.x] = v;
        }
    }
}

// Reduction over cols (dim 1): one warp per row.
template <int W>
__global__ void __launch_bounds__(kThreads) chain_rows_kernel(const __grid_constant__ ChainParams p) {
    constexpr int G = kGroups;
    if (p.prog.has_sigmoid) {
        exp2_table_init_block();
        __syncthreads();
    }
    const long long seg = blockIdx.y;
    const int lane = threadIdx.x & 31;
    const unsigned warp = (blockIdx.x * kThreads + threadIdx.x) >> 5;
    const unsigned nwarps = (gridDim.x * kThreads) >> 5;
    for (unsigned r = warp; r < (unsigned)p.rows; r += nwarps) {
        float sum = 0.0f;
        for (unsigned c0 = lane; c0 < p.cpr; c0 += 32 * G) {
            long long row[G], col[G];
            bool valid[G];
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const unsigned ch = c0 + g * 32;
                valid[g] = ch < p.cpr;
                row[g] = r;
                col[g] = (long long)ch * W;
            }
            float acc[G][W];
            each<G, W>([&](int g, int w) { acc[g][w] = 0.0f; });
            run_program<G, W>(p.prog, acc, seg, row, col, valid);
#pragma unroll
            for (int g = 0; g < G; ++g)
                if (valid[g])
#pragma unroll
                    for (int w = 0; w < W; ++w) sum += acc[g][w];
        }
        sum = warp_sum(sum);
        if (lane == 0) {
            const float v = p.mean ? (float)((double)sum / p.count) : sum;
            p.red_out[seg * p.red_sseg + r] = v;
        }
    }
}

// Reduction over rows (dim 0): a block owns 32*W columns and one split of
// the rows; its 8 warps interleave rows, then combine through shared memory.
template <int W>
__global__ void __launch_bounds__(kThreads) chain_cols_kernel(const __grid_constant__ ChainParams p) {
    constexpr int G = kGroups;
    constexpr int NW = kThreads / 32;
    if (p.prog.has_sigmoid) {
        exp2_table_init_block();
        __syncthreads();
    }
    const long long seg = blockIdx.z;
    const int split = blockIdx.y;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const unsigned ch = blockIdx.x * 32 + lane;
    const bool col_ok = ch < p.cpr;
    const int r0 = split * p.rows_per_split;
    const int r1 = min(p.rows, r0 + p.rows_per_split);
    float s[W];
#pragma unroll
    for (int w = 0; w < W; ++w) s[w] = 0.0f;
    for (int r = r0 + warp; r < r1; r += NW * G) {
        long long row[G], col[G];
        bool valid[G];
#pragma unroll
        for (int g = 0; g < G; ++g) {
            row[g] = r + g * NW;
            col[g] = (long long)ch * W;
            valid[g] = col_ok && row[g] < r1;
        }
        float acc[G][W];
        each<G, W>([&](int g, int w) { acc[g][w] = 0.0f; });
        run_program<G, W>(p.prog, acc, seg, row, col, valid);
#pragma unroll
        for (int g = 0; g < G; ++g)
            if (valid[g])
#pragma unroll
                for (int w = 0; w < W; ++w) s[w] += acc[g][w];
    }
    __shared__ float sm[NW][32 * W + 1];
#pragma unroll
    for (int w = 0; w < W; ++w) sm[warp][lane * W + w] = s[w];
    __syncthreads();
    for (int i = threadIdx.x; i < 32 * W; i += kThreads) {
        float t = 0.0f;
#pragma unroll
        for (int k = 0; k < NW; ++k) t += sm[k][i];
        const long long c = (long long)blockIdx.x * 32 * W + i;
        if (c < p.cols) {
            if (p.nsplit == 1) {
                p.red_out[seg * p.red_sseg + c] = p.mean ? (float)((double)t / p.count) : t;
            } else {
                p.partials[((long long)seg * p.nsplit + split) * p.cols + c] = t;
            }
        }
    }
}

__global__ void finalize_cols_kernel(const float* __restrict__ partials, int nsplit, int cols, float* out,
                                     long long sseg, int mean, double count) {
    const long long seg = blockIdx.y;
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= cols) return;
    double t = 0.0;
    for (int s = 0; s < nsplit; ++s) t += partials[(seg * nsplit + s) * cols + c];
    out[seg * sseg + c] = (float)(mean ? t / count : t);
}

__global__ void finalize_all_kernel(const float* __restrict__ partials, int nparts, float* out, long long sseg,
                                    int mean, double count) {
    const long long seg = blockIdx.x;
    double t = 0.0;
    for (int i = threadIdx.x; i < nparts; i += blockDim.x) t += partials[seg * nparts + i];
    __shared__ double red[32];
    t = warp_sum_d(t);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = t;
    __syncthreads();
    if (threadIdx.x < 32) {
        double v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0;
        v = warp_sum_d(v);
        if (threadIdx.x == 0) out[seg * sseg] = (float)(mean ? v / count : v);
    }
}

__global__ void fill_kernel(float* out, long long n, float v) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
        out[i] = v;
}

template <class K>
int occupancy_grid(K kernel) {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, 0) != cudaSuccess || per_sm < 1)
        per_sm = 1;
    return per_sm * rt().sm_count;
}

// occupancy_grid of `kernel`, queried once per device into the call site's
// own cache (kernels of one signature share a function-pointer type, so the
// cache cannot be keyed by type).
template <class K>
int occupancy_grid_cached(int (&cache)[kMaxDevices], K kernel) {
    const int dev = rt().device;
    if (dev < 0 || dev >= kMaxDevices) return occupancy_grid(kernel);
    if (cache[dev] < 1) cache[dev] = occupancy_grid(kernel);
    return cache[dev];
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

// 128-bit path precondition: every contiguous operand starts on 16 bytes and
// each row / segment offset is a multiple of 4 floats.
bool vector_ok(const ttc_chain_desc& d) {
    if (d.cols % 4 != 0) return false;
    for (int i = 0; i < d.n_inputs; ++i) {
        const ttc_in_view& v = d.inputs[i];
        if (v.col_stride == 0) continue;  // column broadcast: scalar load + splat
        if (!aligned16(v.ptr) || v.row_stride % 4 || v.seg_stride % 4) return false;
    }
    for (int i = 0; i < d.n_outputs; ++i) {
        const ttc_out_view& v = d.outputs[i];
        if (!aligned16(v.ptr) || v.row_stride % 4 || v.seg_stride % 4) return false;
    }
    return true;
}

// Caller-provided reduction scratch (the allocation-free entry point). When
// null, partials live in the library's grow-only workspace.
struct FixedScratch {
    float* ptr;
    size_t floats;
};

int scratch_for(size_t floats, const FixedScratch* fixed, void** out) {
    if (!fixed) return workspace(floats * sizeof(float), out);
    if (floats > fixed->floats)
        return set_error(TTC_ERR_INVALID_ARGUMENT,
                         "tt_cuda: ttc_eltwise_chain_noalloc: this reduction needs %zu bytes of scratch, the static "
                         "buffer holds %zu bytes; use ttc_eltwise_chain",
                         floats * sizeof(float), fixed->floats * sizeof(float));
    *out = fixed->ptr;
    return TTC_OK;
}

template <int W>
int launch_chain(const ttc_chain_desc& d, ChainParams& p, const FixedScratch* fixed) {
    cudaStream_t st = rt().stream;
    const int nseg = d.nseg;
    switch (d.reduce) {
        case TTC_REDUCE_NONE: {
            const long long need = ((long long)p.total + kThreads * kGroups - 1) / (kThreads * kGroups);
            static int cap_cache[kMaxDevices] = {};
            const int cap = occupancy_grid_cached(cap_cache, chain_flat_kernel<W, false>);
            const int gx = (int)std::max<long long>(1, std::min<long long>(need, std::max(1, cap / nseg)));
            chain_flat_kernel<W, false><<<dim3(gx, nseg), kThreads, 0, st>>>(p);
            count_launch();
            break;
        }
        case TTC_REDUCE_ALL: {
            const long long need = ((long long)p.total + kThreads * kGroups - 1) / (kThreads * kGroups);
            static int cap_cache[kMaxDevices] = {};
            const int cap = occupancy_grid_cached(cap_cache, chain_flat_kernel<W, true>);
            long long gx_max = std::max(1, cap / nseg);
            // a fixed scratch array bounds the partials: fewer blocks, each over more tiles
            if (fixed) gx_max = std::min<long long>(gx_max, std::max<long long>(1, (long long)fixed->floats / nseg));
            const int gx = (int)std::max<long long>(1, std::min<long long>(need, gx_max));
            void* ws = nullptr;
            if (int rc = scratch_for((size_t)gx * nseg, fixed, &ws)) return rc;
            p.partials = (float*)ws;
            chain_flat_kernel<W, true><<<dim3(gx, nseg), kThreads, 0, st>>>(p);
            finalize_all_kernel<<<nseg, 256, 0, st>>>(p.partials, gx, p.red_out, p.red_sseg, p.mean, p.count);
            count_launch(2);
            break;
        }
        case TTC_REDUCE_ROWS: {
            static int cap_cache[kMaxDevices] = {};
            const int cap = occupancy_grid_cached(cap_cache, chain_rows_kernel<W>);
            const long long need = ((long long)p.rows + (kThreads / 32) - 1) / (kThreads / 32);
            const int gx = (int)std::max<long long>(1, std::min<long long>(need, std::max(1, cap / nseg)));
            chain_rows_kernel<W><<<dim3(gx, nseg), kThreads, 0, st>>>(p);
            count_launch();
            break;
        }
        case TTC_REDUCE_COLS: {
            static int cap_cache[kMaxDevices] = {};
            const int cap = occupancy_grid_cached(cap_cache, chain_cols_kernel<W>);
            const int gx = (int)((p.cpr + 31) / 32);
            const long long base = (long long)gx * nseg;
            int nsplit = (int)std::min<long long>((cap + base - 1) / base, (p.rows + 63) / 64);
            // a fixed scratch array bounds the partials (nsplit x nseg x cols):
            // fewer, longer row bands; one band needs no partials at all
            if (fixed)
                nsplit = (int)std::min<long long>(nsplit, (long long)fixed->floats / ((long long)nseg * p.cols));
            nsplit = std::max(nsplit, 1);
            p.rows_per_split = (p.rows + nsplit - 1) / nsplit;
            nsplit = (p.rows + p.rows_per_split - 1) / p.rows_per_split;
            p.nsplit = nsplit;
            if (nsplit > 1) {
                void* ws = nullptr;
                if (int rc = scratch_for((size_t)nsplit * nseg * p.cols, fixed, &ws)) return rc;
                p.partials = (float*)ws;
            }
            if (gx > 65535 * 64 || nsplit > 65535 || nseg > 65535)
                return set_error(TTC_ERR_UNSUPPORTED, "tt_cuda: column reduction grid too large");
            chain_cols_kernel<W><<<dim3(gx, nsplit, nseg), kThreads, 0, st>>>(p);
            count_launch();
            if (nsplit > 1) {
                finalize_cols_kernel<<<dim3((p.cols + 255) / 256, nseg), 256, 0, st>>>(
                    p.partials, nsplit, p.cols, p.red_out, p.red_sseg, p.mean, p.count);
                count_launch();
            }
            break;
        }
        default:
            return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: unknown reduce mode %d", d.reduce);
    }
    return check_cuda(cudaGetLastError(), "chain kernel launch");
}

}  // namespace

void launch_finalize_all(const float* partials, int nparts, float* out, int mean, double count) {
    finalize_all_kernel<<<1, 256, 0, rt().stream>>>(partials, nparts, out, 0, mean, count);
    count_launch();
}

void launch_finalize_cols(const float* partials, int nsplit, int cols, int nseg, float* out, long long sseg, int mean,
                          double count) {
    finalize_cols_kernel<<<dim3((cols + 255) / 256, nseg), 256, 0, rt().stream>>>(partials, nsplit, cols, out, sseg,
                                                                                   mean, count);
    count_launch();
}

static int run_chain_impl(const ttc_chain_desc& d, const FixedScratch* fixed);

int run_chain(const ttc_chain_desc& d) { return run_chain_impl(d, nullptr); }

static int run_chain_impl(const ttc_chain_desc& d, const FixedScratch* fixed) {
    if (d.rows < 0 || d.cols < 0 || d.nseg < 1)
        return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: chain shape rows=%d cols=%d nseg=%d is invalid", d.rows,
                         d.cols, d.nseg);
    if (d.nseg > 65535) return set_error(TTC_ERR_UNSUPPORTED, "tt_cuda: more than 65535 segments");
    if (d.reduce != TTC_REDUCE_NONE && !d.reduce_out)
        return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: reduce_out is NULL");
    ChainParams p;
    std::memset(&p, 0, sizeof p);
    if (int rc = decode_program(d, false, &p.prog)) return rc;
    p.rows = d.rows;
    p.cols = d.cols;
    p.nseg = d.nseg;
    p.red_out = d.reduce_out;
    p.red_sseg = d.reduce_seg_stride;
    p.mean = d.reduce_mean;
    const long long nred = d.reduce == TTC_REDUCE_ROWS ? d.cols
                           : d.reduce == TTC_REDUCE_COLS ? d.rows
                                                          : (long long)d.rows * d.cols;
    p.count = (double)nred;
    if (d.rows == 0 || d.cols == 0) {
        // Nothing to evaluate; an empty sum is 0, an empty mean is NaN.
        long long n = d.reduce == TTC_REDUCE_ROWS ? d.rows : d.reduce == TTC_REDUCE_COLS ? d.cols : 1;
        if (d.reduce != TTC_REDUCE_NONE && n > 0) {
            const float v = d.reduce_mean ? __builtin_nanf("") : 0.0f;
            for (int g = 0; g < d.nseg; ++g) {
                fill_kernel<<<1, 256, 0, rt().stream>>>(d.reduce_out + g * d.reduce_seg_stride, n, v);
                count_launch();
            }
            return check_cuda(cudaGetLastError(), "fill kernel launch");
        }
        return TTC_OK;
    }
    static const bool tma_enabled = [] {
        const char* e = getenv("TTC_CHAIN_TMA");
        return !(e && e[0] == '0');
    }();
    static const bool jit_enabled = [] {
        const char* e = getenv("TTC_CHAIN_JIT");
        return !(e && e[0] == '0');
    }();
    if (jit_enabled && !fixed) {
        bool launched = false;
        if (int rc = launch_chain_jit(d, p.prog, &launched)) return rc;
        if (launched) return TTC_OK;
    }
    // The TMA-staged interpreter pays for its pipeline set-up only on large
    // problems (on 1000 x 1000 it replayed the README chain in 10.2 us, the
    // register interpreter in 8.2): it serves layouts the specialised kernel
    // declines, from 1 Mi elements.
    if (tma_enabled && !fixed && (long long)d.rows * d.cols * d.nseg >= (1LL << 20)) {
        bool launched = false;
        if (int rc = launch_chain_tma(d, p.prog, &launched)) return rc;
        if (launched) return TTC_OK;
    }
    const bool vec = vector_ok(d);
    const int W = vec ? 4 : 1;
    p.cpr = (unsigned)(d.cols / W);
    p.cpr_div = make_fastdiv(p.cpr);
    const unsigned long long total = (unsigned long long)d.rows * p.cpr;
    if (total >= (1ull << 31))
        return set_error(TTC_ERR_UNSUPPORTED, "tt_cuda: %llu vector chunks per segment exceed 2^31; split the tensor",
                         total);
    p.total = (unsigned)total;
    return vec ? launch_chain<4>(d, p, fixed) : launch_chain<1>(d, p, fixed);
}

}  // namespace ttc

using namespace ttc;

extern "C" {

int ttc_eltwise_chain(const ttc_chain_desc* desc) {
    TTC_REQUIRE_INIT();
    if (!desc) return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: desc is NULL");
    return run_chain(*desc);
}

int ttc_copy2d(const float* in, int64_t in_ld, float* out, int64_t out_ld, int64_t rows, int64_t cols) {
    TTC_REQUIRE_INIT();
    if (rows < 0 || cols < 0 || rows > INT32_MAX || cols > INT32_MAX)
        return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: copy2d shape %lld x %lld", (long long)rows,
                         (long long)cols);
    if (rows == 0 || cols == 0) return TTC_OK;
    ttc_chain_desc d;
    std::memset(&d, 0, sizeof d);
    d.rows = (int32_t)rows;
    d.cols = (int32_t)cols;
    d.nseg = 1;
    d.n_inputs = 1;
    d.n_outputs = 1;
    d.inputs[0] = ttc_in_view{in, in_ld, 1, 0};
    d.outputs[0] = ttc_out_view{out, out_ld, 0};
    d.n_instr = 2;
    d.program[0] = ttc_instr{TTC_OP_LOAD, 0, 0, 0};
    d.program[1] = ttc_instr{TTC_OP_STORE, 0, 0, 0};
    return run_chain(d);
}

// Reduction over one contiguous run of dims [d0, d1] of a contiguous tensor
// viewed as [outer, red, inner].
static int reduce_run(const float* in, long long outer, long long red, long long inner, int mean, float* out) {
    ttc_chain_desc d;
    std::memset(&d, 0, sizeof d);
    d.n_inputs = 1;
    d.n_instr = 1;
    d.program[0] = ttc_instr{TTC_OP_LOAD, 0, 0, 0};
    d.reduce_mean = mean;
    d.reduce_out = out;
    if (red > INT32_MAX || inner > INT32_MAX || outer > INT32_MAX)
        return set_error(TTC_ERR_UNSUPPORTED, "tt_cuda: reduction extent exceeds 2^31");
    if (inner == 1) {
        d.reduce = TTC_REDUCE_ROWS;
        d.rows = (int32_t)outer;
        d.cols = (int32_t)red;
        d.nseg = 1;
        d.inputs[0] = ttc_in_view{in, red, 1, 0};
    } else {
        d.reduce = TTC_REDUCE_COLS;
        d.rows = (int32_t)red;
        d.cols = (int32_t)inner;
        d.nseg = (int32_t)outer;
        d.inputs[0] = ttc_in_view{in, inner, 1, red * inner};
        d.reduce_seg_stride = inner;
    }
    return run_chain(d);
}

int ttc_reduce(const float* in, const uint32_t* shape, int rank, const int32_t* dims, int ndims, int mean,
               float* out) {
    TTC_REQUIRE_INIT();
    if (!in || !out || !shape || rank < 1 || rank > 4 || ndims < 0 || (ndims > 0 && !dims))
        return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: reduce arguments invalid (rank %d, ndims %d)", rank,
                         ndims);
    bool red[4] = {false, false, false, false};
    if (ndims == 0) {
        for (int i = 0; i < rank; ++i) red[i] = true;
    } else {
        for (int j = 0; j < ndims; ++j) {
            const int dd = dims[j] < 0 ? dims[j] + rank : dims[j];
            if (dd < 0 || dd >= rank)
                return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: reduce dim %d out of range for rank %d", dims[j],
                                 rank);
            red[dd] = true;
        }
    }
    long long ext[4];
    for (int i = 0; i < rank; ++i) ext[i] = shape[i];
    // Runs of reduced dims, last run first; each run is one chain launch.
    const float* cur = in;
    float* tmp[2] = {nullptr, nullptr};
    int ntmp = 0;
    int hi = rank - 1;
    int rc = TTC_OK;
    while (rc == TTC_OK) {
        while (hi >= 0 && !red[hi]) --hi;
        if (hi < 0) break;
        int lo = hi;
        while (lo - 1 >= 0 && red[lo - 1]) --lo;
        long long outer = 1, r = 1, inner = 1;
        for (int i = 0; i < lo; ++i) outer *= ext[i];
        for (int i = lo; i <= hi; ++i) r *= ext[i];
        for (int i = hi + 1; i < rank; ++i) inner *= ext[i];
        int lo2 = lo - 1;
        while (lo2 >= 0 && !red[lo2]) --lo2;
        const bool last = lo2 < 0;
        float* dst = out;
        if (!last) {
            const size_t bytes = (size_t)std::max<long long>(outer * inner, 1) * sizeof(float);
            if (cudaMallocAsync((void**)&tmp[ntmp], bytes, rt().stream) != cudaSuccess) {
                cudaGetLastError();
                rc = set_error(TTC_ERR_OUT_OF_MEMORY, "tt_cuda: reduce temporary of %zu bytes", bytes);
                break;
            }
            dst = tmp[ntmp++];
        }
        rc = reduce_run(cur, outer, r, inner, mean, dst);
        cur = dst;
        for (int i = lo; i <= hi; ++i) ext[i] = 1;
        hi = lo - 1;
        if (last) break;
    }
    for (int i = 0; i < ntmp; ++i) cudaFreeAsync(tmp[i], rt().stream);
    return rc;
}

}  // extern "C"

// ----------------------------------------------------------------------------
// Allocation-free variant of ttc_eltwise_chain, for callers that cannot
// allocate device memory while they run: a serving or real-time loop that
// reserves all its memory at start-up (an allocation mid-request can stall on
// a device synchronisation or fail under memory pressure), or a host
// framework whose own pool owns every device allocation. The only scratch the
// chain kernels need -- per-block partial sums of a reduction -- lives in a
// file-scope device array of fixed size instead of the library workspace.
namespace {
constexpr size_t kNoAllocScratchFloats = 262144;  // 1 MiB; every GPU that loads the library holds it
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];
std::mutex g_noalloc_mu;                                   // serialises the first-call address lookup
std::atomic<float*> g_noalloc_scratch_dev[kMaxDevices] = {};  // device address of the array, per device
}  // namespace

extern "C" int ttc_eltwise_chain_noalloc(const ttc_chain_desc* desc) {
    TTC_REQUIRE_INIT();
    if (!desc) return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: desc is NULL");
    const int dev = rt().device;
    if (dev < 0 || dev >= kMaxDevices) return set_error(TTC_ERR_UNSUPPORTED, "tt_cuda: device %d", dev);
    float* scratch = g_noalloc_scratch_dev[dev].load(std::memory_order_acquire);
    if (!scratch) {
        // First call on this device: the host-side name of the array is not a
        // device address, so look the address up once with the device
        // current. Threads making their first call at the same time wait for
        // one lookup.
        std::lock_guard<std::mutex> lk(g_noalloc_mu);
        scratch = g_noalloc_scratch_dev[dev].load(std::memory_order_relaxed);
        if (!scratch) {
            int cur = -1;
            TTC_CUDA(cudaGetDevice(&cur));
            if (cur != dev)
                return set_error(TTC_ERR_INVALID_ARGUMENT,
                                 "tt_cuda: current device %d is not the library's device %d", cur, dev);
            void* p = nullptr;
            TTC_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
            scratch = static_cast<float*>(p);
            g_noalloc_scratch_dev[dev].store(scratch, std::memory_order_release);
        }
    }
    const FixedScratch fixed{scratch, kNoAllocScratchFloats};
    return run_chain_impl(*desc, &fixed);
}
