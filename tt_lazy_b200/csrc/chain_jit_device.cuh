// chain_jit_device.cuh -- kernel templates of the specialised element-wise
// chain. At run time chain_jit.cu turns one fused program into a small Body
// struct of straight-line code (every operand index, input kind and program
// step fixed), appends it to this file's text and compiles the result once
// for sm_100a with NVRTC; the kernel is cached per distinct program. The
// structures (grid-stride over 128-bit column quads, warp per row for row
// sums, column blocks with row splits for column sums) are the same as the
// interpreted kernels of chain.cu, so results and partial-sum layouts match.
//
// The file is valid under nvcc (the host side uses the parameter struct) and
// under NVRTC (no standard headers). Everything runs with -fmad=false: each
// program step is one IEEE op.
#pragma once

#define TTJ_MAX_IN 6
#define TTJ_MAX_OUT 4

struct JInView {
    const float* ptr;
    long long sr, sc, sseg;
};
struct JOutView {
    float* ptr;
    long long sr, sseg;
};
struct JFastDiv {
    unsigned d, m, s;
};

struct JParams {
    JInView in[TTJ_MAX_IN];
    JOutView out[TTJ_MAX_OUT];
    int rows, cols, nseg;
    unsigned cpr;
    JFastDiv cpr_div;
    unsigned total;
    float* red_out;
    long long red_sseg;
    float* partials;
    int nsplit, rows_per_split;
    int mean;
    double count;
};

#if defined(__CUDACC_RTC__) || defined(__CUDA_ARCH__)

#ifndef __CUDACC_RTC__
#include "expf_ref.cuh"
#endif

#define TTJ_THREADS 256

__device__ __forceinline__ unsigned ttj_fdiv(unsigned n, const JFastDiv& f) { return (__umulhi(n, f.m) + n) >> f.s; }

__device__ __forceinline__ float ttj_relu(float x) { return (0.0f < x) ? x : 0.0f; }

// sigmoid with the exp of expf_ref.cuh (NVRTC receives that file's text ahead
// of this one): one range test for all G*W values of a thread.
__shared__ ExpTable ttj_exp_tab;

__device__ __forceinline__ void ttj_exp_table_init() { exp_table_init(ttj_exp_tab); }

template <int G, int W>
__device__ __forceinline__ void ttj_sigmoid_all(float (&acc)[G][W]) {
    sigmoid_ref_n<G * W>(&acc[0][0], ttj_exp_tab);
}

// Operand kinds: 0 full (contiguous columns), 1 row broadcast ([1,C]),
// 2 column broadcast ([R,1]).
template <int W, int KIND>
__device__ __forceinline__ void ttj_load(const JInView& v, long long seg, long long row, long long col, float* d) {
    if (KIND == 2) {
        const float s = __ldg(v.ptr + seg * v.sseg + row * v.sr);
#pragma unroll
        for (int w = 0; w < W; ++w) d[w] = s;
    } else {
        const float* q = v.ptr + seg * v.sseg + (KIND == 1 ? 0 : row * v.sr) + col;
        if (W == 4) {
            const float4 t = __ldg(reinterpret_cast<const float4*>(q));
            d[0] = t.x;
            d[1] = t.y;
            d[2] = t.z;
            d[3] = t.w;
        } else {
            d[0] = __ldg(q);
        }
    }
}

template <int W>
__device__ __forceinline__ void ttj_store(const JOutView& v, long long seg, long long row, long long col,
                                          const float* s) {
    float* q = v.ptr + seg * v.sseg + row * v.sr + col;
    if (W == 4)
        *reinterpret_cast<float4*>(q) = make_float4(s[0], s[1], s[2], s[3]);
    else
        q[0] = s[0];
}

__device__ __forceinline__ float ttj_warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ---------------------------------------------------------------- kernels
// Software pipelining: every kernel issues the loads of its next iteration
// (Body::load into a second register buffer) before it computes the current
// one (Body::run), so the memory latency of the next tile hides behind the
// arithmetic of this one. Summation order per thread is the plain loop's.
template <class Body, int G, int W>
__device__ __forceinline__ void ttj_copy_buf(float (&dst)[Body::NB][G][W], const float (&src)[Body::NB][G][W]) {
#pragma unroll
    for (int b = 0; b < Body::NB; ++b)
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
            for (int w = 0; w < W; ++w) dst[b][g][w] = src[b][g][w];
}

template <int W, int G>
__device__ __forceinline__ void ttj_flat_index(const JParams& p, unsigned blk, unsigned (&row)[G], unsigned (&col)[G],
                                               bool (&valid)[G]) {
    const unsigned q0 = blk * (TTJ_THREADS * G) + threadIdx.x;
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const unsigned q = q0 + g * TTJ_THREADS;
        valid[g] = q < p.total;
        const unsigned r = ttj_fdiv(q, p.cpr_div);
        row[g] = r;
        col[g] = (q - r * p.cpr) * W;
    }
}

template <int W, int G, bool SIG, bool REDUCE_ALL, class Body>
__device__ __forceinline__ void ttj_flat(const JParams& p) {
    if (SIG) {
        ttj_exp_table_init();
        __syncthreads();
    }
    const long long seg = blockIdx.y;
    float sum = 0.0f;
    unsigned blk = blockIdx.x;
    unsigned row[G], col[G];
    bool valid[G];
    ttj_flat_index<W, G>(p, blk, row, col, valid);
    float buf[Body::NB][G][W];
    Body::load(p, buf, seg, row, col, valid);
    while ((unsigned long long)blk * (TTJ_THREADS * G) < p.total) {
        const unsigned nblk = blk + gridDim.x;
        unsigned nrow[G], ncol[G];
        bool nvalid[G];
        ttj_flat_index<W, G>(p, nblk, nrow, ncol, nvalid);
        float nbuf[Body::NB][G][W];
        Body::load(p, nbuf, seg, nrow, ncol, nvalid);
        float acc[G][W];
        Body::run(p, acc, buf, seg, row, col, valid);
        if (REDUCE_ALL) {
#pragma unroll
            for (int g = 0; g < G; ++g)
                if (valid[g])
#pragma unroll
                    for (int w = 0; w < W; ++w) sum += acc[g][w];
        }
        blk = nblk;
#pragma unroll
        for (int g = 0; g < G; ++g) {
            row[g] = nrow[g];
            col[g] = ncol[g];
            valid[g] = nvalid[g];
        }
        ttj_copy_buf<Body, G, W>(buf, nbuf);
    }
    if (REDUCE_ALL) {
        __shared__ float red[TTJ_THREADS / 32];
        sum = ttj_warp_sum(sum);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sum;
        __syncthreads();
        if (threadIdx.x < 32) {
            float v = threadIdx.x < TTJ_THREADS / 32 ? red[threadIdx.x] : 0.0f;
            v = ttj_warp_sum(v);
            if (threadIdx.x == 0) p.partials[seg * gridDim.x + blockIdx.x] = v;
        }
    }
}

// Row sums: a warp per row, lanes across the row's column quads; the walk
// over (row, column block) pairs is flattened so the prefetch crosses rows.
template <int W, int G>
__device__ __forceinline__ void ttj_rows_index(const JParams& p, unsigned r, unsigned c0, unsigned (&row)[G],
                                               unsigned (&col)[G], bool (&valid)[G]) {
    const unsigned lane = threadIdx.x & 31;
#pragma unroll
    for (int g = 0; g < G; ++g) {
        const unsigned ch = c0 + lane + g * 32;
        valid[g] = r < (unsigned)p.rows && ch < p.cpr;
        row[g] = r;
        col[g] = ch * W;
    }
}

template <int W, int G, bool SIG, class Body>
__device__ __forceinline__ void ttj_rows(const JParams& p) {
    if (SIG) {
        ttj_exp_table_init();
        __syncthreads();
    }
    const long long seg = blockIdx.y;
    const int lane = threadIdx.x & 31;
    const unsigned nwarps = (gridDim.x * TTJ_THREADS) >> 5;
    unsigned r = (blockIdx.x * TTJ_THREADS + threadIdx.x) >> 5;
    unsigned c0 = 0;  // warp-uniform column-quad base of this step
    unsigned row[G], col[G];
    bool valid[G];
    ttj_rows_index<W, G>(p, r, c0, row, col, valid);
    float buf[Body::NB][G][W];
    Body::load(p, buf, seg, row, col, valid);
    float sum = 0.0f;
    while (r < (unsigned)p.rows) {
        unsigned nc0 = c0 + 32 * G, nr = r;
        if (nc0 >= p.cpr) {
            nc0 = 0;
            nr = r + nwarps;
        }
        unsigned nrow[G], ncol[G];
        bool nvalid[G];
        ttj_rows_index<W, G>(p, nr, nc0, nrow, ncol, nvalid);
        float nbuf[Body::NB][G][W];
        Body::load(p, nbuf, seg, nrow, ncol, nvalid);
        float acc[G][W];
        Body::run(p, acc, buf, seg, row, col, valid);
#pragma unroll
        for (int g = 0; g < G; ++g)
            if (valid[g])
#pragma unroll
                for (int w = 0; w < W; ++w) sum += acc[g][w];
        if (nr != r) {  // row finished (warp-uniform)
            sum = ttj_warp_sum(sum);
            if (lane == 0) p.red_out[seg * p.red_sseg + r] = p.mean ? (float)((double)sum / p.count) : sum;
            sum = 0.0f;
        }
        r = nr;
        c0 = nc0;
#pragma unroll
        for (int g = 0; g < G; ++g) {
            row[g] = nrow[g];
            col[g] = ncol[g];
            valid[g] = nvalid[g];
        }
        ttj_copy_buf<Body, G, W>(buf, nbuf);
    }
}

template <int W, int G>
__device__ __forceinline__ void ttj_cols_index(int r, int r1, unsigned ch, bool col_ok, unsigned (&row)[G],
                                               unsigned (&col)[G], bool (&valid)[G]) {
    const int NW = TTJ_THREADS / 32;
#pragma unroll
    for (int g = 0; g < G; ++g) {
        row[g] = (unsigned)(r + g * NW);
        col[g] = ch * W;
        valid[g] = col_ok && r + g * NW < r1;
    }
}

template <int W, int G, bool SIG, class Body>
__device__ __forceinline__ void ttj_cols(const JParams& p) {
    const int NW = TTJ_THREADS / 32;
    if (SIG) {
        ttj_exp_table_init();
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
    int r = r0 + warp;
    unsigned row[G], col[G];
    bool valid[G];
    ttj_cols_index<W, G>(r, r1, ch, col_ok, row, col, valid);
    float buf[Body::NB][G][W];
    Body::load(p, buf, seg, row, col, valid);
    for (; r < r1; r += NW * G) {
        unsigned nrow[G], ncol[G];
        bool nvalid[G];
        ttj_cols_index<W, G>(r + NW * G, r1, ch, col_ok, nrow, ncol, nvalid);
        float nbuf[Body::NB][G][W];
        Body::load(p, nbuf, seg, nrow, ncol, nvalid);
        float acc[G][W];
        Body::run(p, acc, buf, seg, row, col, valid);
#pragma unroll
        for (int g = 0; g < G; ++g)
            if (valid[g])
#pragma unroll
                for (int w = 0; w + 1 < W; w += 2) f32x2_add(s[w], s[w + 1], acc[g][w], acc[g][w + 1]);
        if (W & 1)
#pragma unroll
            for (int g = 0; g < G; ++g)
                if (valid[g]) s[W - 1] += acc[g][W - 1];
#pragma unroll
        for (int g = 0; g < G; ++g) {
            row[g] = nrow[g];
            col[g] = ncol[g];
            valid[g] = nvalid[g];
        }
        ttj_copy_buf<Body, G, W>(buf, nbuf);
    }
    __shared__ float sm[TTJ_THREADS / 32][32 * W + 1];
#pragma unroll
    for (int w = 0; w < W; ++w) sm[warp][lane * W + w] = s[w];
    __syncthreads();
    for (int i = threadIdx.x; i < 32 * W; i += TTJ_THREADS) {
        float t = 0.0f;
#pragma unroll
        for (int k = 0; k < NW; ++k) t += sm[k][i];
        const long long c = (long long)blockIdx.x * 32 * W + i;
        if (c < p.cols) {
            if (p.nsplit == 1)
                p.red_out[seg * p.red_sseg + c] = p.mean ? (float)((double)t / p.count) : t;
            else
                p.partials[((long long)seg * p.nsplit + split) * p.cols + c] = t;
        }
    }
}

#endif  // device compilation
