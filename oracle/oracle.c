/*
 * oracle.c -- CPU restatement of tt_lazy's `namespace math` backend.
 *
 * TEST INFRASTRUCTURE ONLY: the parity checker for libtt_cuda. Loaded only by
 * tests/, __graft_entry__.smoke() and bench.py's CPU-baseline legs.
 *
 * Pinned: tests/test_oracle.py checks every function here against the
 * reference's own code compiled from its sources (oracle/_ref, built by
 * oracle/build_ref.sh) and against the known answers in the reference tests.
 *
 * Build: gcc -O2 -ffp-contract=off -fPIC -shared (see oracle/build.py).
 * x86-64 gcc without -mfma emits no FMA, so every `a * b + c` below is two
 * IEEE single roundings, as in the reference's g++ build.
 */
#include "oracle.h"

#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static char g_err[256];

static int fail(const char* msg) {
    snprintf(g_err, sizeof g_err, "%s", msg);
    return -1;
}

const char* orc_last_error(void) { return g_err; }

static size_t numel(const uint32_t* shape, int rank) {
    size_t n = 1;
    for (int i = 0; i < rank; ++i) n *= shape[i];
    return n;
}

static int same_shape(const uint32_t* a, int ar, const uint32_t* b, int br) {
    if (ar != br) return 0;
    for (int i = 0; i < ar; ++i)
        if (a[i] != b[i]) return 0;
    return 1;
}

/* eltwise.cpp:19-24: result = std::max(0.0f, x) == (0.0f < x) ? x : 0.0f.
 * NaN and -0.0 both map to +0.0f. */
int orc_relu(const float* x, float* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = (0.0f < x[i]) ? x[i] : 0.0f;
    return 0;
}

/* README.md:332: output = 1.0f / (1.0f + std::exp(-x)). */
int orc_sigmoid(const float* x, float* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = 1.0f / (1.0f + expf(-x[i]));
    return 0;
}

/* glibc's expf as its x86-64 FMA build computes it (glibc 2.27+,
 * sysdeps/ieee754/flt-32/e_expf.c compiled with FMA contraction, the build
 * selected on hosts with AVX2 and FMA): a restatement of the published
 * method, used to pin what the reference's std::exp(float) returns. The
 * tests compare it with this process's expf on a sweep of floats and report
 * which glibc build the host runs (orc_expf_is_fma_build). */
/* 2^(j/32) rounded to double. */
static const double g_exp2_32[32] = {
    0x1.0000000000000p+0, 0x1.059b0d3158574p+0, 0x1.0b5586cf9890fp+0, 0x1.11301d0125b51p+0,
    0x1.172b83c7d517bp+0, 0x1.1d4873168b9aap+0, 0x1.2387a6e756238p+0, 0x1.29e9df51fdee1p+0,
    0x1.306fe0a31b715p+0, 0x1.371a7373aa9cbp+0, 0x1.3dea64c123422p+0, 0x1.44e086061892dp+0,
    0x1.4bfdad5362a27p+0, 0x1.5342b569d4f82p+0, 0x1.5ab07dd485429p+0, 0x1.6247eb03a5585p+0,
    0x1.6a09e667f3bcdp+0, 0x1.71f75e8ec5f74p+0, 0x1.7a11473eb0187p+0, 0x1.82589994cce13p+0,
    0x1.8ace5422aa0dbp+0, 0x1.93737b0cdc5e5p+0, 0x1.9c49182a3f090p+0, 0x1.a5503b23e255dp+0,
    0x1.ae89f995ad3adp+0, 0x1.b7f76f2fb5e47p+0, 0x1.c199bdd85529cp+0, 0x1.cb720dcef9069p+0,
    0x1.d5818dcfba487p+0, 0x1.dfc97337b9b5fp+0, 0x1.ea4afa2a490dap+0, 0x1.f50765b6e4540p+0,
};

static float expf_glibc_fma(float x) {
    uint32_t ux;
    memcpy(&ux, &x, 4);
    const uint32_t abstop = (ux >> 20) & 0x7ff;
    if (abstop >= 0x42b) { /* |x| >= 88 or NaN */
        if (ux == 0xff800000u) return 0.0f;
        if (abstop >= 0x7f8) return x + x;
        if (x > 0x1.62e42ep6f) return INFINITY;
        if (x < -0x1.9fe368p6f) return 0.0f;
    }
    const double xd = x, inv_ln2_n = 0x1.71547652b82fep+5, shift = 0x1.8p+52;
    double kd = fma(inv_ln2_n, xd, shift);
    uint64_t ki;
    memcpy(&ki, &kd, 8);
    kd -= shift;
    const double r = fma(inv_ln2_n, xd, -kd);
    uint64_t t;
    memcpy(&t, &g_exp2_32[ki % 32], 8);
    t += (ki - ki % 32) << 47; /* exponent: (k >> 5) << 52 */
    double s;
    memcpy(&s, &t, 8);
    const double z = fma(0x1.c6af84b912394p-20, r, 0x1.ebfce50fac4f3p-13);
    const double r2 = r * r;
    double y = fma(0x1.62e42ff0c52d6p-6, r, 1.0);
    y = fma(z, r2, y);
    return (float)(y * s);
}

int orc_expf_ref(const float* x, float* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = expf_glibc_fma(x[i]);
    return 0;
}

int orc_expf_libm(const float* x, float* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = expf(x[i]);
    return 0;
}

/* 1 when this process's expf is glibc's FMA build: the two x86-64 builds
 * differ at x = 0x1.04845ep+5 (the FMA build returns 0x1.f93e38p+46). */
int orc_expf_is_fma_build(void) {
    volatile float probe = 0x1.04845ep+5f;
    const float e = expf(probe);
    uint32_t u;
    memcpy(&u, &e, 4);
    const float want = 0x1.f93e38p+46f;
    uint32_t w;
    memcpy(&w, &want, 4);
    return u == w;
}

/* Broadcast compatibility of eltwise.cpp:40-42 (Tensor::can_broadcast,
 * Tensor.cpp:495-524): trailing-aligned dims equal or 1. */
static int can_broadcast(const uint32_t* a, int ar, const uint32_t* b, int br) {
    int r = ar > br ? ar : br;
    for (int i = 0; i < r; ++i) {
        int ia = ar - 1 - i, ib = br - 1 - i;
        uint32_t da = ia >= 0 ? a[ia] : 1, db = ib >= 0 ? b[ib] : 1;
        if (da != db && da != 1 && db != 1) return 0;
    }
    return 1;
}

/* eltwise.cpp:29-83. */
int orc_add(const float* a, const uint32_t* as, int ar, const float* b, const uint32_t* bs, int br,
            float* out) {
    if (!can_broadcast(as, ar, bs, br)) return fail("Cannot broadcast shapes for addition");
    if (same_shape(as, ar, bs, br)) {
        size_t n = numel(as, ar);
        for (size_t i = 0; i < n; ++i) out[i] = a[i] + b[i];
        return 0;
    }
    /* eltwise.cpp:62-76: [N, M] + [1, M] only. */
    if (ar == 2 && br == 2 && bs[0] == 1 && as[1] == bs[1]) {
        size_t rows = as[0], cols = as[1];
        for (size_t r = 0; r < rows; ++r)
            for (size_t c = 0; c < cols; ++c) out[r * cols + c] = a[r * cols + c] + b[c];
        return 0;
    }
    return fail("Broadcasting addition not implemented for these shapes");
}

/* eltwise.cpp:85-111. */
int orc_multiply(const float* a, const uint32_t* as, int ar, const float* b, const uint32_t* bs, int br,
                 float* out) {
    if (!can_broadcast(as, ar, bs, br)) return fail("Cannot broadcast shapes for multiplication");
    if (!same_shape(as, ar, bs, br)) return fail("Broadcasting multiplication not fully implemented");
    size_t n = numel(as, ar);
    for (size_t i = 0; i < n; ++i) out[i] = a[i] * b[i];
    return 0;
}

/* matmul.cpp:36-85 with the loop of matmul.cpp:43-53. */
int orc_matmul(const float* a, uint32_t ars, uint32_t acs, const float* b, uint32_t brs, uint32_t bcs,
               int ta, int tb, float* out) {
    uint32_t a_rows = ta ? acs : ars, a_cols = ta ? ars : acs;
    uint32_t b_rows = tb ? bcs : brs, b_cols = tb ? brs : bcs;
    if (a_cols != b_rows) return fail("Matrix dimension mismatch for multiplication");
    for (uint32_t i = 0; i < a_rows; ++i) {
        for (uint32_t j = 0; j < b_cols; ++j) {
            float sum = 0.0f;
            for (uint32_t k = 0; k < a_cols; ++k) {
                float av = ta ? a[(size_t)k * a_rows + i] : a[(size_t)i * a_cols + k];
                float bv = tb ? b[(size_t)j * b_rows + k] : b[(size_t)k * b_cols + j];
                sum += av * bv;
            }
            out[(size_t)i * b_cols + j] = sum;
        }
    }
    return 0;
}

/* fused_ops.cpp:8-64 with the loop of fused_ops.cpp:39-61. */
int orc_fused_mlp(const float* x, const float* w, const float* bias, uint32_t batch, uint32_t in_f,
                  uint32_t out_f, int has_relu, float* out) {
    for (size_t r = 0; r < batch; ++r) {
        for (size_t o = 0; o < out_f; ++o) {
            float sum = 0.0f;
            for (size_t k = 0; k < in_f; ++k) sum += x[r * in_f + k] * w[k * out_f + o];
            sum += bias[o];
            if (has_relu) sum = (0.0f < sum) ? sum : 0.0f;
            out[r * out_f + o] = sum;
        }
    }
    return 0;
}

/* Output offset of each input element for a reduction over `dims`. Walking
 * the input in row-major order visits the terms of every output element in
 * row-major order of the reduced indices, i.e. the sequential order of
 * reduce_sum.cpp:28-52. */
static int reduce_plan(const uint32_t* shape, int rank, const int32_t* dims, int ndims, int red[4],
                       size_t* count) {
    if (rank < 1 || rank > 4) return fail("reduce: rank must be 1..4");
    for (int i = 0; i < 4; ++i) red[i] = 0;
    if (ndims == 0) {
        for (int i = 0; i < rank; ++i) red[i] = 1;
    } else {
        for (int j = 0; j < ndims; ++j) {
            int d = dims[j] < 0 ? dims[j] + rank : dims[j];
            if (d < 0 || d >= rank) return fail("reduce: dim out of range");
            red[d] = 1;
        }
    }
    size_t c = 1;
    for (int i = 0; i < rank; ++i)
        if (red[i]) c *= shape[i];
    *count = c;
    return 0;
}

#define REDUCE_BODY(ACC_T)                                                              \
    int red[4];                                                                         \
    size_t count;                                                                       \
    if (reduce_plan(shape, rank, dims, ndims, red, &count)) return -1;                  \
    uint32_t s[4] = {1, 1, 1, 1};                                                       \
    for (int i = 0; i < rank; ++i) s[4 - rank + i] = shape[i];                          \
    int r4[4] = {0, 0, 0, 0};                                                           \
    for (int i = 0; i < rank; ++i) r4[4 - rank + i] = red[i];                           \
    size_t os[4], acc = 1;                                                              \
    for (int i = 3; i >= 0; --i) {                                                      \
        os[i] = r4[i] ? 0 : acc;                                                        \
        if (!r4[i]) acc *= s[i];                                                        \
    }                                                                                   \
    size_t nout = acc;                                                                  \
    ACC_T* tmp = (ACC_T*)calloc(nout, sizeof(ACC_T));                                   \
    if (!tmp) return fail("reduce: out of memory");                                     \
    size_t idx = 0;                                                                     \
    for (uint32_t i0 = 0; i0 < s[0]; ++i0)                                              \
        for (uint32_t i1 = 0; i1 < s[1]; ++i1)                                          \
            for (uint32_t i2 = 0; i2 < s[2]; ++i2)                                      \
                for (uint32_t i3 = 0; i3 < s[3]; ++i3, ++idx) {                         \
                    size_t o = i0 * os[0] + i1 * os[1] + i2 * os[2] + i3 * os[3];       \
                    tmp[o] += (ACC_T)x[idx];                                            \
                }                                                                       \
    for (size_t o = 0; o < nout; ++o) out[o] = mean ? tmp[o] / (ACC_T)count : tmp[o];   \
    free(tmp);                                                                          \
    return 0;

int orc_reduce(const float* x, const uint32_t* shape, int rank, const int32_t* dims, int ndims, int mean,
               float* out) {
    REDUCE_BODY(float)
}

int orc_reduce_f64(const float* x, const uint32_t* shape, int rank, const int32_t* dims, int ndims,
                   int mean, double* out) {
    REDUCE_BODY(double)
}

/* transpose.cpp:14-30 per matrix: result[j * rows + i] = input[i * cols + j]. */
int orc_transpose(const float* x, const uint32_t* shape, int rank, float* out) {
    if (rank < 2) return fail("Transpose requires at least 2D tensor");
    size_t rows = shape[rank - 2], cols = shape[rank - 1];
    size_t batch = numel(shape, rank - 2);
    for (size_t bt = 0; bt < batch; ++bt) {
        const float* in = x + bt * rows * cols;
        float* o = out + bt * rows * cols;
        for (size_t i = 0; i < rows; ++i)
            for (size_t j = 0; j < cols; ++j) o[j * rows + i] = in[i * cols + j];
    }
    return 0;
}

/* split.cpp:17-37: chunk i covers [i*split_size, min((i+1)*split_size, size)). */
int orc_split_chunk(const float* x, const uint32_t* shape, int rank, int64_t split_size, int32_t dim,
                    uint32_t index, float* out) {
    if (dim < 0 || dim >= rank) return fail("Invalid dimension for split operation");
    if (split_size <= 0) return fail("Split size must be positive");
    size_t size = shape[dim];
    size_t nchunks = (size + (size_t)split_size - 1) / (size_t)split_size;
    if (index >= nchunks) return fail("split: chunk index out of range");
    size_t start = (size_t)index * (size_t)split_size;
    size_t len = size - start < (size_t)split_size ? size - start : (size_t)split_size;
    size_t outer = numel(shape, dim), inner = numel(shape + dim + 1, rank - dim - 1);
    for (size_t o = 0; o < outer; ++o)
        memcpy(out + o * len * inner, x + (o * size + start) * inner, len * inner * sizeof(float));
    return 0;
}
