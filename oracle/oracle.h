/*
 * oracle.h -- CPU restatement of tt_lazy's `namespace math` backend.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the parity checker for the CUDA
 * backend (libtt_cuda). Only tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline / reference arm may load it. The product path never calls it.
 *
 * Every function restates the arithmetic of one reference function, in the
 * same operation order, with plain IEEE single-precision operations (compiled
 * with -ffp-contract=off so no fused multiply-add changes a rounding).
 * Citations are to the reference project (ayerofieiev-tt/tt_lazy).
 *
 * Where the reference path is wrong or missing (see each function), the
 * restatement implements the documented intent and says so.
 *
 * All functions return 0 on success and a negative code on a shape error,
 * mirroring the reference's std::runtime_error; orc_last_error() gives the text.
 */
#ifndef TT_ORACLE_H
#define TT_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

const char* orc_last_error(void);

/* src/backend/cpu/eltwise.cpp:8-27 -- result[i] = std::max(0.0f, x[i]). */
int orc_relu(const float* x, float* out, size_t n);

/* README.md:332 -- 1.0f / (1.0f + std::exp(-x)); std::exp(float) is expf. */
int orc_sigmoid(const float* x, float* out, size_t n);

/* glibc's expf, restated as its x86-64 FMA build computes it, and the
 * process's own expf (libm); orc_expf_is_fma_build reports whether the
 * process's expf is that build. */
int orc_expf_ref(const float* x, float* out, size_t n);
int orc_expf_libm(const float* x, float* out, size_t n);
int orc_expf_is_fma_build(void);

/* src/backend/cpu/eltwise.cpp:29-83 -- same-shape add, or [N,M] + [1,M]. */
int orc_add(const float* a, const uint32_t* ashape, int arank,
            const float* b, const uint32_t* bshape, int brank, float* out);

/* src/backend/cpu/eltwise.cpp:85-111 -- same-shape multiply only. */
int orc_multiply(const float* a, const uint32_t* ashape, int arank,
                 const float* b, const uint32_t* bshape, int brank, float* out);

/* src/backend/cpu/matmul.cpp:36-85 -- i-j-k loop, sequential fp32 sum.
 * a is stored [a_rows_st, a_cols_st] and b is stored [b_rows_st, b_cols_st]
 * (row-major); transpose flags follow matmul.cpp:6-12 and 47-48. */
int orc_matmul(const float* a, uint32_t a_rows_st, uint32_t a_cols_st,
               const float* b, uint32_t b_rows_st, uint32_t b_cols_st,
               int transpose_a, int transpose_b, float* out);

/* src/backend/cpu/fused_ops.cpp:8-64 -- act(x . W + b), bias added after the
 * full dot product, then relu if has_relu. */
int orc_fused_mlp(const float* x, const float* w, const float* bias,
                  uint32_t batch, uint32_t in_features, uint32_t out_features,
                  int has_relu, float* out);

/* src/backend/cpu/reduce_sum.cpp:9-62 -- sum over `dims` (empty = all),
 * each output element a sequential fp32 sum in row-major order of the
 * reduced indices (the order of reduce_sum.cpp:28-52). The reference only
 * implements rank-2 dim 1 and rank-1 dim 0 and folds every other case into a
 * full sum in element 0 (reduce_sum.cpp:53-58); this restates the intended
 * per-dim reduction for every case. `mean` divides each sum by the count
 * (ReduceArgs::Type::MEAN, src/frontend/operations.hpp:13-14; no reference
 * implementation). out has the reduced shape (keepdim does not change data). */
int orc_reduce(const float* x, const uint32_t* shape, int rank,
               const int32_t* dims, int ndims, int mean, float* out);

/* Same reduction accumulated in fp64: the tolerance anchor for GPU tree
 * reductions (a sequential fp32 sum is itself ~1e-4 from exact at 1e6 terms). */
int orc_reduce_f64(const float* x, const uint32_t* shape, int rank,
                   const int32_t* dims, int ndims, int mean, double* out);

/* src/backend/cpu/transpose.cpp:7-36 -- swap the last two dims. The
 * reference transposes only the first matrix of a batched tensor; this
 * restatement transposes every matrix of the leading (batch) dims. */
int orc_transpose(const float* x, const uint32_t* shape, int rank, float* out);

/* src/backend/cpu/split.cpp:8-55 -- chunk `index` of size split_size along
 * `dim` (the last chunk may be short). The reference copies only rank-1
 * inputs (split.cpp:40-49); this restates the slice for any rank. */
int orc_split_chunk(const float* x, const uint32_t* shape, int rank,
                    int64_t split_size, int32_t dim, uint32_t index, float* out);

#ifdef __cplusplus
}
#endif
#endif
