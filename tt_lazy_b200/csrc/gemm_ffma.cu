// gemm_ffma.cu -- fp32 CUDA-core GEMM (the 1e-5 accuracy path) and the
// ttc_gemm entry point that picks between it and the tcgen05 kernels (TF32,
// and the fp32-accurate three-pass TF32X3).
//
// Replaces math::matmul (src/backend/cpu/matmul.cpp:36-85, an i-j-k loop with
// a strided read of B, 0.82 GFLOP/s) and math::fused_mlp
// (src/backend/cpu/fused_ops.cpp:8-64). The reference sums each dot product
// sequentially in fp32; this kernel accumulates with fused multiply-adds over
// 16-deep k-slices, so results differ from the CPU by rounding only
// (norm-wise ~1e-6 relative at K = 4096).
//
// 128x128 output tile per 256-thread block, 8x8 outputs per thread, k-slices
// of 16 double-buffered through shared memory, next slice prefetched into
// registers while the current one is multiplied. The epilogue program
// (bias / relu / sigmoid / stores, see ttc_internal.cuh) runs on the
// accumulators before anything is written.
#include <cstring>

#include "ttc_internal.cuh"

namespace ttc {

int run_gemm_tf32(const ttc_gemm_desc& d, const DProgram& epi, float* reduce_out, int mean, bool x3);
bool tf32_supported(const ttc_gemm_desc& d, const DProgram& epi, bool epi_vec);
int run_chain(const ttc_chain_desc& d);

namespace {

constexpr int BM = 128, BN = 128, BK = 16, kThreads = 256;

struct GemmParams {
    int M, N, K;
    const float* a;
    long long lda;
    const float* b;
    long long ldb;
    DProgram epi;
};

template <bool TA, bool TB, bool VEC>
__global__ void __launch_bounds__(kThreads) sgemm_kernel(const __grid_constant__ GemmParams p) {
    __shared__ __align__(16) float As[2][BK][BM + 4];
    __shared__ __align__(16) float Bs[2][BK][BN + 4];
    if (p.epi.has_sigmoid) {
        exp2_table_init_block();
        __syncthreads();
    }
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
    float ra[8], rb[8];

    auto a_coord = [&](int e, int& m, int& k) {
        if (!TA) {
            m = e >> 4;
            k = e & 15;
        } else {
            k = e >> 7;
            m = e & 127;
        }
    };
    auto b_coord = [&](int e, int& k, int& n) {
        if (!TB) {
            k = e >> 7;
            n = e & 127;
        } else {
            n = e >> 4;
            k = e & 15;
        }
    };
    auto load = [&](int k0) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            int m, k, n, kb;
            a_coord(tid + i * kThreads, m, k);
            const int gm = m0 + m, gk = k0 + k;
            ra[i] = (gm < p.M && gk < p.K) ? __ldg(TA ? p.a + (long long)gk * p.lda + gm
                                                      : p.a + (long long)gm * p.lda + gk)
                                           : 0.0f;
            b_coord(tid + i * kThreads, kb, n);
            const int gn = n0 + n, gkb = k0 + kb;
            rb[i] = (gn < p.N && gkb < p.K) ? __ldg(TB ? p.b + (long long)gn * p.ldb + gkb
                                                       : p.b + (long long)gkb * p.ldb + gn)
                                            : 0.0f;
        }
    };
    auto stash = [&](int buf) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            int m, k, n, kb;
            a_coord(tid + i * kThreads, m, k);
            As[buf][k][m] = ra[i];
            b_coord(tid + i * kThreads, kb, n);
            Bs[buf][kb][n] = rb[i];
        }
    };

    load(0);
    stash(0);
    __syncthreads();
    int buf = 0;
    for (int k0 = 0; k0 < p.K; k0 += BK) {
        const bool more = k0 + BK < p.K;
        if (more) load(k0 + BK);
#pragma unroll
        for (int kk = 0; kk < BK; ++kk) {
            float a[8], b[8];
            const float4 a0 = *reinterpret_cast<const float4*>(&As[buf][kk][ty * 4]);
            const float4 a1 = *reinterpret_cast<const float4*>(&As[buf][kk][64 + ty * 4]);
            const float4 b0 = *reinterpret_cast<const float4*>(&Bs[buf][kk][tx * 4]);
            const float4 b1 = *reinterpret_cast<const float4*>(&Bs[buf][kk][64 + tx * 4]);
            a[0] = a0.x; a[1] = a0.y; a[2] = a0.z; a[3] = a0.w;
            a[4] = a1.x; a[5] = a1.y; a[6] = a1.z; a[7] = a1.w;
            b[0] = b0.x; b[1] = b0.y; b[2] = b0.z; b[3] = b0.w;
            b[4] = b1.x; b[5] = b1.y; b[6] = b1.z; b[7] = b1.w;
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[i][j] = __fmaf_rn(a[i], b[j], acc[i][j]);
        }
        if (more) stash(buf ^ 1);
        __syncthreads();
        buf ^= 1;
    }

    // Epilogue: row i of this thread is m0 + (i < 4 ? ty*4 + i : 64 + ty*4 + i - 4).
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const long long row = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
        if (VEC) {
            float v[2][4];
            long long rr[2] = {row, row}, cc[2];
            bool ok[2];
#pragma unroll
            for (int g = 0; g < 2; ++g) {
                cc[g] = n0 + g * 64 + tx * 4;
                ok[g] = row < p.M && cc[g] < p.N;
#pragma unroll
                for (int w = 0; w < 4; ++w) v[g][w] = acc[i][g * 4 + w];
            }
            run_program<2, 4>(p.epi, v, 0, rr, cc, ok);
        } else {
            float v[8][1];
            long long rr[8], cc[8];
            bool ok[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                rr[j] = row;
                cc[j] = n0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + (j - 4));
                ok[j] = row < p.M && cc[j] < p.N;
                v[j][0] = acc[i][j];
            }
            run_program<8, 1>(p.epi, v, 0, rr, cc, ok);
        }
    }
}

template <bool TA, bool TB>
int launch_sgemm(const GemmParams& p, bool vec) {
    dim3 grid((p.N + BN - 1) / BN, (p.M + BM - 1) / BM);
    if (grid.y > 65535) return set_error(TTC_ERR_UNSUPPORTED, "tt_cuda: M = %d too large for the FFMA grid", p.M);
    if (vec)
        sgemm_kernel<TA, TB, true><<<grid, kThreads, 0, rt().stream>>>(p);
    else
        sgemm_kernel<TA, TB, false><<<grid, kThreads, 0, rt().stream>>>(p);
    count_launch();
    return check_cuda(cudaGetLastError(), "FFMA GEMM launch");
}

bool aligned16(const void* ptr) { return ((uintptr_t)ptr & 15) == 0; }

}  // namespace

// Epilogue views with col_stride 1 must be 16-byte aligned with row strides
// that are multiples of 4 for the 128-bit epilogue path.
bool epilogue_vec_ok(const ttc_chain_desc& e, int N) {
    if (N % 4) return false;
    for (int i = 0; i < e.n_inputs; ++i) {
        const ttc_in_view& v = e.inputs[i];
        if (v.col_stride == 0) continue;
        if (!aligned16(v.ptr) || v.row_stride % 4) return false;
    }
    for (int i = 0; i < e.n_outputs; ++i)
        if (!aligned16(e.outputs[i].ptr) || e.outputs[i].row_stride % 4) return false;
    return true;
}

// Builds the effective epilogue: an empty program means "STORE to c" (or
// nothing, when only the column sum of the product is asked for).
int make_epilogue(const ttc_gemm_desc& d, ttc_chain_desc* e) {
    *e = d.epilogue;
    if (e->reduce != TTC_REDUCE_NONE && e->reduce != TTC_REDUCE_COLS)
        return set_error(TTC_ERR_UNSUPPORTED, "tt_cuda: a GEMM epilogue reduces over rows (TTC_REDUCE_COLS) only");
    if (e->reduce == TTC_REDUCE_COLS && !e->reduce_out)
        return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: GEMM epilogue reduction without reduce_out");
    if (e->n_instr == 0 && !(e->reduce == TTC_REDUCE_COLS && !d.c)) {
        if (!d.c) return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: GEMM with no epilogue needs c");
        if (e->n_outputs != 0)
            return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: empty GEMM epilogue with outputs");
        e->n_outputs = 1;
        e->outputs[0] = ttc_out_view{d.c, d.ldc, 0};
        e->n_instr = 1;
        e->program[0] = ttc_instr{TTC_OP_STORE, 0, 0, 0};
    }
    e->rows = d.M;
    e->cols = d.N;
    e->nseg = 1;
    return TTC_OK;
}

int validate_gemm(const ttc_gemm_desc& d) {
    if (d.M < 0 || d.N < 0 || d.K < 0)
        return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: GEMM shape %d x %d x %d", d.M, d.N, d.K);
    if ((d.M && d.K && !d.a) || (d.N && d.K && !d.b))
        return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: GEMM operand is NULL");
    const long long a_min = d.trans_a ? d.M : d.K, b_min = d.trans_b ? d.K : d.N;
    if (d.lda < a_min || d.ldb < b_min)
        return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: GEMM leading dimension too small (lda %lld, ldb %lld)",
                         (long long)d.lda, (long long)d.ldb);
    return TTC_OK;
}

}  // namespace ttc

using namespace ttc;

extern "C" {

int ttc_gemm_select_path(const ttc_gemm_desc* desc) {
    if (!desc) return TTC_GEMM_FFMA;
    if (desc->path == TTC_GEMM_FFMA) return TTC_GEMM_FFMA;
    ttc_chain_desc e;
    if (make_epilogue(*desc, &e) != TTC_OK) return TTC_GEMM_FFMA;
    DProgram prog;
    if (decode_program(e, true, &prog) != TTC_OK) return TTC_GEMM_FFMA;
    if (tf32_supported(*desc, prog, epilogue_vec_ok(e, desc->N)))
        return desc->path == TTC_GEMM_TF32X3 ? TTC_GEMM_TF32X3 : TTC_GEMM_TF32;
    return TTC_GEMM_FFMA;
}

int ttc_gemm(const ttc_gemm_desc* desc) {
    TTC_REQUIRE_INIT();
    if (!desc) return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: desc is NULL");
    const ttc_gemm_desc& d = *desc;
    if (int rc = validate_gemm(d)) return rc;
    ttc_chain_desc e;
    if (int rc = make_epilogue(d, &e)) return rc;
    const bool reduce = e.reduce == TTC_REDUCE_COLS;
    if (d.M == 0 || d.N == 0) {
        if (!reduce || d.N == 0) return TTC_OK;
        ttc_chain_desc z;  // column sums over no rows: 0 (NaN for a mean); the input is never read
        std::memset(&z, 0, sizeof z);
        z.rows = 0;
        z.cols = d.N;
        z.nseg = 1;
        z.n_inputs = 1;
        z.inputs[0] = ttc_in_view{e.reduce_out, d.N, 1, 0};
        z.n_instr = 1;
        z.program[0] = ttc_instr{TTC_OP_LOAD, TTC_SRC_INPUT, 0, 0};
        z.reduce = TTC_REDUCE_COLS;
        z.reduce_mean = e.reduce_mean;
        z.reduce_out = e.reduce_out;
        return run_chain(z);
    }
    GemmParams p;
    std::memset(&p, 0, sizeof p);
    if (int rc = decode_program(e, true, &p.epi)) return rc;
    const bool vec = epilogue_vec_ok(e, d.N);
    if (d.path != TTC_GEMM_FFMA && tf32_supported(d, p.epi, vec))
        return run_gemm_tf32(d, p.epi, reduce ? e.reduce_out : nullptr, e.reduce_mean, d.path == TTC_GEMM_TF32X3);
    if (reduce) {
        // FFMA path: the final epilogue value goes to a scratch matrix, then
        // one column-sum chain over it.
        if (d.path == TTC_GEMM_TF32)
            return set_error(TTC_ERR_UNSUPPORTED, "tt_cuda: TF32 path does not take this GEMM (%d x %d x %d)", d.M,
                             d.N, d.K);
        if (e.n_outputs >= TTC_CHAIN_MAX_OUTPUTS || e.n_instr >= TTC_CHAIN_MAX_INSTR)
            return set_error(TTC_ERR_UNSUPPORTED, "tt_cuda: GEMM epilogue too long to add a column sum");
        float* tmp = nullptr;
        TTC_CUDA(cudaMallocAsync((void**)&tmp, (size_t)d.M * d.N * sizeof(float), rt().stream));
        ttc_gemm_desc g = d;
        g.epilogue = e;
        g.epilogue.reduce = TTC_REDUCE_NONE;
        g.epilogue.reduce_out = nullptr;
        g.epilogue.outputs[g.epilogue.n_outputs] = ttc_out_view{tmp, d.N, 0};
        g.epilogue.program[g.epilogue.n_instr++] = ttc_instr{TTC_OP_STORE, 0, (uint8_t)g.epilogue.n_outputs++, 0};
        g.path = TTC_GEMM_FFMA;
        int rc = ttc_gemm(&g);
        if (rc == TTC_OK) {
            ttc_chain_desc r;
            std::memset(&r, 0, sizeof r);
            r.rows = d.M;
            r.cols = d.N;
            r.nseg = 1;
            r.n_inputs = 1;
            r.inputs[0] = ttc_in_view{tmp, d.N, 1, 0};
            r.n_instr = 1;
            r.program[0] = ttc_instr{TTC_OP_LOAD, TTC_SRC_INPUT, 0, 0};
            r.reduce = TTC_REDUCE_COLS;
            r.reduce_mean = e.reduce_mean;
            r.reduce_out = e.reduce_out;
            rc = run_chain(r);
        }
        cudaFreeAsync(tmp, rt().stream);
        return rc;
    }
    if (d.path == TTC_GEMM_TF32)
        return set_error(TTC_ERR_UNSUPPORTED,
                         "tt_cuda: TF32 path needs M, N multiples of 128/16 and K of 32 with 16-byte aligned rows "
                         "(got %d x %d x %d)",
                         d.M, d.N, d.K);
    p.M = d.M;
    p.N = d.N;
    p.K = d.K;
    p.a = d.a;
    p.lda = d.lda;
    p.b = d.b;
    p.ldb = d.ldb;
    if (!d.trans_a && !d.trans_b) return launch_sgemm<false, false>(p, vec);
    if (d.trans_a && !d.trans_b) return launch_sgemm<true, false>(p, vec);
    if (!d.trans_a && d.trans_b) return launch_sgemm<false, true>(p, vec);
    return launch_sgemm<true, true>(p, vec);
}

}  // extern "C"
