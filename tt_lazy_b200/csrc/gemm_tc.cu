// gemm_tc.cu -- TF32 tensor-core GEMM for sm_100a: tcgen05.mma (kind::tf32)
// with accumulators in tensor memory, operands staged by TMA, and the
// element-wise epilogue program applied on the way out of TMEM.
//
// Replaces math::matmul (src/backend/cpu/matmul.cpp:36-85) and
// math::fused_mlp (src/backend/cpu/fused_ops.cpp:8-64) on the fast path:
// norm-wise relative error ~1e-3 (TF32 keeps 10 mantissa bits of each
// operand; accumulation is fp32).
//
// Structure (one CTA per SM, persistent over output tiles):
//   warp 0     TMA producer: per k-block, one TMA box (K-major operand) or
//              one box per 32 columns (MN-major operand) into a 4-stage ring
//              of shared-memory buffers (128-byte swizzle).
//   warp 1     allocates 512 TMEM columns (two 128x256 fp32 accumulators),
//              then one lane issues 4 tcgen05.mma (K = 8 each) per k-block and
//              commits each stage back to the producer and each finished tile
//              to the epilogue.
//   warps 2-5  epilogue: tcgen05.ld 32 columns at a time (each warp reads
//              its own 32 TMEM lanes = 32 output rows), run the epilogue
//              program (bias / relu / sigmoid / store), release the
//              accumulator so the MMA warp can start the tile after next.
// The tile order is grouped by 16 row-blocks so the A and B panels a wave of
// CTAs touches stay in the 126 MB L2.
//
// The CTA-pair kernel below (tcgen05.mma.cta_group::2) runs as clusters of
// 2; the single-CTA kernels launch no clusters. No kernel here uses TMA
// multicast, and every TMA load reads this GPU's own memory into the issuing
// CTA's shared memory: the kernels also run on every rank of a multi-GPU job.
// Every mbarrier wait is bounded (about 2 s); an expired
// wait records an error in a host-mapped status word, lets the other roles
// time out too, waits for its own TMA loads, frees TMEM and returns.
#include <cstdlib>
#include <cstring>

#include "tma_util.cuh"

namespace ttc {

namespace {

constexpr int BM = 128, BN = 256, BK = 32, STAGES = 4;
constexpr int A_BYTES = BM * BK * 4;  // 16 KB
constexpr int B_BYTES = BN * BK * 4;  // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int kThreads = 192;
constexpr int GROUP_M = 16;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
// TF32X3 variant: 128x128 output tiles, 3 stages of 64 KB (A and B, each as
// its TF32 part and TF32 remainder), same shared memory footprint.
constexpr int X3_BN = 128, X3_STAGES = 3;
constexpr int X3_SMEM_BYTES = X3_STAGES * 2 * (A_BYTES + X3_BN * BK * 4) + 1024 + 256;
static_assert(X3_SMEM_BYTES <= SMEM_BYTES, "TF32X3 stages exceed the kernel's shared memory");

struct TcParams {
    CUtensorMap tma_a;
    CUtensorMap tma_b;
    CUtensorMap tma_a2;  // TF32X3: the TF32 remainders of A and B (same geometry)
    CUtensorMap tma_b2;
    int M, N, K;
    int m_blocks, n_blocks, k_blocks;
    int a_mn_major, b_mn_major;
    unsigned idesc;
    int* status;
    long long wait_limit;  // cycles a bounded wait spins before it gives up
    int stall;             // failure-detection test: the producer issues no loads
    DProgram epi;
    float* partials;  // column sums of the final epilogue value per 32-row group, or null
    // Split-K (single-CTA kernel only). Work items [0, full_tiles) are whole
    // tiles 0 .. full_tiles - 1 with the fused epilogue; every later tile t
    // is `splits` work items, split s covering k-blocks
    // [kb_per_split * s, ...), each storing its raw accumulator tile into
    // split_ws (tile-local, row-major BM x tile width, at slot
    // (t - full_tiles) * splits + s); a second kernel adds a tile's splits in
    // split order and runs the epilogue on the sum. full_tiles = 0 splits
    // every tile (GEMMs with few tiles); full_tiles = the tiles of the full
    // waves splits only the last, partly filled wave's tiles.
    int full_tiles, splits, kb_per_split;
    float* split_ws;
    // TF32X3: nonzero where a row block of A / a column block of B holds an
    // infinity or NaN; such tiles take the big * big product alone.
    const int* nonfinite_a;
    const int* nonfinite_b;
};

__device__ __forceinline__ void work_item(const TcParams& p, int w, int& tile, int& split, int& kb0, int& kb1) {
    if (w < p.full_tiles) {
        tile = w;
        split = -1;
        kb0 = 0;
        kb1 = p.k_blocks;
        return;
    }
    const int v = w - p.full_tiles;
    tile = p.full_tiles + v / p.splits;
    split = v % p.splits;
    kb0 = split * p.kb_per_split;
    kb1 = min(p.k_blocks, kb0 + p.kb_per_split);
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_mma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: register j of lane l = TMEM
// (lane base + l, column + j).
__device__ __forceinline__ void tc_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tc_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Column sums over a warp's 32 rows (one per lane) of 16 consecutive columns
// (v[g][w] is column 4 g + w; invalid elements already zeroed): a fixed-order
// transpose reduction, 16 shuffles; lanes 2c and 2c+1 end with column c and
// the even lane writes it to out[c] when c < ncols (columns past the matrix
// edge would land in the next row group's partials). Deterministic.
__device__ __forceinline__ void warp_col_sums16(const float (&v)[4][4], float* out, int lane, long long ncols) {
    // The epilogue program branches per lane (row validity, sigmoid's range
    // test): reconverge the warp before the shuffles read other lanes.
    __syncwarp();
    float a[16];
#pragma unroll
    for (int g = 0; g < 4; ++g)
#pragma unroll
        for (int w = 0; w < 4; ++w) a[4 * g + w] = v[g][w];
    const bool h16 = lane & 16, h8 = lane & 8, h4 = lane & 4, h2 = lane & 2;
    float b[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
        b[i] = (h16 ? a[i + 8] : a[i]) + __shfl_xor_sync(0xffffffffu, h16 ? a[i] : a[i + 8], 16);
#pragma unroll
    for (int i = 0; i < 4; ++i)
        b[i] = (h8 ? b[i + 4] : b[i]) + __shfl_xor_sync(0xffffffffu, h8 ? b[i] : b[i + 4], 8);
#pragma unroll
    for (int i = 0; i < 2; ++i)
        b[i] = (h4 ? b[i + 2] : b[i]) + __shfl_xor_sync(0xffffffffu, h4 ? b[i] : b[i + 2], 4);
    float c = (h2 ? b[1] : b[0]) + __shfl_xor_sync(0xffffffffu, h2 ? b[0] : b[1], 2);
    c += __shfl_xor_sync(0xffffffffu, c, 1);
    if ((lane & 1) == 0 && ((lane >> 1) & 15) < ncols) out[(lane >> 1) & 15] = c;
}

// Shared-memory matrix descriptor (sm_100 layout: start address, leading /
// stride byte offsets in 16-byte units, version 1, layout type in bits
// 61-63). Layout 2 = 128-byte rows swizzled in 16-byte chunks over 8 rows
// (K-major operands); layout 1 = 128-byte rows swizzled in 32-byte chunks
// over 4 rows, the only layout tcgen05 accepts for MN-major 32-bit operands.
constexpr uint32_t kLayoutSW128 = 2, kLayoutSW128Base32 = 1;
__device__ __forceinline__ uint64_t make_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                              uint32_t layout) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFF);
    d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
    d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)layout << 61;
    return d;
}

__device__ __forceinline__ void tile_coords(int tile, int m_blocks, int n_blocks, int& mb, int& nb) {
    const int per_group = GROUP_M * n_blocks;
    const int group = tile / per_group;
    const int first_m = group * GROUP_M;
    const int gm = min(GROUP_M, m_blocks - first_m);
    const int local = tile - group * per_group;
    mb = first_m + local % gm;
    nb = local / gm;
}

template <bool X3>
__global__ void __launch_bounds__(kThreads, 1) tf32_gemm_kernel(const __grid_constant__ TcParams p) {
    // X3: 128x128 tiles, stages of [A big | B big | A small | B small].
    constexpr int TBN = X3 ? X3_BN : BN, TSTAGES = X3 ? X3_STAGES : STAGES;
    constexpr int TB_BYTES = TBN * BK * 4;
    constexpr int TSTAGE = X3 ? 2 * (A_BYTES + TB_BYTES) : A_BYTES + TB_BYTES;
    constexpr int TTMEM = 2 * TBN;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = (uint64_t*)(smem + TSTAGES * TSTAGE);
    uint32_t* tmem_slot = (uint32_t*)(bars + 2 * TSTAGES + 4);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar0 = smem_u32(bars);
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (TSTAGES + s); };
    auto tfull_bar = [&](int b) { return bar0 + 8u * (2 * TSTAGES + b); };
    auto tempty_bar = [&](int b) { return bar0 + 8u * (2 * TSTAGES + 2 + b); };

    if (threadIdx.x == 0) {
        for (int s = 0; s < TSTAGES; ++s) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(tfull_bar(b), 1);
            mbar_init(tempty_bar(b), 4);
        }
        mbar_fence_init();
    }
    if (p.epi.has_sigmoid) exp2_table_init_block();
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(TTMEM)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int num_work = p.full_tiles + (p.m_blocks * p.n_blocks - p.full_tiles) * p.splits;
    bool failed = false;

    if (warp == 0) {
        if (lane == 0) {
            asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&p.tma_a) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)&p.tma_b) : "memory");
            int stage = 0;
            uint32_t phase = 0;
            long long issued = 0;
            for (int w = blockIdx.x; w < num_work && !failed && !p.stall; w += gridDim.x) {
                int tile, split, kb0, kb1;
                work_item(p, w, tile, split, kb0, kb1);
                int mb, nb;
                tile_coords(tile, p.m_blocks, p.n_blocks, mb, nb);
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait(empty_bar(stage), phase ^ 1, p.wait_limit)) {
                        failed = true;
                        break;
                    }
                    mbar_arrive_expect_tx(full_bar(stage), TSTAGE);
                    const uint32_t a_dst = sbase + stage * TSTAGE, b_dst = a_dst + A_BYTES;
                    if (!p.a_mn_major) {
                        tma_load_2d(a_dst, &p.tma_a, full_bar(stage), kb * BK, mb * BM);
                    } else {
#pragma unroll
                        for (int j = 0; j < BM / 32; ++j)
                            tma_load_2d(a_dst + j * (BK * 128), &p.tma_a, full_bar(stage), mb * BM + 32 * j, kb * BK);
                    }
                    if (!p.b_mn_major) {
                        tma_load_2d(b_dst, &p.tma_b, full_bar(stage), kb * BK, nb * TBN);
                    } else {
#pragma unroll
                        for (int j = 0; j < TBN / 32; ++j)
                            tma_load_2d(b_dst + j * (BK * 128), &p.tma_b, full_bar(stage), nb * TBN + 32 * j, kb * BK);
                    }
                    if (X3) {  // the same boxes of the small parts
                        const uint32_t a2_dst = b_dst + TB_BYTES, b2_dst = a2_dst + A_BYTES;
                        if (!p.a_mn_major) {
                            tma_load_2d(a2_dst, &p.tma_a2, full_bar(stage), kb * BK, mb * BM);
                        } else {
#pragma unroll
                            for (int j = 0; j < BM / 32; ++j)
                                tma_load_2d(a2_dst + j * (BK * 128), &p.tma_a2, full_bar(stage), mb * BM + 32 * j,
                                            kb * BK);
                        }
                        if (!p.b_mn_major) {
                            tma_load_2d(b2_dst, &p.tma_b2, full_bar(stage), kb * BK, nb * TBN);
                        } else {
#pragma unroll
                            for (int j = 0; j < TBN / 32; ++j)
                                tma_load_2d(b2_dst + j * (BK * 128), &p.tma_b2, full_bar(stage), nb * TBN + 32 * j,
                                            kb * BK);
                        }
                    }
                    ++issued;
                    if (++stage == TSTAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            // Never leave with loads in flight: wait (bounded) for the most
            // recent load of every stage to land.
            const long long last = issued < TSTAGES ? issued : TSTAGES;
            for (long long i = 0; i < last; ++i) {
                const long long n = issued - 1 - i;
                const int s = (int)(n % TSTAGES);
                const uint32_t ph = (uint32_t)((n / TSTAGES) & 1);
                if (!mbar_wait(full_bar(s), ph, p.wait_limit)) failed = true;
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // K-major: 8-row atoms of 1024 B (SBO), K advances 32 B per MMA
            // inside the 128-byte row. MN-major: one TMA box of 32 rows x 128 B
            // per 32 columns (LBO = box size), 4-row atoms of 512 B (SBO), K
            // advances 8 rows = 1024 B per MMA.
            const uint32_t a_lbo = p.a_mn_major ? BK * 128 : 16, a_sbo = p.a_mn_major ? 512 : 1024;
            const uint32_t b_lbo = p.b_mn_major ? BK * 128 : 16, b_sbo = p.b_mn_major ? 512 : 1024;
            const uint32_t a_lay = p.a_mn_major ? kLayoutSW128Base32 : kLayoutSW128;
            const uint32_t b_lay = p.b_mn_major ? kLayoutSW128Base32 : kLayoutSW128;
            const uint32_t a_kstep = p.a_mn_major ? 8 * 128 : 32;
            const uint32_t b_kstep = p.b_mn_major ? 8 * 128 : 32;
            int stage = 0;
            uint32_t phase = 0;
            int t = 0;
            for (int w = blockIdx.x; w < num_work && !failed; w += gridDim.x, ++t) {
                int tile, split, kb0, kb1;
                work_item(p, w, tile, split, kb0, kb1);
                bool cross = X3;  // the big * small + small * big terms
                if (X3 && p.nonfinite_a) {
                    // An infinity times the other operand's remainder, which is
                    // often exactly zero, would make NaN where fp32 gives +-inf.
                    int mb, nb;
                    tile_coords(tile, p.m_blocks, p.n_blocks, mb, nb);
                    cross = !(__ldcg(p.nonfinite_a + mb) | __ldcg(p.nonfinite_b + nb));
                }
                const int b = t & 1;
                const uint32_t acc_phase = (t >> 1) & 1;
                if (!mbar_wait(tempty_bar(b), acc_phase ^ 1, p.wait_limit)) {
                    failed = true;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(b * TBN);
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!mbar_wait(full_bar(stage), phase, p.wait_limit)) {
                        failed = true;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_s = sbase + stage * TSTAGE, b_s = a_s + A_BYTES;
#pragma unroll
                    for (int k = 0; k < BK / 8; ++k) {
                        const uint64_t ad = make_desc(a_s + k * a_kstep, a_lbo, a_sbo, a_lay);
                        const uint64_t bd = make_desc(b_s + k * b_kstep, b_lbo, b_sbo, b_lay);
                        tc_mma_tf32(d_tmem, ad, bd, p.idesc, (kb != kb0 || k != 0) ? 1u : 0u);
                        if (cross) {  // + big * small + small * big
                            const uint32_t a2_s = b_s + TB_BYTES, b2_s = a2_s + A_BYTES;
                            const uint64_t ad2 = make_desc(a2_s + k * a_kstep, a_lbo, a_sbo, a_lay);
                            const uint64_t bd2 = make_desc(b2_s + k * b_kstep, b_lbo, b_sbo, b_lay);
                            tc_mma_tf32(d_tmem, ad, bd2, p.idesc, 1u);
                            tc_mma_tf32(d_tmem, ad2, bd, p.idesc, 1u);
                        }
                    }
                    tc_commit(empty_bar(stage));
                    if (++stage == TSTAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (failed) break;
                tc_commit(tfull_bar(b));
            }
        }
    } else {
        const int q = warp & 3;  // this warp's quarter of the 128 TMEM lanes
        // Bias / activation / stores / column sums of one 32-column slice of
        // this lane's row, from the tile's final values v32.
        auto finish = [&](int mb, int nb, int c, const float (&v32)[32]) {
            const long long row = (long long)mb * BM + q * 32 + lane;
            const long long col0 = (long long)nb * TBN + c * 32;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                float v[4][4];
                long long rr[4], cc[4];
                bool vv[4];
#pragma unroll
                for (int g = 0; g < 4; ++g) {
                    rr[g] = row;
                    cc[g] = col0 + h * 16 + g * 4;
                    vv[g] = row < p.M && cc[g] < p.N;
#pragma unroll
                    for (int w = 0; w < 4; ++w) v[g][w] = v32[h * 16 + g * 4 + w];
                }
                run_program<4, 4>(p.epi, v, 0, rr, cc, vv);
                if (p.partials) {
#pragma unroll
                    for (int g = 0; g < 4; ++g)
#pragma unroll
                        for (int w = 0; w < 4; ++w) v[g][w] = vv[g] ? v[g][w] : 0.0f;
                    const long long rg = (long long)mb * (BM / 32) + q;
                    warp_col_sums16(v, p.partials + rg * p.N + col0 + h * 16, lane, p.N - (col0 + h * 16));
                }
            }
        };
        int t = 0;
        for (int wi = blockIdx.x; wi < num_work; wi += gridDim.x, ++t) {
            int tile, split, kb0, kb1;
            work_item(p, wi, tile, split, kb0, kb1);
            int mb, nb;
            tile_coords(tile, p.m_blocks, p.n_blocks, mb, nb);
            const int b = t & 1;
            const uint32_t acc_phase = (t >> 1) & 1;
            const bool ok = __all_sync(0xffffffffu, mbar_wait(tfull_bar(b), acc_phase, p.wait_limit));
            if (split < 0) {
                if (!ok) {
                    failed = true;
                    break;
                }
                tc_fence_after();
                for (int c = 0; c < TBN / 32; ++c) {
                    uint32_t r[32];
                    tc_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * TBN + c * 32), r);
                    tc_wait_ld();
                    if ((long long)nb * TBN + c * 32 >= p.N) continue;
                    float v32[32];
#pragma unroll
                    for (int j = 0; j < 32; ++j) v32[j] = __uint_as_float(r[j]);
                    finish(mb, nb, c, v32);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(tempty_bar(b));
                continue;
            }
            // Split-K: store this split's raw tile and release the accumulator.
            if (!ok) {
                failed = true;
                break;
            }
            tc_fence_after();
            const long long slot = (long long)(tile - p.full_tiles) * p.splits + split;
            float* const dst = p.split_ws + (slot * BM + q * 32 + lane) * TBN;
            for (int c = 0; c < TBN / 32; ++c) {
                uint32_t r[32];
                tc_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * TBN + c * 32), r);
                tc_wait_ld();
#pragma unroll
                for (int j = 0; j < 32; j += 4)
                    *reinterpret_cast<float4*>(dst + c * 32 + j) =
                        make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]), __uint_as_float(r[j + 2]),
                                    __uint_as_float(r[j + 3]));
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(tempty_bar(b));
        }
    }

    if (failed) *(volatile int*)p.status = 1;
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TTMEM)
                     : "memory");
}

// Split-K epilogue: one warp per (split tile, 32-row group, 16-column group),
// lane = row. Adds the tile's splits in split order (deterministic), then runs
// the epilogue program and, for a fused column sum, writes the same
// per-32-row-group partials as the GEMM epilogue (rows past M contributing
// zeros).
struct SplitEpiParams {
    const float* ws;
    int full_tiles, split_tiles, splits, tile_n;  // tile_n: tile width (256, 128 for TF32X3)
    int m_blocks, n_blocks, M, N;
    DProgram epi;
    float* partials;
};

__global__ void __launch_bounds__(256) splitk_epilogue_kernel(const __grid_constant__ SplitEpiParams p) {
    if (p.epi.has_sigmoid) exp2_table_init_block();
    __syncthreads();
    const int lane = threadIdx.x & 31;
    const int cg_per_tile = p.tile_n / 16, warps_per_tile = (BM / 32) * cg_per_tile;
    const long long warp_id = (long long)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (warp_id >= (long long)p.split_tiles * warps_per_tile) return;  // whole warps only
    const int tt = (int)(warp_id / warps_per_tile), rem = (int)(warp_id % warps_per_tile);
    const int q = rem / cg_per_tile, cg = rem % cg_per_tile;
    int mb, nb;
    tile_coords(p.full_tiles + tt, p.m_blocks, p.n_blocks, mb, nb);
    const long long row = (long long)mb * BM + q * 32 + lane;
    const long long col0 = (long long)nb * p.tile_n + cg * 16;
    if (col0 >= p.N) return;  // warp-uniform
    const long long split_stride = (long long)BM * p.tile_n;
    const float* src = p.ws + ((long long)tt * p.splits * BM + q * 32 + lane) * p.tile_n + cg * 16;
    float v[4][4];
    long long rr[4], cc[4];
    bool vv[4];
#pragma unroll
    for (int g = 0; g < 4; ++g) {
        rr[g] = row;
        cc[g] = col0 + 4 * g;
        vv[g] = row < p.M && cc[g] < p.N;
    }
    // Four splits' loads in flight per round trip; the adds stay in split order.
    for (int s0 = 0; s0 < p.splits; s0 += 4) {
        float4 t[4][4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
            if (s0 + u < p.splits)
#pragma unroll
                for (int g = 0; g < 4; ++g)
                    t[u][g] = __ldcg(reinterpret_cast<const float4*>(src + (s0 + u) * split_stride + 4 * g));
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            if (s0 + u >= p.splits) break;
#pragma unroll
            for (int g = 0; g < 4; ++g) {
                if (s0 + u == 0) {
                    v[g][0] = t[u][g].x;
                    v[g][1] = t[u][g].y;
                    v[g][2] = t[u][g].z;
                    v[g][3] = t[u][g].w;
                } else {
                    v[g][0] += t[u][g].x;
                    v[g][1] += t[u][g].y;
                    v[g][2] += t[u][g].z;
                    v[g][3] += t[u][g].w;
                }
            }
        }
    }
    run_program<4, 4>(p.epi, v, 0, rr, cc, vv);
    if (p.partials) {
#pragma unroll
        for (int g = 0; g < 4; ++g)
#pragma unroll
            for (int w = 0; w < 4; ++w) v[g][w] = vv[g] ? v[g][w] : 0.0f;
        const long long rg = (long long)mb * (BM / 32) + q;
        warp_col_sums16(v, p.partials + rg * p.N + col0, lane, p.N - col0);
    }
}

// ------------------------------------------------------------------ pair MMA
// The CTA-pair variant: a cluster of two CTAs on two SMs computes a 256x256
// output tile with tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 8). CTA r of
// the pair holds rows [128 r, 128 r + 128) of the A tile and columns
// [128 r, 128 r + 128) of the B tile in its own shared memory, and receives
// its 128 output rows x 256 columns in its own TMEM. Per 32-deep k-block a CTA
// loads 32 KB (16 KB of A, 16 KB of B) instead of the single-CTA kernel's
// 48 KB for the same 128x256 MACs: two thirds of the L2 -> SM traffic, which
// is what bounds the single-CTA kernel.
//
// Roles (both CTAs): warp 0 TMA producer into this CTA's 6-stage ring, each
// stage completing on this CTA's own full barrier; warp 1 of CTA 0 issues the
// MMAs once both CTAs' stage is full, and commits stage / accumulator
// releases to the barriers of both CTAs (one commit per CTA address); warp 1
// of CTA 1 forwards "my stage s is full" to CTA 0 (it waits on its own full
// barrier, so every CTA observes the completion of its own loads); warps 2-5
// are the epilogue of the CTA's 128 rows and release the accumulator on
// CTA 0's barrier (8 arrivals: 4 warps x 2 CTAs). All waits are bounded.
// Every TMA load lands in the issuing CTA's own shared memory.
constexpr int P_BNH = 128;                      // B columns per CTA
constexpr int P_BN = 2 * P_BNH;                 // N of the pair tile
constexpr int P_STAGES = 6;  // 5 and 7 measured the same on the MLP's GEMMs
constexpr int P_A_BYTES = BM * BK * 4;          // 16 KB
constexpr int P_B_BYTES = P_BNH * BK * 4;       // 16 KB
constexpr int P_STAGE_BYTES = P_A_BYTES + P_B_BYTES;
constexpr int P_TMEM_COLS = 2 * P_BN;           // two 128 x 256 accumulators
// Pair-tile rows per raster group. Measured on 8192x16384x4096 (pair
// kernel, one launch): 8 rows read 2.27 GB from DRAM in 1.61 ms, 16 rows
// 2.57 GB in 1.62 ms; 4 and 32 ran 1-4 % slower on the MLP's shapes. With
// K = 4096 every 256-row A panel and 256-column B panel is 4 MB, and the
// panels a wave of 74 clusters touches exceed what one die's half of the L2
// keeps, so the operands are re-read ~6x whatever the group (the L2 bound,
// not the raster order, sets the traffic).
constexpr int P_GROUP_M = 8;
constexpr int P_SMEM_BYTES = P_STAGES * P_STAGE_BYTES + 1024 + 256;

__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// Address of the same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_addr(uint32_t local, uint32_t rank) {
    uint32_t out;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(local), "r"(rank));
    return out;
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_bar) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}
// Relaxed remote arrive for the per-stage forward: the forwarding thread has
// already observed the stage's TMA bytes land (its own full barrier), so the
// data is in shared memory before the arrive; a release arrive would add a
// cluster-scope fence to every k-block and made the forward the bottleneck
// (about 1.5k cycles each, measured: 358 vs 827 TFLOP/s on zero data).
__device__ __forceinline__ void mbar_arrive_cluster_relaxed(uint32_t cluster_bar) {
    asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_bar) : "memory");
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void tc2_commit(uint32_t cluster_bar) {
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cluster_bar)
                 : "memory");
}
__device__ __forceinline__ void tc2_mma_tf32(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void pair_tile_coords(int tile, int m2_blocks, int n_blocks, int& mb2, int& nb) {
    const int per_group = P_GROUP_M * n_blocks;
    const int group = tile / per_group;
    const int first_m = group * P_GROUP_M;
    const int gm = min(P_GROUP_M, m2_blocks - first_m);
    const int local = tile - group * per_group;
    mb2 = first_m + local % gm;
    nb = local / gm;
}

// p.m_blocks counts 256-row pair tiles, p.n_blocks 256-column tiles.
__global__ void __launch_bounds__(kThreads, 1) tf32_gemm_pair_kernel(const __grid_constant__ TcParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = (uint64_t*)(smem + P_STAGES * P_STAGE_BYTES);
    uint32_t* tmem_slot = (uint32_t*)(bars + 2 * P_STAGES + 4);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar0 = smem_u32(bars);
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (P_STAGES + s); };
    auto tfull_bar = [&](int b) { return bar0 + 8u * (2 * P_STAGES + b); };
    auto tempty_bar = [&](int b) { return bar0 + 8u * (2 * P_STAGES + 2 + b); };

    if (threadIdx.x == 0) {
        for (int s = 0; s < P_STAGES; ++s) {
            mbar_init(full_bar(s), rank == 0 ? 2 : 1);  // CTA 0: own producer + the peer's forward
            mbar_init(empty_bar(s), 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(tfull_bar(b), 1);
            mbar_init(tempty_bar(b), 8);
        }
        mbar_fence_init();
    }
    if (p.epi.has_sigmoid) exp2_table_init_block();
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(P_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // both CTAs' barriers are initialised before anyone signals across
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    const int num_tiles = p.m_blocks * p.n_blocks;
    const int cluster_id = blockIdx.x >> 1, nclusters = gridDim.x >> 1;
    bool failed = false;

    if (warp == 0) {
        if (lane == 0) {
            prefetch_tensor_map(&p.tma_a);
            prefetch_tensor_map(&p.tma_b);
            int stage = 0;
            uint32_t phase = 0;
            long long issued = 0;
            for (int tile = cluster_id; tile < num_tiles && !failed && !p.stall; tile += nclusters) {
                int mb2, nb;
                pair_tile_coords(tile, p.m_blocks, p.n_blocks, mb2, nb);
                const int row0 = mb2 * (2 * BM) + (int)rank * BM;
                const int col0 = nb * P_BN + (int)rank * P_BNH;
                for (int kb = 0; kb < p.k_blocks; ++kb) {
                    if (!mbar_wait(empty_bar(stage), phase ^ 1, p.wait_limit)) {
                        failed = true;
                        break;
                    }
                    mbar_arrive_expect_tx(full_bar(stage), P_STAGE_BYTES);
                    const uint32_t a_dst = sbase + stage * P_STAGE_BYTES, b_dst = a_dst + P_A_BYTES;
                    if (!p.a_mn_major) {
                        tma_load_2d(a_dst, &p.tma_a, full_bar(stage), kb * BK, row0);
                    } else {
#pragma unroll
                        for (int j = 0; j < BM / 32; ++j)
                            tma_load_2d(a_dst + j * (BK * 128), &p.tma_a, full_bar(stage), row0 + 32 * j, kb * BK);
                    }
                    if (!p.b_mn_major) {
                        tma_load_2d(b_dst, &p.tma_b, full_bar(stage), kb * BK, col0);
                    } else {
#pragma unroll
                        for (int j = 0; j < P_BNH / 32; ++j)
                            tma_load_2d(b_dst + j * (BK * 128), &p.tma_b, full_bar(stage), col0 + 32 * j, kb * BK);
                    }
                    ++issued;
                    if (++stage == P_STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
            // Never leave with loads in flight (CTA 1's own full barrier sees
            // exactly its loads; CTA 0's also needs the peer's forward, which
            // comes unless the peer failed -- then this wait expires).
            const long long last = issued < P_STAGES ? issued : P_STAGES;
            for (long long i = 0; i < last; ++i) {
                const long long n = issued - 1 - i;
                if (!mbar_wait(full_bar((int)(n % P_STAGES)), (uint32_t)((n / P_STAGES) & 1), p.wait_limit)) failed = true;
            }
        }
    } else if (warp == 1 && rank == 1) {
        if (lane == 0) {
            // forward every completed stage of this CTA to CTA 0's full barrier
            int stage = 0;
            uint32_t phase = 0;
            for (int tile = cluster_id; tile < num_tiles && !failed; tile += nclusters) {
                for (int kb = 0; kb < p.k_blocks; ++kb) {
                    if (!mbar_wait(full_bar(stage), phase, p.wait_limit)) {
                        failed = true;
                        break;
                    }
                    mbar_arrive_cluster_relaxed(cluster_addr(full_bar(stage), 0));
                    if (++stage == P_STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t a_lbo = p.a_mn_major ? BK * 128 : 16, a_sbo = p.a_mn_major ? 512 : 1024;
            const uint32_t b_lbo = p.b_mn_major ? BK * 128 : 16, b_sbo = p.b_mn_major ? 512 : 1024;
            const uint32_t a_lay = p.a_mn_major ? kLayoutSW128Base32 : kLayoutSW128;
            const uint32_t b_lay = p.b_mn_major ? kLayoutSW128Base32 : kLayoutSW128;
            const uint32_t a_kstep = p.a_mn_major ? 8 * 128 : 32;
            const uint32_t b_kstep = p.b_mn_major ? 8 * 128 : 32;
            int stage = 0;
            uint32_t phase = 0;
            int t = 0;
            for (int tile = cluster_id; tile < num_tiles && !failed; tile += nclusters, ++t) {
                const int b = t & 1;
                const uint32_t acc_phase = (t >> 1) & 1;
                if (!mbar_wait(tempty_bar(b), acc_phase ^ 1, p.wait_limit)) {
                    failed = true;
                    break;
                }
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(b * P_BN);
                for (int kb = 0; kb < p.k_blocks; ++kb) {
                    if (!mbar_wait(full_bar(stage), phase, p.wait_limit)) {
                        failed = true;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_s = sbase + stage * P_STAGE_BYTES, b_s = a_s + P_A_BYTES;
#pragma unroll
                    for (int k = 0; k < BK / 8; ++k) {
                        const uint64_t ad = make_desc(a_s + k * a_kstep, a_lbo, a_sbo, a_lay);
                        const uint64_t bd = make_desc(b_s + k * b_kstep, b_lbo, b_sbo, b_lay);
                        tc2_mma_tf32(d_tmem, ad, bd, p.idesc, (kb | k) != 0 ? 1u : 0u);
                    }
                    tc2_commit(cluster_addr(empty_bar(stage), 0));
                    tc2_commit(cluster_addr(empty_bar(stage), 1));
                    if (++stage == P_STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (failed) break;
                tc2_commit(cluster_addr(tfull_bar(b), 0));
                tc2_commit(cluster_addr(tfull_bar(b), 1));
            }
        }
    } else {
        const int q = warp & 3;  // this warp's quarter of the 128 TMEM lanes
        int t = 0;
        for (int tile = cluster_id; tile < num_tiles; tile += nclusters, ++t) {
            int mb2, nb;
            pair_tile_coords(tile, p.m_blocks, p.n_blocks, mb2, nb);
            const int b = t & 1;
            const uint32_t acc_phase = (t >> 1) & 1;
            const bool ok = __all_sync(0xffffffffu, mbar_wait(tfull_bar(b), acc_phase, p.wait_limit));
            if (!ok) {
                failed = true;
                break;
            }
            tc_fence_after();
            const long long row = (long long)mb2 * (2 * BM) + rank * BM + q * 32 + lane;
            for (int c = 0; c < P_BN / 32; ++c) {
                uint32_t r[32];
                tc_ld_32x32b_x32(tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * P_BN + c * 32), r);
                tc_wait_ld();
                const long long col0 = (long long)nb * P_BN + c * 32;
                if (col0 >= p.N) continue;
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    float v[4][4];
                    long long rr[4], cc[4];
                    bool vv[4];
#pragma unroll
                    for (int g = 0; g < 4; ++g) {
                        rr[g] = row;
                        cc[g] = col0 + h * 16 + g * 4;
                        vv[g] = row < p.M && cc[g] < p.N;
#pragma unroll
                        for (int w = 0; w < 4; ++w) v[g][w] = __uint_as_float(r[h * 16 + g * 4 + w]);
                    }
                    run_program<4, 4>(p.epi, v, 0, rr, cc, vv);
                    if (p.partials) {
#pragma unroll
                        for (int g = 0; g < 4; ++g)
#pragma unroll
                            for (int w = 0; w < 4; ++w) v[g][w] = vv[g] ? v[g][w] : 0.0f;
                        const long long rg = (long long)mb2 * (2 * BM / 32) + rank * (BM / 32) + q;
                        warp_col_sums16(v, p.partials + rg * p.N + col0 + h * 16, lane, p.N - (col0 + h * 16));
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(cluster_addr(tempty_bar(b), 0));
        }
    }

    if (failed) *(volatile int*)p.status = 1;
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // the pair's MMAs and signals are done before TMEM is freed or a CTA exits
    tc_fence_after();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(P_TMEM_COLS)
                     : "memory");
}

// 2-D fp32 tensor map over a row-major matrix with `outer` rows of `inner`
// elements (row pitch ld elements), box {32, box_outer}, out-of-bounds reads
// filled with zeros. K-major tiles use the 16-byte-chunk 128-byte swizzle;
// MN-major tiles the 32-byte-chunk one (matching descriptor layout 1).
// TF32X3 operand split. big = x rounded to TF32 (nearest, ties to even; a
// rounding that would carry into the exponent's all-ones pattern truncates
// instead), small = (x - big) rounded the same way, so x = big + small to
// ~2^-22 relative and both parts pass the tensor core's TF32 reading
// unchanged. Non-finite x: big = x, small = 0.
__device__ __forceinline__ float tf32_rn(float x) {
    const unsigned u = __float_as_uint(x);
    if ((u & 0x7f800000u) == 0x7f800000u) return x;
    const unsigned r = (u + 0xfffu + ((u >> 13) & 1u)) & 0xffffe000u;
    return __uint_as_float((r & 0x7f800000u) == 0x7f800000u ? (u & 0xffffe000u) : r);
}

// Rows of a stored operand (rows x cols, leading dimension lds) into dense
// big / small copies with leading dimension ldd; blocks stride over rows,
// threads over columns (coalesced).
// A non-finite element sets flags[(by_col ? c : r) / blk]: the row block of
// A or the column block of B (in output-tile units) it belongs to.
__global__ void __launch_bounds__(256) tf32_split_kernel(const float* __restrict__ src, long long rows, long long cols,
                                                         long long lds, float* __restrict__ big,
                                                         float* __restrict__ small, long long ldd, int* flags,
                                                         int by_col, int blk) {
    for (long long r = blockIdx.x; r < rows; r += gridDim.x) {
        for (long long c = threadIdx.x; c < cols; c += blockDim.x) {
            const float x = __ldg(src + r * lds + c);
            const float b = tf32_rn(x);
            const bool finite = (__float_as_uint(x) & 0x7f800000u) != 0x7f800000u;
            big[r * ldd + c] = b;
            small[r * ldd + c] = finite ? tf32_rn(__fsub_rn(x, b)) : 0.0f;
            if (!finite) atomicOr(flags + (by_col ? c : r) / blk, 1);
        }
    }
}

int make_map(CUtensorMap* map, const float* ptr, long long inner, long long outer, long long ld, int box_outer,
             bool mn_major) {
    const unsigned long long dims[2] = {(unsigned long long)inner, (unsigned long long)outer};
    const unsigned long long strides[1] = {(unsigned long long)ld};
    const unsigned box[2] = {32, (unsigned)box_outer};
    return encode_tensor_map_f32(map, ptr, 2, dims, strides, box,
                                 mn_major ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B);
}

}  // namespace

bool tf32_supported(const ttc_gemm_desc& d, const DProgram& epi, bool epi_vec) {
    (void)epi;
    if (d.M < 1 || d.N < 1 || d.K < 1) return false;
    if (!epi_vec) return false;
    if (d.lda % 4 || d.ldb % 4) return false;
    if (((uintptr_t)d.a & 15) || ((uintptr_t)d.b & 15)) return false;
    if ((long long)d.M * d.N < 128 * 64) return false;  // too small to fill a tensor-core tile
    return true;
}

namespace {

// The CTA-pair kernel (cta_group::2, 256x256 per pair) runs by default when
// its tiles fill the GPU: at least one tile per CTA pair (sms / 2). Measured
// back to back on the large MLP step (power-capped at 1 kW, both kernels held
// to the same clocks), the device-resident step rate is the same (553 / 550
// vs 552 / 550 TFLOP/s) and the streamed end-to-end step, whose GEMMs run
// beside the host-to-device copies, is faster (583 / 583 vs 537 / 537
// TFLOP/s). Each CTA of a pair loads half of the B tile, so the kernel pulls
// 2/3 of the single-CTA kernel's operand bytes from L2.
// With fewer tiles the single-CTA kernel (and its split-K) keeps more SMs
// busy. TTC_GEMM_PAIR=0 / 1 (read at every call) forces it off / on.
bool use_pair(const ttc_gemm_desc& d, int sms) {
    if (d.M < 2 * BM || d.N < P_BN) return false;
    const char* e = getenv("TTC_GEMM_PAIR");
    if (e && e[0] == '0') return false;
    if (e && e[0] == '1') return true;
    const long long pair_tiles = (long long)((d.M + 2 * BM - 1) / (2 * BM)) * ((d.N + P_BN - 1) / P_BN);
    return pair_tiles >= sms / 2;
}

int launch_pair(TcParams& p) {
    static int max_clusters_by_dev[kMaxDevices] = {};  // 0: not queried yet on that device
    if (rt().device < 0 || rt().device >= kMaxDevices)
        return set_error(TTC_ERR_UNSUPPORTED, "tt_cuda: device %d", rt().device);
    int& max_clusters = max_clusters_by_dev[rt().device];
    cudaLaunchConfig_t cfg;
    std::memset(&cfg, 0, sizeof cfg);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = P_SMEM_BYTES;
    cfg.stream = rt().stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (max_clusters < 1) {
        TTC_CUDA(cudaFuncSetAttribute(tf32_gemm_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      P_SMEM_BYTES));
        cfg.gridDim = dim3(2 * (rt().sm_count / 2), 1, 1);
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, tf32_gemm_pair_kernel, &cfg) != cudaSuccess || n < 1) {
            cudaGetLastError();
            n = rt().sm_count / 2;
        }
        max_clusters = n;
    }
    const long long tiles = (long long)p.m_blocks * p.n_blocks;
    const int clusters = (int)(tiles < max_clusters ? tiles : max_clusters);
    cfg.gridDim = dim3(2 * clusters, 1, 1);
    TTC_CUDA(cudaLaunchKernelEx(&cfg, tf32_gemm_pair_kernel, p));
    count_launch();
    return TTC_OK;
}

// Split-K for GEMMs with too few output tiles to occupy the GPU (the small
// MLP's 256 x 1024 x 512 is 8 tiles on 148 SMs): at most one work item per
// SM, at least 4 k-blocks (128 deep) per split, at most 16 splits. Fewer,
// deeper splits write and re-read fewer partial tiles: the small MLP ran at
// 34.9 us per graph replay with 4 k-blocks per split, 41.0 with 2 (3 and 8
// measured as 4). Off with TTC_GEMM_SPLITK=0 (read at every call).
int split_count(long long tiles, int k_blocks, int sms) {
    const char* e = getenv("TTC_GEMM_SPLITK");
    if ((e && e[0] == '0') || tiles * 2 > sms || k_blocks < 8) return 1;
    const long long fill = (sms + tiles - 1) / tiles;
    constexpr long long cap = 16, min_kb = 4;
    return (int)std::max<long long>(1, std::min<long long>(std::min<long long>(fill, k_blocks / min_kb), cap));
}

// Split of the last, partly filled wave (opt-in: TTC_GEMM_TAILSPLIT=1, read
// at every call). With W full waves of `sms` tiles and R < sms tiles left, a
// wave model says the launch takes W + 1 wave times and splitting the R tiles
// along K into s parts takes W + ceil(R s / sms) / s (4096x4096 on 148 SMs:
// 3 + 68 tiles -> 3.5 instead of 4). Measured, the partly filled wave is much
// shorter than a full one (its CTAs share the L2 bandwidth that bounds this
// kernel with fewer others): 4096^3 gained 3 % (229 vs 236 us), 4096x4096x1024
// lost 10 % and 2048x4096x16384 lost 1 % to the extra epilogue launch and the
// partial tiles' traffic, so it is not the default. Returns s (1: no split)
// and the number of whole tiles in *full.
int tail_split(long long tiles, int k_blocks, int sms, int* full) {
    const char* e = getenv("TTC_GEMM_TAILSPLIT");
    if (!(e && e[0] == '1') || tiles < sms || k_blocks < 32) return 1;
    const long long waves = tiles / sms, rest = tiles % sms;
    if (rest == 0) return 1;
    int best = 1;
    double best_t = (double)(waves + 1);
    for (int s = 2; s <= 4; ++s) {
        if (k_blocks < 2 * s) break;
        const double t = (double)waves + (double)((rest * s + sms - 1) / sms) / s;
        if (t < best_t - 1e-9) {
            best_t = t;
            best = s;
        }
    }
    if (best == 1 || best_t > 0.95 * (double)(waves + 1)) return 1;
    *full = (int)(waves * sms);
    return best;
}

}  // namespace

void launch_finalize_cols(const float* partials, int nsplit, int cols, int nseg, float* out, long long sseg, int mean,
                          double count);

// `reduce_out` (or null): column sums (mean with `mean`) of the final
// epilogue value over the M rows, from per-32-row partial sums the epilogue
// writes into the workspace and a fixed-order fp64 finalize.
int run_gemm_tf32(const ttc_gemm_desc& d, const DProgram& epi, float* reduce_out, int mean, bool x3) {
    static bool attr_set_by_dev[kMaxDevices] = {};
    if (rt().device < 0 || rt().device >= kMaxDevices)
        return set_error(TTC_ERR_UNSUPPORTED, "tt_cuda: device %d", rt().device);
    bool& attr_set = attr_set_by_dev[rt().device];
    if (!attr_set) {
        TTC_CUDA(cudaFuncSetAttribute(tf32_gemm_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      SMEM_BYTES));
        TTC_CUDA(cudaFuncSetAttribute(tf32_gemm_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      X3_SMEM_BYTES));
        attr_set = true;
    }
    const bool pair = !x3 && use_pair(d, rt().sm_count);
    const int bn = pair ? P_BNH : x3 ? X3_BN : BN;  // B columns one CTA loads per tile
    TcParams p;
    std::memset(&p, 0, sizeof p);
    p.a_mn_major = d.trans_a ? 1 : 0;
    p.b_mn_major = d.trans_b ? 0 : 1;
    // Stored operands: A is [M, K] ([K, M] when trans_a), B is [K, N] ([N, K]
    // when trans_b). TF32X3 reads dense big / small copies of both.
    const long long a_rows = d.trans_a ? d.K : d.M, a_cols = d.trans_a ? d.M : d.K;
    const long long b_rows = d.trans_b ? d.N : d.K, b_cols = d.trans_b ? d.K : d.N;
    const long long a_ld = x3 ? (a_cols + 3) & ~3ll : d.lda, b_ld = x3 ? (b_cols + 3) & ~3ll : d.ldb;
    const size_t a_part = ((size_t)a_rows * a_ld * sizeof(float) + 255) & ~(size_t)255;
    const size_t b_part = ((size_t)b_rows * b_ld * sizeof(float) + 255) & ~(size_t)255;
    size_t x3_bytes = x3 ? 2 * (a_part + b_part) : 0;  // + the non-finite block flags (below)
    const float* a_ptr[2] = {d.a, nullptr};
    const float* b_ptr[2] = {d.b, nullptr};
    p.M = d.M;
    p.N = d.N;
    p.K = d.K;
    const int tm = pair ? 2 * BM : BM, tn = pair ? P_BN : x3 ? X3_BN : BN;  // output tile of one CTA / CTA pair
    p.m_blocks = (d.M + tm - 1) / tm;
    p.n_blocks = (d.N + tn - 1) / tn;
    p.k_blocks = (d.K + BK - 1) / BK;
    p.idesc = (1u << 4)                       // D format: f32
              | (2u << 7) | (2u << 10)        // A, B format: tf32
              | ((unsigned)p.a_mn_major << 15) | ((unsigned)p.b_mn_major << 16) |
              ((unsigned)(tn >> 3) << 17)     // N
              | ((unsigned)(tm >> 4) << 24);  // M (256 for the pair: 128 rows per CTA)
    if (int rc = device_status_ptr(&p.status)) return rc;
    p.stall = stall_test("gemm") ? 1 : 0;
    p.wait_limit = p.stall ? kStallTestLimitCycles : kWaitLimitCycles;
    p.epi = epi;
    const long long tiles = (long long)p.m_blocks * p.n_blocks;
    if (tiles > INT32_MAX) return set_error(TTC_ERR_UNSUPPORTED, "tt_cuda: too many GEMM tiles");
    const long long groups = (long long)p.m_blocks * (tm / 32);  // every 32-row group of every row tile
    if (reduce_out && groups > INT32_MAX)
        return set_error(TTC_ERR_UNSUPPORTED, "tt_cuda: too many rows for the fused column sum");
    // split-K: every tile when there are few (or, opt-in, the tiles of a
    // partly filled last wave)
    p.full_tiles = (int)tiles;
    p.splits = 1;
    if (!pair) {
        const int s = split_count(tiles, p.k_blocks, rt().sm_count);
        if (s > 1) {
            p.full_tiles = 0;
            p.splits = s;
        } else {
            int full = 0;
            const int ts = tail_split(tiles, p.k_blocks, rt().sm_count, &full);
            if (ts > 1) {
                p.full_tiles = full;
                p.splits = ts;
            }
        }
    }
    p.kb_per_split = (p.k_blocks + p.splits - 1) / p.splits;
    p.splits = (p.k_blocks + p.kb_per_split - 1) / p.kb_per_split;  // every split has k-blocks
    if (p.splits == 1) p.full_tiles = (int)tiles;
    const long long split_tiles = tiles - p.full_tiles;
    const size_t part_bytes = reduce_out ? ((size_t)groups * d.N * sizeof(float) + 255) & ~(size_t)255 : 0;
    const size_t split_bytes =
        split_tiles ? ((size_t)split_tiles * p.splits * BM * tn * sizeof(float) + 255) & ~(size_t)255 : 0;
    if (x3) x3_bytes += ((size_t)(p.m_blocks + p.n_blocks) * sizeof(int) + 255) & ~(size_t)255;
    if (part_bytes + split_bytes + x3_bytes) {
        void* ws = nullptr;
        if (int rc = workspace(part_bytes + split_bytes + x3_bytes, &ws)) return rc;
        if (reduce_out) p.partials = (float*)ws;
        if (split_tiles) p.split_ws = (float*)((char*)ws + part_bytes);
        if (x3) {
            char* x = (char*)ws + part_bytes + split_bytes;
            float* parts[4] = {(float*)x, (float*)(x + a_part), (float*)(x + 2 * a_part),
                               (float*)(x + 2 * a_part + b_part)};
            int* flags = (int*)(x + 2 * (a_part + b_part));  // [m_blocks] for A, then [n_blocks] for B
            TTC_CUDA(cudaMemsetAsync(flags, 0, (size_t)(p.m_blocks + p.n_blocks) * sizeof(int), rt().stream));
            const int sms = rt().sm_count;
            // A stored [M, K]: its row r is output row r; stored [K, M]: column c is.
            tf32_split_kernel<<<(unsigned)std::min<long long>(a_rows, 8ll * sms), 256, 0, rt().stream>>>(
                d.a, a_rows, a_cols, d.lda, parts[0], parts[1], a_ld, flags, d.trans_a ? 1 : 0, BM);
            count_launch();
            // B stored [K, N]: its column c is output column c; stored [N, K]: row r is.
            tf32_split_kernel<<<(unsigned)std::min<long long>(b_rows, 8ll * sms), 256, 0, rt().stream>>>(
                d.b, b_rows, b_cols, d.ldb, parts[2], parts[3], b_ld, flags + p.m_blocks, d.trans_b ? 0 : 1,
                tn);
            count_launch();
            p.nonfinite_a = flags;
            p.nonfinite_b = flags + p.m_blocks;
            if (int rc = check_cuda(cudaGetLastError(), "TF32X3 operand split launch")) return rc;
            a_ptr[0] = parts[0];
            a_ptr[1] = parts[1];
            b_ptr[0] = parts[2];
            b_ptr[1] = parts[3];
        }
    }
    // A: logical [M, K]; K-major when stored [M, K] (trans_a = 0).
    // B: logical [K, N]; MN-major when stored [K, N] (trans_b = 0).
    for (int h = 0; h < (x3 ? 2 : 1); ++h) {
        CUtensorMap* ma = h ? &p.tma_a2 : &p.tma_a;
        CUtensorMap* mb_ = h ? &p.tma_b2 : &p.tma_b;
        if (!p.a_mn_major) {
            if (int rc = make_map(ma, a_ptr[h], d.K, d.M, a_ld, BM, false)) return rc;
        } else {
            if (int rc = make_map(ma, a_ptr[h], d.M, d.K, a_ld, BK, true)) return rc;
        }
        if (p.b_mn_major) {
            if (int rc = make_map(mb_, b_ptr[h], d.N, d.K, b_ld, BK, true)) return rc;
        } else {
            if (int rc = make_map(mb_, b_ptr[h], d.K, d.N, b_ld, bn, false)) return rc;
        }
    }
    if (pair) {
        if (int rc = launch_pair(p)) return rc;
        if (int rc = check_cuda(cudaGetLastError(), "TF32 pair GEMM launch")) return rc;
    } else {
        const long long work = p.full_tiles + split_tiles * p.splits;
        const int grid = (int)(work < rt().sm_count ? work : rt().sm_count);
        if (x3)
            tf32_gemm_kernel<true><<<grid, kThreads, X3_SMEM_BYTES, rt().stream>>>(p);
        else
            tf32_gemm_kernel<false><<<grid, kThreads, SMEM_BYTES, rt().stream>>>(p);
        count_launch();
        if (int rc = check_cuda(cudaGetLastError(), "TF32 GEMM launch")) return rc;
        if (split_tiles) {
            SplitEpiParams e;
            std::memset(&e, 0, sizeof e);
            e.ws = p.split_ws;
            e.full_tiles = p.full_tiles;
            e.split_tiles = (int)split_tiles;
            e.splits = p.splits;
            e.tile_n = tn;
            e.m_blocks = p.m_blocks;
            e.n_blocks = p.n_blocks;
            e.M = d.M;
            e.N = d.N;
            e.epi = epi;
            e.partials = p.partials;
            const long long warps = split_tiles * (BM / 32) * (tn / 16);
            splitk_epilogue_kernel<<<(unsigned)((warps + 7) / 8), 256, 0, rt().stream>>>(e);
            count_launch();
            if (int rc = check_cuda(cudaGetLastError(), "split-K epilogue launch")) return rc;
        }
    }
    if (reduce_out) {  // rows past M contribute exact zeros
        launch_finalize_cols(p.partials, (int)groups, d.N, 1, reduce_out, 0, mean, (double)d.M);
        return check_cuda(cudaGetLastError(), "column-sum finalize launch");
    }
    return TTC_OK;
}

}  // namespace ttc
