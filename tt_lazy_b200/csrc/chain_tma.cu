// chain_tma.cu -- TMA-staged element-wise chain kernel: the fast path of
// ttc_eltwise_chain for contiguous, 16-byte aligned operands with cols >= 64.
//
// One persistent CTA per SM. Warp 8 is the producer: it streams tiles of
// every full input (TR x TC elements, TC in {64, 128, 256}, G * 1024
// elements per input) with 2-D / 3-D TMA into a ring of shared-memory stages,
// so the bytes in flight per SM (up to ~190 KB) are independent of
// registers. Warps 0-7 (256 threads) run the element-wise program on the
// staged tile: each thread owns G float4 groups (one column quad, G rows), so
// one dispatch of a program step covers 4G elements and the interpreter's
// per-step cost is amortised over 32 elements at G = 8. Outputs leave as
// coalesced 128-bit stores; the tail reduction stays in registers until the
// end of a work item. Broadcast operands ([1,C] bias, [R,1] column) are read
// through L1 from global memory.
//
// Work items: one tile (no reduction / full reduction), one row band with
// all its column tiles (reduction over cols), or one column band over a
// split of the row tiles (reduction over rows). Every mbarrier wait is
// bounded; an expired wait turns the consumer warp into a pass-through (it
// keeps taking the same named barriers, so nobody deadlocks), records the
// failure in the host-mapped status word, and the producer never exits with
// a TMA load in flight.
#include <algorithm>
#include <cstring>

#include "tma_util.cuh"

namespace ttc {

void launch_finalize_all(const float* partials, int nparts, float* out, int mean, double count);
void launch_finalize_cols(const float* partials, int nsplit, int cols, int nseg, float* out, long long sseg, int mean,
                          double count);

namespace {

constexpr int kConsumers = 256;
constexpr int kThreads = kConsumers + 32;
constexpr int kMaxStages = 8;
constexpr int kSmemBudget = 196 * 1024;

struct Params {
    CUtensorMap maps[TTC_CHAIN_MAX_INPUTS];
    DProgram prog;
    int slot_of[TTC_CHAIN_MAX_INPUTS];  // staged buffer of input k; -1: read from global
    int is3d[TTC_CHAIN_MAX_INPUTS];
    int n_staged, stages, tile_bytes;
    int rows, cols, nseg;
    int tc, tr, tc_shift, rpp;  // tile cols / rows, log2(tc/4), tile rows per group pass
    int tiles_r, tiles_c;
    int mode;
    int nsplit, split_tiles;
    unsigned n_items;  // < 2^31
    float* red_out;
    long long red_sseg;
    float* partials;
    int mean;
    double count;
    int* status;
    long long wait_limit;  // cycles a bounded wait spins before it gives up
    int stall;             // failure-detection test: the producer issues no loads
};

template <int G>
struct StagedIO {
    const Params& p;
    const uint8_t* stage_base;  // staged slot 0 of the current stage
    const int (&q)[G];          // float4 index of each group inside the tile
    long long seg;
    const long long (&row)[G];
    const long long (&col)[G];
    const bool (&valid)[G];
    __device__ __forceinline__ bool ok(int g) const { return valid[g]; }
    __device__ __forceinline__ void load(int k, int g, float (&dst)[4]) const {
        const int slot = p.slot_of[k];
        if (slot >= 0) {
            const float4 v = *reinterpret_cast<const float4*>(stage_base + slot * p.tile_bytes + q[g] * 16);
            dst[0] = v.x;
            dst[1] = v.y;
            dst[2] = v.z;
            dst[3] = v.w;
        } else {
            load_group<4>(p.prog.in[k], seg, row[g], col[g], dst);
        }
    }
    __device__ __forceinline__ void store(int j, int g, const float (&src)[4]) const {
        store_group<4>(p.prog.out[j], seg, row[g], col[g], src);
    }
};

struct Item {
    int seg, rt0, nrt, ct0, nct;
};

// Work-item decoding in 32-bit unsigned arithmetic (the host guarantees
// n_items < 2^31); a 64-bit divide is a long software sequence and this runs
// once per item in every consumer thread.
__device__ __forceinline__ Item item_of(const Params& p, unsigned i) {
    Item it;
    if (p.mode == TTC_REDUCE_ROWS) {  // a row band, all column tiles
        const unsigned tr = (unsigned)p.tiles_r;
        it.seg = (int)(i / tr);
        it.rt0 = (int)(i - (unsigned)it.seg * tr);
        it.nrt = 1;
        it.ct0 = 0;
        it.nct = p.tiles_c;
    } else if (p.mode == TTC_REDUCE_COLS) {  // a column band, one split of the row tiles
        const unsigned per_seg = (unsigned)p.tiles_c * (unsigned)p.nsplit;
        it.seg = (int)(i / per_seg);
        const unsigned rem = i - (unsigned)it.seg * per_seg;
        it.ct0 = (int)(rem / (unsigned)p.nsplit);
        it.nct = 1;
        it.rt0 = (int)(rem - (unsigned)it.ct0 * (unsigned)p.nsplit) * p.split_tiles;
        it.nrt = min(p.split_tiles, p.tiles_r - it.rt0);
    } else {  // a single tile
        const unsigned per_seg = (unsigned)p.tiles_r * (unsigned)p.tiles_c;
        it.seg = (int)(i / per_seg);
        const unsigned rem = i - (unsigned)it.seg * per_seg;
        it.rt0 = (int)(rem / (unsigned)p.tiles_c);
        it.nrt = 1;
        it.ct0 = (int)(rem - (unsigned)it.rt0 * (unsigned)p.tiles_c);
        it.nct = 1;
    }
    return it;
}

template <int G, int NS>
__global__ void __launch_bounds__(kThreads, 1) chain_staged_kernel(const __grid_constant__ Params p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    const int stage_bytes = p.n_staged * p.tile_bytes;
    uint64_t* bars = (uint64_t*)(smem + p.stages * stage_bytes);
    float* red = (float*)(bars + 2 * kMaxStages);  // max(G, 4) * kConsumers floats
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t bar0 = smem_u32(bars);
    auto full_bar = [&](int s) { return bar0 + 8u * s; };
    auto empty_bar = [&](int s) { return bar0 + 8u * (kMaxStages + s); };
    if (threadIdx.x == 0) {
        for (int s = 0; s < p.stages; ++s) {
            mbar_init(full_bar(s), 1);
            mbar_init(empty_bar(s), kConsumers / 32);
        }
        mbar_fence_init();
    }
    if (p.prog.has_sigmoid) exp2_table_init_block();
    __syncthreads();

    if (warp == kConsumers / 32) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            for (int k = 0; k < p.prog.n_in; ++k)
                if (p.slot_of[k] >= 0) prefetch_tensor_map(&p.maps[k]);
            int stage = 0;
            uint32_t phase = 0;
            long long issued = 0;
            bool failed = false;
            for (unsigned i = blockIdx.x; i < p.n_items && !failed && !p.stall; i += gridDim.x) {
                const Item it = item_of(p, i);
                for (int r = 0; r < it.nrt && !failed; ++r) {
                    for (int c = 0; c < it.nct; ++c) {
                        if (!mbar_wait(empty_bar(stage), phase ^ 1, p.wait_limit)) {
                            failed = true;
                            break;
                        }
                        mbar_arrive_expect_tx(full_bar(stage), stage_bytes);
                        const uint32_t dst0 = smem_u32(smem + stage * stage_bytes);
                        const int x = (it.ct0 + c) * p.tc, y = (it.rt0 + r) * p.tr;
                        for (int k = 0; k < p.prog.n_in; ++k) {
                            const int slot = p.slot_of[k];
                            if (slot < 0) continue;
                            if (p.is3d[k])
                                tma_load_3d(dst0 + slot * p.tile_bytes, &p.maps[k], full_bar(stage), x, y, it.seg);
                            else
                                tma_load_2d(dst0 + slot * p.tile_bytes, &p.maps[k], full_bar(stage), x, y);
                        }
                        ++issued;
                        if (++stage == p.stages) {
                            stage = 0;
                            phase ^= 1;
                        }
                    }
                }
            }
            // Never exit with a load in flight: the last load of every stage lands first.
            const long long last = issued < p.stages ? issued : p.stages;
            for (long long j = 0; j < last; ++j) {
                const long long n = issued - 1 - j;
                if (!mbar_wait(full_bar((int)(n % p.stages)), (uint32_t)((n / p.stages) & 1), p.wait_limit)) failed = true;
            }
            if (failed) *(volatile int*)p.status = 1;
        }
        return;
    }

    // ------------------------------------------------------------- consumers
    const int t = threadIdx.x;
    const int per_row = p.tc >> 2;  // threads (float4 columns) per tile row
    const int c4 = t & (per_row - 1), r0 = t >> p.tc_shift;
    int q[G];
#pragma unroll
    for (int g = 0; g < G; ++g) q[g] = (r0 + g * p.rpp) * per_row + c4;
    int stage = 0;
    uint32_t phase = 0;
    bool failed = false;
    float run_sum = 0.0f;
    for (unsigned i = blockIdx.x; i < p.n_items; i += gridDim.x) {
        const Item it = item_of(p, i);
        float rsum[G];
        float csum[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int g = 0; g < G; ++g) rsum[g] = 0.0f;
        for (int r = 0; r < it.nrt; ++r) {
            for (int c = 0; c < it.nct; ++c) {
                if (!failed) failed = !__all_sync(0xffffffffu, mbar_wait(full_bar(stage), phase, p.wait_limit));
                if (!failed) {
                    long long row[G], col[G];
                    bool valid[G];
                    const long long rbase = (long long)(it.rt0 + r) * p.tr + r0;
                    const long long cc = (long long)(it.ct0 + c) * p.tc + c4 * 4;
#pragma unroll
                    for (int g = 0; g < G; ++g) {
                        row[g] = rbase + g * p.rpp;
                        col[g] = cc;
                        valid[g] = row[g] < p.rows && cc < p.cols;
                    }
                    float acc[G][4];
                    each<G, 4>([&](int g, int w) { acc[g][w] = 0.0f; });
                    const StagedIO<G> io{p, smem + stage * stage_bytes, q, (long long)it.seg, row, col, valid};
                    run_program_io<G, 4, NS>(p.prog, acc, io);
                    if (p.mode != TTC_REDUCE_NONE) {
#pragma unroll
                        for (int g = 0; g < G; ++g) {
                            if (!valid[g]) continue;
                            if (p.mode == TTC_REDUCE_COLS) {
#pragma unroll
                                for (int w = 0; w < 4; ++w) csum[w] += acc[g][w];
                            } else {
                                const float s4 = (acc[g][0] + acc[g][1]) + (acc[g][2] + acc[g][3]);
                                if (p.mode == TTC_REDUCE_ALL)
                                    run_sum += s4;
                                else
                                    rsum[g] += s4;
                            }
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(empty_bar(stage));
                if (++stage == p.stages) {
                    stage = 0;
                    phase ^= 1;
                }
            }
        }
        if (p.mode == TTC_REDUCE_ROWS) {
            // Tile row rr = r0 + g * rpp is shared by the per_row threads with that r0.
#pragma unroll
            for (int g = 0; g < G; ++g) red[g * kConsumers + t] = rsum[g];
            named_barrier(1, kConsumers);
            for (int rr = t; rr < p.tr; rr += kConsumers) {
                const int g = rr / p.rpp, rl = rr % p.rpp;
                float s = 0.0f;
                for (int j = 0; j < per_row; ++j) s += red[g * kConsumers + rl * per_row + j];
                const long long row = (long long)it.rt0 * p.tr + rr;
                if (row < p.rows && !failed)
                    p.red_out[(long long)it.seg * p.red_sseg + row] = p.mean ? (float)((double)s / p.count) : s;
            }
            named_barrier(1, kConsumers);
        } else if (p.mode == TTC_REDUCE_COLS) {
            // Column quad c4 is shared by the rpp threads with that c4.
#pragma unroll
            for (int w = 0; w < 4; ++w) red[w * kConsumers + t] = csum[w];
            named_barrier(1, kConsumers);
            for (int cc = t; cc < p.tc; cc += kConsumers) {
                const int cq = cc >> 2, w = cc & 3;
                float s = 0.0f;
                for (int j = 0; j < p.rpp; ++j) s += red[w * kConsumers + j * per_row + cq];
                const long long col = (long long)it.ct0 * p.tc + cc;
                if (col < p.cols && !failed) {
                    if (p.nsplit == 1) {
                        p.red_out[(long long)it.seg * p.red_sseg + col] = p.mean ? (float)((double)s / p.count) : s;
                    } else {
                        const int sp = it.rt0 / p.split_tiles;
                        p.partials[((long long)it.seg * p.nsplit + sp) * p.cols + col] = s;
                    }
                }
            }
            named_barrier(1, kConsumers);
        }
    }
    if (p.mode == TTC_REDUCE_ALL) {
        run_sum = warp_sum(run_sum);
        if (lane == 0) red[warp] = run_sum;
        named_barrier(1, kConsumers);
        if (t < 32) {
            float v = t < kConsumers / 32 ? red[t] : 0.0f;
            v = warp_sum(v);
            if (t == 0) p.partials[blockIdx.x] = v;
        }
    }
    if (failed && lane == 0) *(volatile int*)p.status = 1;
}

bool aligned16(const void* ptr) { return ((uintptr_t)ptr & 15) == 0; }

template <int G, int NS>
void set_smem_attr() {
    static bool done_by_dev[kMaxDevices] = {};
    const int dev = rt().device;
    if (dev < 0 || dev >= kMaxDevices) return;  // run_chain_impl's device check rejects these first
    bool& done = done_by_dev[dev];
    if (!done) {
        cudaFuncSetAttribute(chain_staged_kernel<G, NS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             1024 + kSmemBudget + 2 * kMaxStages * 8 + 8 * kConsumers * 4);
        done = true;
    }
}

}  // namespace

int launch_chain_tma(const ttc_chain_desc& d, const DProgram& prog, bool* launched) {
    *launched = false;
    if (d.cols < 64 || d.cols % 4 || d.rows < 1) return TTC_OK;
    if (d.reduce == TTC_REDUCE_ALL && d.nseg != 1) return TTC_OK;
    Params p;
    std::memset(&p, 0, sizeof p);
    int n_staged = 0;
    for (int k = 0; k < d.n_inputs; ++k) {
        const ttc_in_view& v = d.inputs[k];
        p.slot_of[k] = -1;
        if (v.col_stride == 0) continue;  // column broadcast
        if (!aligned16(v.ptr) || v.seg_stride % 4) return TTC_OK;
        if (v.row_stride == 0) continue;  // row broadcast (bias)
        if (v.row_stride % 4 || v.row_stride < d.cols) return TTC_OK;
        p.slot_of[k] = n_staged++;
    }
    if (n_staged == 0) return TTC_OK;
    for (int j = 0; j < d.n_outputs; ++j) {
        const ttc_out_view& v = d.outputs[j];
        if (!aligned16(v.ptr) || v.row_stride % 4 || v.seg_stride % 4) return TTC_OK;
    }
    // G = 8 float4 groups per thread (32 elements per program dispatch); 4
    // when the program needs more than one save slot (register budget).
    const int G = prog.n_slots <= 1 ? 8 : 4;
    p.tc = d.cols >= 256 ? 256 : d.cols >= 128 ? 128 : 64;
    p.tc_shift = p.tc == 256 ? 6 : p.tc == 128 ? 5 : 4;
    p.rpp = kConsumers / (p.tc / 4);
    p.tr = G * p.rpp;
    p.tile_bytes = p.tc * p.tr * 4;
    p.n_staged = n_staged;
    p.stages = std::min(kMaxStages, kSmemBudget / (n_staged * p.tile_bytes));
    if (p.stages < 2) return TTC_OK;
    for (int k = 0; k < d.n_inputs; ++k) {
        if (p.slot_of[k] < 0) continue;
        const ttc_in_view& v = d.inputs[k];
        const bool three = d.nseg > 1 && v.seg_stride > 0;
        p.is3d[k] = three;
        const unsigned long long dims[3] = {(unsigned long long)d.cols, (unsigned long long)d.rows,
                                            (unsigned long long)d.nseg};
        const unsigned long long strides[2] = {(unsigned long long)v.row_stride, (unsigned long long)v.seg_stride};
        const unsigned box[3] = {(unsigned)p.tc, (unsigned)p.tr, 1u};
        if (encode_tensor_map_f32(&p.maps[k], v.ptr, three ? 3 : 2, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_NONE) !=
            TTC_OK) {
            clear_error();  // a layout TMA cannot describe: the register path takes it
            return TTC_OK;
        }
    }
    p.prog = prog;
    p.rows = d.rows;
    p.cols = d.cols;
    p.nseg = d.nseg;
    p.tiles_r = (d.rows + p.tr - 1) / p.tr;
    p.tiles_c = (d.cols + p.tc - 1) / p.tc;
    p.mode = d.reduce;
    p.red_out = d.reduce_out;
    p.red_sseg = d.reduce_seg_stride;
    p.mean = d.reduce_mean;
    p.count = d.reduce == TTC_REDUCE_ROWS ? (double)d.cols
              : d.reduce == TTC_REDUCE_COLS ? (double)d.rows
                                             : (double)d.rows * d.cols;
    if (int rc = device_status_ptr(&p.status)) return rc;
    p.stall = stall_test("chain") ? 1 : 0;
    p.wait_limit = p.stall ? kStallTestLimitCycles : kWaitLimitCycles;
    const int sms = rt().sm_count;
    p.nsplit = 1;
    p.split_tiles = p.tiles_r;
    if (d.reduce == TTC_REDUCE_ROWS) {
        p.n_items = (long long)d.nseg * p.tiles_r;
    } else if (d.reduce == TTC_REDUCE_COLS) {
        const long long base = (long long)d.nseg * p.tiles_c;
        int nsplit = (int)std::min<long long>((2LL * sms + base - 1) / base, p.tiles_r);
        nsplit = std::max(nsplit, 1);
        p.split_tiles = (p.tiles_r + nsplit - 1) / nsplit;
        p.nsplit = (p.tiles_r + p.split_tiles - 1) / p.split_tiles;
        p.n_items = base * p.nsplit;
    } else {
        p.n_items = (long long)d.nseg * p.tiles_r * p.tiles_c;
    }
    const long long n_items =
        d.reduce == TTC_REDUCE_ROWS ? (long long)d.nseg * p.tiles_r
        : d.reduce == TTC_REDUCE_COLS ? (long long)d.nseg * p.tiles_c * p.nsplit
                                      : (long long)d.nseg * p.tiles_r * p.tiles_c;
    if (n_items >= (1LL << 31)) return TTC_OK;  // the register path takes it
    const int grid = (int)std::min<long long>(p.n_items, sms);
    if (d.reduce == TTC_REDUCE_ALL || (d.reduce == TTC_REDUCE_COLS && p.nsplit > 1)) {
        const size_t n = d.reduce == TTC_REDUCE_ALL ? (size_t)grid : (size_t)d.nseg * p.nsplit * d.cols;
        void* ws = nullptr;
        if (int rc = workspace(n * sizeof(float), &ws)) return rc;
        p.partials = (float*)ws;
    }
    const int smem = 1024 + p.stages * n_staged * p.tile_bytes + 2 * kMaxStages * 8 + 8 * kConsumers * 4;
    cudaStream_t st = rt().stream;
    if (G == 8) {
        set_smem_attr<8, 1>();
        chain_staged_kernel<8, 1><<<grid, kThreads, smem, st>>>(p);
    } else {
        set_smem_attr<4, 4>();
        chain_staged_kernel<4, 4><<<grid, kThreads, smem, st>>>(p);
    }
    count_launch();
    if (int rc = check_cuda(cudaGetLastError(), "staged chain kernel launch")) return rc;
    if (d.reduce == TTC_REDUCE_ALL)
        launch_finalize_all(p.partials, grid, d.reduce_out, d.reduce_mean, p.count);
    else if (d.reduce == TTC_REDUCE_COLS && p.nsplit > 1)
        launch_finalize_cols(p.partials, p.nsplit, d.cols, d.nseg, d.reduce_out, d.reduce_seg_stride, d.reduce_mean,
                             p.count);
    *launched = true;
    return check_cuda(cudaGetLastError(), "chain finalize launch");
}

}  // namespace ttc
