// transpose.cu -- math::transpose (src/backend/cpu/transpose.cpp:7-36):
// out[b][j][i] = in[b][i][j] for a contiguous [batch, rows, cols] tensor.
//
// The reference writes result[j * rows + i] one scalar at a time (a strided
// store per element, 0.69 GB/s). Here a 256-thread block moves a 64x64 tile:
// 128-bit coalesced loads of 64 input rows into shared memory, then 128-bit
// coalesced stores of 64 output rows read down the tile's columns. The tile
// row pitch is 65 floats, so a column read touches each bank at most twice.
// HBM-bound: 8 bytes of traffic per element.
#include "ttc_internal.cuh"

namespace ttc {
namespace {

constexpr int T = 64;
constexpr int kThreads = 256;

template <bool VEC>
__global__ void __launch_bounds__(kThreads) transpose_kernel(const float* __restrict__ in, float* __restrict__ out,
                                                              long long rows, long long cols) {
    __shared__ float tile[T][T + 1];
    const long long b = blockIdx.z;
    const long long r0 = (long long)blockIdx.y * T, c0 = (long long)blockIdx.x * T;
    const float* src = in + b * rows * cols;
    float* dst = out + b * rows * cols;
    // load: 64 rows x 16 float4
#pragma unroll
    for (int i = 0; i < (T * T / 4) / kThreads; ++i) {
        const int e = threadIdx.x + i * kThreads;
        const int lr = e >> 4, lc = (e & 15) * 4;
        const long long r = r0 + lr, c = c0 + lc;
        float v[4] = {0.f, 0.f, 0.f, 0.f};
        if (r < rows) {
            if (VEC && c + 3 < cols) {
                const float4 q = __ldg(reinterpret_cast<const float4*>(src + r * cols + c));
                v[0] = q.x;
                v[1] = q.y;
                v[2] = q.z;
                v[3] = q.w;
            } else {
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    if (c + k < cols) v[k] = __ldg(src + r * cols + c + k);
            }
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) tile[lr][lc + k] = v[k];
    }
    __syncthreads();
    // store: output rows are input columns
#pragma unroll
    for (int i = 0; i < (T * T / 4) / kThreads; ++i) {
        const int e = threadIdx.x + i * kThreads;
        const int oc = e >> 4, orr = (e & 15) * 4;  // output row = input col c0+oc
        const long long j = c0 + oc, ii = r0 + orr;
        if (j >= cols) continue;
        float v[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) v[k] = tile[orr + k][oc];
        if (VEC && ii + 3 < rows) {
            *reinterpret_cast<float4*>(dst + j * rows + ii) = make_float4(v[0], v[1], v[2], v[3]);
        } else {
#pragma unroll
            for (int k = 0; k < 4; ++k)
                if (ii + k < rows) dst[j * rows + ii + k] = v[k];
        }
    }
}

}  // namespace
}  // namespace ttc

using namespace ttc;

extern "C" int ttc_transpose(const float* in, float* out, int64_t batch, int64_t rows, int64_t cols) {
    TTC_REQUIRE_INIT();
    if (!in || !out || batch < 0 || rows < 0 || cols < 0)
        return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: transpose arguments invalid");
    if (batch == 0 || rows == 0 || cols == 0) return TTC_OK;
    if (in == out) return set_error(TTC_ERR_INVALID_ARGUMENT, "tt_cuda: transpose cannot run in place");
    const long long gx = (cols + T - 1) / T, gy = (rows + T - 1) / T;
    if (gy > 65535 || batch > 65535 || gx > INT32_MAX)
        return set_error(TTC_ERR_UNSUPPORTED, "tt_cuda: transpose grid %lld x %lld x %lld too large", gx, gy,
                         (long long)batch);
    const bool vec = (cols % 4 == 0) && (rows % 4 == 0) && (((uintptr_t)in | (uintptr_t)out) & 15) == 0;
    dim3 grid((unsigned)gx, (unsigned)gy, (unsigned)batch);
    if (vec)
        transpose_kernel<true><<<grid, kThreads, 0, rt().stream>>>(in, out, rows, cols);
    else
        transpose_kernel<false><<<grid, kThreads, 0, rt().stream>>>(in, out, rows, cols);
    count_launch();
    return check_cuda(cudaGetLastError(), "transpose kernel launch");
}
