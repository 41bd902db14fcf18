// On-device checks of tt_lazy_b200/csrc/expf_ref.cuh:
//  1. rcp_rn_ge1(d) == __frcp_rn(d) for every float d in [1, 2^126);
//  2. the packed pair reciprocal rcp_1p_x2(e) == __frcp_rn(1 + e) for every
//     float e in [0, 2^126);
//  3. expf_ref(x) on the device == this host's expf(x), and the vector
//     sigmoid sigmoid_ref_n<8> (one range test for 8 values, packed pairs,
//     the form the kernels use) == 1.0f / (1.0f + expf(-x)) on the host, for
//     all 2^32 bit patterns (NaN compares equal to NaN), in chunks of 2^26.
// Prints "rcp_mismatch=<n> rcp2_mismatch=<n> exp_mismatch=<n> sig_mismatch=<n>
// sig_over1ulp=<n> fma_variant=<0|1>"; fma_variant says whether the host's
// expf is glibc's FMA build (the one the header restates).
// Every kernel index stays below its bound: the chunk kernel's thread t
// writes elements 8t .. 8t+7 of arrays of kChunk floats, and the grid has
// kChunk / 8 threads.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <cuda_runtime.h>

#include "expf_ref.cuh"

static const unsigned kChunk = 1u << 26;

__global__ void check_rcp(unsigned long long* out) {
    unsigned long long bad = 0;
    const unsigned stride = gridDim.x * blockDim.x;
    const unsigned total = 126u << 23;  // d = 2^e (1 + m 2^-23), e in [0, 126)
    for (unsigned u = blockIdx.x * blockDim.x + threadIdx.x; u < total; u += stride) {
        const float d = __int_as_float((int)(0x3F800000u + u));
        bad += __float_as_int(rcp_rn_ge1(d)) != __float_as_int(__frcp_rn(d));
    }
    atomicAdd(&out[0], bad);
}

__global__ void check_rcp2(unsigned long long* out) {
    unsigned long long bad = 0;
    const unsigned total = 0x7E800000u;  // bit patterns of [0, 2^126)
    for (unsigned u = 2 * (blockIdx.x * blockDim.x + threadIdx.x); u + 1 < total; u += 2 * gridDim.x * blockDim.x) {
        const float e0 = __int_as_float((int)u), e1 = __int_as_float((int)(u + 1));
        float y0, y1;
        rcp_1p_x2(e0, e1, y0, y1);
        bad += __float_as_int(y0) != __float_as_int(__frcp_rn(__fadd_rn(1.0f, e0)));
        bad += __float_as_int(y1) != __float_as_int(__frcp_rn(__fadd_rn(1.0f, e1)));
    }
    atomicAdd(&out[1], bad);
}

__global__ void chunk_kernel(unsigned base, float* exp_out, float* sig_out) {
    __shared__ ExpTable t;
    exp_table_init(t);
    __syncthreads();
    const unsigned i = 8u * (blockIdx.x * blockDim.x + threadIdx.x);
    if (i >= kChunk) return;
    float v[8];
    for (int k = 0; k < 8; ++k) {
        const float x = __int_as_float((int)(base + i + k));
        v[k] = x;
        exp_out[i + k] = expf_ref(x, t);
    }
    sigmoid_ref_n<8>(v, t);
    for (int k = 0; k < 8; ++k) sig_out[i + k] = v[k];
}

static int bits(float f) {
    int i;
    memcpy(&i, &f, 4);
    return i;
}
static bool same(float a, float b) { return bits(a) == bits(b) || (a != a && b != b); }

int main() {
    unsigned long long* d = nullptr;
    float *dexp = nullptr, *dsig = nullptr, *hexp = nullptr, *hsig = nullptr;
    if (cudaMalloc(&d, 2 * sizeof(unsigned long long)) != cudaSuccess) return 2;
    if (cudaMalloc(&dexp, kChunk * sizeof(float)) != cudaSuccess) return 2;
    if (cudaMalloc(&dsig, kChunk * sizeof(float)) != cudaSuccess) return 2;
    if (cudaMallocHost(&hexp, kChunk * sizeof(float)) != cudaSuccess) return 2;
    if (cudaMallocHost(&hsig, kChunk * sizeof(float)) != cudaSuccess) return 2;
    cudaMemset(d, 0, 2 * sizeof(unsigned long long));
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
    check_rcp<<<sms * 8, 256>>>(d);
    check_rcp2<<<sms * 8, 256>>>(d);
    unsigned long long h[2] = {0, 0};
    cudaError_t e = cudaMemcpy(h, d, sizeof h, cudaMemcpyDeviceToHost);
    long long exp_bad = 0, sig_bad = 0, sig_far = 0;
    for (unsigned long long base = 0; e == cudaSuccess && base < (1ull << 32); base += kChunk) {
        chunk_kernel<<<kChunk / 8 / 256, 256>>>((unsigned)base, dexp, dsig);
        e = cudaMemcpy(hexp, dexp, kChunk * sizeof(float), cudaMemcpyDeviceToHost);
        if (e == cudaSuccess) e = cudaMemcpy(hsig, dsig, kChunk * sizeof(float), cudaMemcpyDeviceToHost);
        if (e != cudaSuccess) break;
#pragma omp parallel for reduction(+ : exp_bad, sig_bad, sig_far) schedule(static)
        for (long long i = 0; i < (long long)kChunk; ++i) {
            const unsigned u = (unsigned)(base + i);
            float x;
            memcpy(&x, &u, 4);
            exp_bad += !same(hexp[i], ::expf(x));
            const float want = 1.0f / (1.0f + ::expf(-x));
            if (!same(hsig[i], want)) {
                ++sig_bad;
                const long long dd = (long long)bits(hsig[i]) - bits(want);
                if (dd > 1 || dd < -1) ++sig_far;
            }
        }
    }
    if (e != cudaSuccess) {
        printf("cuda error %s\n", cudaGetErrorString(e));
        return 1;
    }
    volatile float probe = 0x1.04845ep+5f;  // volatile: no compile-time folding of expf
    const int fma_variant = bits(::expf(probe)) == bits(0x1.f93e38p+46f);
    printf("rcp_mismatch=%llu rcp2_mismatch=%llu exp_mismatch=%lld sig_mismatch=%lld sig_over1ulp=%lld "
           "fma_variant=%d\n",
           h[0], h[1], exp_bad, sig_bad, sig_far, fma_variant);
    return 0;
}
