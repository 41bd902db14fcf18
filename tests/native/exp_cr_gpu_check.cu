// On-device checks of tt_lazy_b200/csrc/exp_cr.cuh:
//  1. rcp_rn_ge1(d) == __frcp_rn(d) for every float d in [1, 2^126);
//  2. exp_cr(x) against CUDA's double exp rounded to float, every float with
//     |x| <= 104 (they differ only where the exact value is within ~2^-44 of
//     a rounding midpoint);
//  3. sigmoid_cr_n (one range test per vector, packed pairs) == sigmoid_cr per
//     element on a sweep that includes NaN, +-inf and the slow-path range;
//  4. the packed pair reciprocal rcp_1p_x2(e) == __frcp_rn(1 + e) for every
//     float e in [0, 2^126).
// Prints "rcp_mismatch=<n> exp_mismatch=<n> exp_over1ulp=<n> vec_mismatch=<n>
// rcp2_mismatch=<n>".
// Every loop index stays below its bound; the kernels take no input buffers.
#include <cstdio>
#include <cuda_runtime.h>

#include "exp_cr.cuh"

__global__ void check(unsigned long long* out, unsigned top) {
    __shared__ ExpCrTable t;
    exp_cr_table_init(t);
    __syncthreads();
    unsigned long long rcp_bad = 0, exp_bad = 0, exp_far = 0, vec_bad = 0;
    const unsigned stride = gridDim.x * blockDim.x;
    const unsigned rcp_total = 126u << 23;  // d = 2^e (1 + m 2^-23), e in [0, 126)
    for (unsigned u = blockIdx.x * blockDim.x + threadIdx.x; u < rcp_total; u += stride) {
        const float d = __int_as_float((int)(0x3F800000u + u));
        rcp_bad += __float_as_int(rcp_rn_ge1(d)) != __float_as_int(__frcp_rn(d));
    }
    for (unsigned u = blockIdx.x * blockDim.x + threadIdx.x; u <= top; u += stride) {
        for (int s = 0; s < 2; ++s) {
            const float x = __int_as_float((int)(u | (s ? 0x80000000u : 0u)));
            const int got = __float_as_int(exp_cr(x, t));
            const int want = __float_as_int(__double2float_rn(exp((double)x)));
            if (got != want) {
                ++exp_bad;
                if (got - want > 1 || want - got > 1) ++exp_far;
            }
        }
        if ((u & 1023u) == 0) {  // vector form vs scalar form, 8 lanes incl. specials
            float v[8] = {__int_as_float((int)u),         -__int_as_float((int)u), 0.5f, -3.0f,
                          __int_as_float(0x7fc00000),     __int_as_float(0x7f800000),
                          -__int_as_float(0x7f800000),    (u & 2048u) ? 88.5f : -88.5f};
            float w[8];
            for (int i = 0; i < 8; ++i) w[i] = sigmoid_cr(v[i], t);
            sigmoid_cr_n<8>(v, t);
            for (int i = 0; i < 8; ++i) vec_bad += __float_as_int(v[i]) != __float_as_int(w[i]);
        }
    }
    atomicAdd(&out[0], rcp_bad);
    atomicAdd(&out[1], exp_bad);
    atomicAdd(&out[2], exp_far);
    atomicAdd(&out[3], vec_bad);
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
    atomicAdd(&out[4], bad);
}

int main() {
    unsigned long long* d = nullptr;
    if (cudaMalloc(&d, 5 * sizeof(unsigned long long)) != cudaSuccess) return 2;
    cudaMemset(d, 0, 5 * sizeof(unsigned long long));
    const float f104 = 104.0f;
    unsigned top;
    memcpy(&top, &f104, 4);
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
    check<<<sms * 8, 256>>>(d, top);
    check_rcp2<<<sms * 8, 256>>>(d);
    unsigned long long h[5] = {0, 0, 0, 0, 0};
    const cudaError_t e = cudaMemcpy(h, d, sizeof h, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) {
        printf("cuda error %s\n", cudaGetErrorString(e));
        return 1;
    }
    printf("rcp_mismatch=%llu exp_mismatch=%llu exp_over1ulp=%llu vec_mismatch=%llu rcp2_mismatch=%llu\n", h[0], h[1],
           h[2], h[3], h[4]);
    return 0;
}
