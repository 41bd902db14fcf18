// exp_cr.cuh -- e^x and sigmoid for the element-wise chains and the GEMM
// epilogues, accurate enough that rounding once gives the correctly rounded
// float except within ~2^-44 of a rounding midpoint. The CPU reference
// computes sigmoid as 1 / (1 + expf(-x)) with glibc's expf (within 0.502
// ulp, nearly always correctly rounded), so both sides almost always hold
// the same float and the IEEE add and reciprocal that follow match bit for
// bit; a 2-ulp exp would put sigmoid up to 4 ulp away from the reference.
//
// Method: table-driven reduction (P. T. P. Tang, "Table-driven implementation
// of the exponential function in IEEE floating-point arithmetic", ACM TOMS
// 15(2), 1989):
//   k = round(x * 64/ln2) = 64 m + j,  r = x - k ln2/64  (|r| <~ ln2/128)
//   e^x = 2^m * 2^(j/64) * e^r,  e^r = 1 + r + r^2/2 + r^3/6 + r^4/24 + r^5/120
// k comes from the fp32 shifter trick (no float-to-int conversion), r and the
// polynomial are evaluated in double (relative error < 2^-47 on |r| <= ln2/128,
// table 2^-52), the product is rounded to float once and scaled by 2^m with
// an integer add to the exponent field. On sm_100a the fp64 pipe runs beside
// the fp32 pipe, so this issues fewer instructions than a float-float
// evaluation of the same formula. Checked over every float with |x| <= 104
// against a long-double exp (tests/native/exp_cr_host.cpp compiles this file
// for the host): 2 of 2.24e9 results are 1 ulp off the correctly rounded
// value, none further.
//
// The reciprocal of sigmoid is Markstein's (P. Markstein, "Computation of
// elementary functions on the IBM RISC System/6000 processor", IBM J. Res.
// Dev. 34(1), 1990): y0 = hardware reciprocal approximation, one correction
// y1 = y0 + y0 (1 - d y0) with the residual exact by FMA. On the operand
// range it is used for, d in [1, 2^126), it equals the IEEE reciprocal (the
// GPU tests compare it with __frcp_rn on every float of that range).
//
// Valid under nvcc and NVRTC (no standard headers; explicit __fmaf_rn / fma
// so the result does not depend on -fmad).
#pragma once

struct ExpCrTable {
    double t[64];  // 2^(j/64)
};

// Fills the table (the block's threads cooperate; the caller synchronises
// before the first use).
__device__ __forceinline__ void exp_cr_table_init(ExpCrTable& t) {
    for (int i = threadIdx.x; i < 64; i += blockDim.x) t.t[i] = exp2((double)i * (1.0 / 64.0));
}

// |x| <= 87: the result is a normal float (e^-87 > 2^-126, e^87 < 2^126).
__device__ __forceinline__ float exp_cr_fast(float x, const ExpCrTable& t) {
    const float shifter = 12582912.0f;  // 1.5 * 2^23: t0's low bits hold k
    const float t0 = __fmaf_rn(x, 92.33248138427734f, shifter);
    const float kf = __fsub_rn(t0, shifter);
    const int bits = __float_as_int(t0);
    const int scale = (bits << 17) & (int)0xFF800000;  // (k >> 6) << 23, i.e. m in the exponent field
    const double r = fma(-(double)kf, 0.010830424696249145, (double)x);
    double p = fma(r, 1.0 / 120.0, 1.0 / 24.0);
    p = fma(p, r, 1.0 / 6.0);
    p = fma(p, r, 0.5);
    p = fma(p, r, 1.0);
    p = fma(p, r, 1.0);
    const float y = __double2float_rn(p * t.t[bits & 63]);
    return __int_as_float(__float_as_int(y) + scale);
}

// Any x: NaN, overflow to +inf, results in the subnormal range rounded once
// from the double value.
static __device__ __noinline__ float exp_cr_slow(float x, const ExpCrTable& t) {
    if (x != x) return x;
    if (x > 89.0f) return __int_as_float(0x7f800000);  // overflows to +inf
    if (x < -104.0f) return 0.0f;                      // below half the smallest subnormal
    const float shifter = 12582912.0f;
    const float kf = __fsub_rn(__fmaf_rn(x, 92.33248138427734f, shifter), shifter);
    const int k = (int)kf;
    const double r = fma(-(double)kf, 0.010830424696249145, (double)x);
    double p = fma(r, 1.0 / 120.0, 1.0 / 24.0);
    p = fma(p, r, 1.0 / 6.0);
    p = fma(p, r, 0.5);
    p = fma(p, r, 1.0);
    p = fma(p, r, 1.0);
    double e = p * t.t[k & 63];
    e = __longlong_as_double(__double_as_longlong(e) + (long long)(k >> 6) * (1ll << 52));  // * 2^m
    return __double2float_rn(e);
}

__device__ __forceinline__ float exp_cr(float x, const ExpCrTable& t) {
    return fabsf(x) <= 87.0f ? exp_cr_fast(x, t) : exp_cr_slow(x, t);
}

// IEEE round-to-nearest 1/d for d in [1, 2^126) (see the header comment).
__device__ __forceinline__ float rcp_rn_ge1(float d) {
#if defined(__CUDA_ARCH__) || defined(__CUDACC_RTC__)
    float y0;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y0) : "f"(d));
    const float e = __fmaf_rn(-d, y0, 1.0f);
    return __fmaf_rn(y0, e, y0);
#else
    return 1.0f / d;  // host compilation of this header (the exp sweep test) only
#endif
}

// sigmoid as the reference computes it: 1 / (1 + e^-x), each step rounded
// once (the IEEE reciprocal equals the IEEE quotient 1 / d).
static __device__ __noinline__ float sigmoid_cr_slow(float x, const ExpCrTable& t) {
    return __frcp_rn(__fadd_rn(1.0f, exp_cr_slow(-x, t)));
}

__device__ __forceinline__ float sigmoid_cr_fast(float x, const ExpCrTable& t) {
    return rcp_rn_ge1(__fadd_rn(1.0f, exp_cr_fast(-x, t)));
}

__device__ __forceinline__ float sigmoid_cr(float x, const ExpCrTable& t) {
    return fabsf(x) <= 87.0f ? sigmoid_cr_fast(x, t) : sigmoid_cr_slow(x, t);
}

// N values at once: one range test for all of them (the slow path is for
// |x| > 87 only, which ordinary data never reaches).
template <int N>
__device__ __forceinline__ void sigmoid_cr_n(float* v, const ExpCrTable& t) {
    bool fast = true;
#pragma unroll
    for (int i = 0; i < N; ++i) fast = fast && fabsf(v[i]) <= 87.0f;  // false for NaN too
    if (fast) {
#pragma unroll
        for (int i = 0; i < N; ++i) v[i] = sigmoid_cr_fast(v[i], t);
    } else {
#pragma unroll
        for (int i = 0; i < N; ++i) v[i] = sigmoid_cr(v[i], t);
    }
}
