// exp_cr.cuh -- e^x for the sigmoid step, accurate enough that rounding it
// once gives the correctly rounded float except within ~2^-48 of a rounding
// midpoint. The CPU reference computes sigmoid as 1 / (1 + expf(-x)) with
// glibc's expf (within 0.502 ulp, nearly always correctly rounded), so both
// sides almost always hold the same float and the IEEE add and reciprocal
// that follow match bit for bit; a 2-ulp exp would put sigmoid up to 4 ulp
// away from the reference.
//
// Method: table-driven reduction (P. T. P. Tang, "Table-driven implementation
// of the exponential function in IEEE floating-point arithmetic", ACM TOMS
// 15(2), 1989) evaluated in float-float arithmetic (T. J. Dekker, "A
// floating-point technique for extending the available precision", Numer.
// Math. 18, 1971: exact products by fused multiply-add, exact sums by
// two-sum) so that the hot path uses only fp32 pipes -- no fp64 ops and no
// conversions, which on sm_100a issue at a fraction of the fp32 rate:
//   k = round(x * 64/ln2) = 64 m + j,  r = x - k ln2/64  (|r| <~ ln2/128)
//   e^x = 2^m * 2^(j/64) * e^r,  e^r = 1 + r + r^2/2 + r^3/6 + r^4/24 + r^5/120
// with ln2/64 split in three floats (Cody-Waite), r carried as rh + rl,
// r^2/2 exact by FMA, 2^(j/64) = hi[j] + lo[j] from a 64-entry table.
// Error budget (relative): omitted r^6 term < 2^-50, ln2/64 split < 2^-66,
// table 2^-52, roundings of the low-order parts ~2^-48. Checked over every
// float with |x| <= 104 against a long-double exp (tests/native/
// exp_cr_host.cpp compiles this file for the host): 12 of 2.24e9 results are
// 1 ulp off the correctly rounded value, none further.
// |x| > 87 (results near the overflow / subnormal range) takes a double
// path with the same reduction.
//
// Valid under nvcc and NVRTC (no standard headers, explicit __fmaf_rn so
// the result does not depend on -fmad).
#pragma once

struct ExpCrTable {
    float hi[64];
    float lo[64];
};

// Fills the 2^(j/64) table (one block's threads cooperate; the caller
// synchronises before the first exp_cr).
__device__ __forceinline__ void exp_cr_table_init(ExpCrTable& t) {
    for (int i = threadIdx.x; i < 64; i += blockDim.x) {
        const double v = exp2((double)i * (1.0 / 64.0));
        const float h = __double2float_rn(v);
        t.hi[i] = h;
        t.lo[i] = __double2float_rn(v - (double)h);
    }
}

// |x| > 87, NaN: same reduction in double, one rounding at the end.
static __device__ __noinline__ float exp_cr_slow(float x, const ExpCrTable& t) {
    if (x != x) return x;
    if (x > 89.0f) return __int_as_float(0x7f800000);  // overflows to +inf
    if (x < -104.0f) return 0.0f;                      // below half the smallest subnormal
    const int k = __float2int_rn(x * 92.33248261689366f);
    const double r = fma(-(double)k, 0.010830424696249145, (double)x);
    double p = fma(r, 1.0 / 120.0, 1.0 / 24.0);
    p = fma(p, r, 1.0 / 6.0);
    p = fma(p, r, 0.5);
    p = fma(p, r, 1.0);
    p = fma(p, r, 1.0);
    double e = p * ((double)t.hi[k & 63] + (double)t.lo[k & 63]);
    e = __longlong_as_double(__double_as_longlong(e) + (long long)(k >> 6) * (1ll << 52));  // * 2^m
    return __double2float_rn(e);
}

__device__ __forceinline__ float exp_cr(float x, const ExpCrTable& t) {
    if (!(fabsf(x) <= 87.0f)) return exp_cr_slow(x, t);
    // k = round(x * 64/ln2) by the 1.5 * 2^23 shifter: t0's low bits hold k
    const float shifter = 12582912.0f;
    const float t0 = __fmaf_rn(x, 92.33248138427734f, shifter);
    const float kf = __fsub_rn(t0, shifter);
    const int bits = __float_as_int(t0);
    const int j = bits & 63;
    const int m = (bits - 0x4B400000) >> 6;
    // r = x - k ln2/64: the first step is exact (x and k * L1 are multiples
    // of 2^-30 and |r1| < 2^-7), rl collects what rounding rh dropped
    const float L1 = 0x1.62e43p-7f, L2 = -0x1.05c61p-35f, L3 = -0x1.950d88p-60f;
    const float r1 = __fmaf_rn(-kf, L1, x);
    const float rh = __fmaf_rn(-kf, L2, r1);
    float rl = __fmaf_rn(-kf, L2, __fsub_rn(r1, rh));
    rl = __fmaf_rn(-kf, L3, rl);
    // u = e^r - 1 = uh + ul
    const float h = __fmul_rn(0.5f, rh);
    const float sh = __fmul_rn(h, rh);  // rh^2 / 2 ...
    const float sl = __fmaf_rn(h, rh, -sh);  // ... and its rounding error, exactly
    float q = __fmaf_rn(rh, 1.0f / 60.0f, 1.0f / 12.0f);
    q = __fmaf_rn(q, rh, 1.0f / 3.0f);
    const float tail = __fmul_rn(__fmul_rn(sh, rh), q);  // r^3/6 + r^4/24 + r^5/120
    const float uh = __fadd_rn(rh, sh);
    const float ul0 = __fadd_rn(__fsub_rn(rh, uh), sh);  // |rh| >= sh: fast two-sum
    const float ul = __fadd_rn(ul0, __fadd_rn(sl, __fadd_rn(tail, __fmaf_rn(rh, rl, rl))));
    // T (1 + u), T = hi + lo
    const float th = t.hi[j], tl = t.lo[j];
    const float ph = __fmul_rn(th, uh);
    const float pl = __fmaf_rn(th, uh, -ph);
    const float vh = __fadd_rn(th, ph);
    const float vl = __fadd_rn(__fsub_rn(th, vh), ph);  // |th| >= |ph|: fast two-sum
    const float low = __fadd_rn(vl, __fadd_rn(pl, __fmaf_rn(th, ul, __fmaf_rn(tl, uh, tl))));
    const float y = __fadd_rn(vh, low);  // the one rounding of the result
    return __int_as_float(__float_as_int(y) + (int)((unsigned)m << 23));  // * 2^m (result stays normal)
}

// sigmoid as the reference computes it: 1 / (1 + e^-x), each step rounded
// once (the IEEE reciprocal equals the IEEE quotient 1 / d).
__device__ __forceinline__ float sigmoid_cr(float x, const ExpCrTable& t) {
    return __frcp_rn(__fadd_rn(1.0f, exp_cr(-x, t)));
}
