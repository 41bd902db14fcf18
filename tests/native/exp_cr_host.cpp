// Host build of tt_lazy_b200/csrc/exp_cr.cuh (the device exp of the sigmoid
// step) with each CUDA intrinsic mapped to the IEEE operation it names, so
// table method can be checked against a long-double exp over a large sweep
// of floats on the CPU. Compile with -ffp-contract=off: every
// intrinsic below is one correctly rounded operation, as on the device.
//
// usage: exp_cr_host STRIDE  -> prints "n=<count> mismatches=<m> over1ulp=<k>"
// over every STRIDE-th float bit pattern with |x| <= 104 (both signs).
#include <cmath>
#include <math.h>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#define __device__
#define __forceinline__ inline
#define __noinline__
struct Dim {
    unsigned x;
};
static Dim threadIdx{0}, blockDim{1};
static inline float __fmaf_rn(float a, float b, float c) { return std::fma(a, b, c); }
static inline float __fadd_rn(float a, float b) { return a + b; }
static inline float __fsub_rn(float a, float b) { return a - b; }
static inline float __fmul_rn(float a, float b) { return a * b; }
static inline float __frcp_rn(float a) { return 1.0f / a; }
static inline int __float_as_int(float f) {
    int i;
    std::memcpy(&i, &f, 4);
    return i;
}
static inline float __int_as_float(int i) {
    float f;
    std::memcpy(&f, &i, 4);
    return f;
}
static inline long long __double_as_longlong(double d) {
    long long i;
    std::memcpy(&i, &d, 8);
    return i;
}
static inline double __longlong_as_double(long long i) {
    double d;
    std::memcpy(&d, &i, 8);
    return d;
}
static inline float __double2float_rn(double d) { return (float)d; }
static inline int __double2loint(double d) {
    unsigned long long u;
    std::memcpy(&u, &d, 8);
    return (int)(unsigned)u;
}
// fma rounded toward -inf, in the one form the header uses: S + floor(a * b)
// for a shifter S = 1.5 * 2^52 (the sum's ulp is 1), with the product exact.
static inline double __fma_rd(double a, double b, double S) {
    const double p = a * b;
    const double e = std::fma(a, b, -p);  // a * b = p + e exactly
    double f = std::floor(p);
    if (f == p && e < 0) f -= 1.0;
    return S + f;
}
static inline int __float2int_rn(float f) { return (int)std::lrintf(f); }
using std::exp2;

using std::fma;

#include "exp_cr.cuh"

int main(int argc, char** argv) {
    const long long stride = argc > 1 ? std::atoll(argv[1]) : 1;
    ExpCrTable tab;
    exp_cr_table_init(tab);  // one "thread" of a one-thread block fills every entry
    const long long top = __float_as_int(104.0f);
    long long n = 0, bad = 0, over1 = 0;
#pragma omp parallel for reduction(+ : n, bad, over1) schedule(dynamic, 4096)
    for (long long u = 0; u <= top; u += stride) {
        for (int s = 0; s < 2; ++s) {
            const float x = __int_as_float((int)u | (s ? (int)0x80000000u : 0));
            const float want = (float)::expl((long double)x);
            const float got = exp_cr(x, tab);
            ++n;
            if (__float_as_int(got) != __float_as_int(want)) {
                ++bad;
                const long long d = (long long)__float_as_int(got) - __float_as_int(want);
                if (d > 1 || d < -1) ++over1;
            }
        }
    }
    std::printf("n=%lld mismatches=%lld over1ulp=%lld\n", n, bad, over1);
    return 0;
}
