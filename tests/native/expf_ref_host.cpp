// Host build of tt_lazy_b200/csrc/expf_ref.cuh (the device exp of the
// sigmoid step) with each CUDA intrinsic mapped to the IEEE operation it
// names, compared with this process's own expf (glibc, the function the
// reference's std::exp(float) calls) and with the reference's sigmoid
// formula 1.0f / (1.0f + expf(-x)). Compile with -ffp-contract=off: every
// intrinsic below is one correctly rounded operation, as on the device.
//
// usage: expf_ref_host STRIDE -> prints
//   "n=<count> exp_mismatch=<m> fast_mismatch=<f> sig_mismatch=<s> sig_over1ulp=<k> fma_variant=<0|1>"
// over every STRIDE-th 32-bit pattern (NaN results compare equal to NaN);
// fast_mismatch counts the inputs with |x| <= 87 where expf_ref_fast (the
// kernels' rearranged form) differs from expf.
// fma_variant reports whether this libm's expf is glibc's FMA build (the one
// the header restates) at the input where its two x86-64 builds differ.
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
static inline float __frcp_rn(float a) { return 1.0f / a; }
static inline double __dsub_rn(double a, double b) { return a - b; }
static inline double __dmul_rn(double a, double b) { return a * b; }
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
static inline int __double2loint(double d) { return (int)(unsigned)(unsigned long long)__double_as_longlong(d); }
static inline int __double2hiint(double d) { return (int)(unsigned)((unsigned long long)__double_as_longlong(d) >> 32); }
static inline double __hiloint2double(int hi, int lo) {
    return __longlong_as_double((long long)(((unsigned long long)(unsigned)hi << 32) | (unsigned)lo));
}
using std::fma;

#include "expf_ref.cuh"

static bool same(float a, float b) { return __float_as_int(a) == __float_as_int(b) || (a != a && b != b); }

int main(int argc, char** argv) {
    const long long stride = argc > 1 ? std::atoll(argv[1]) : 1;
    ExpTable tab;
    exp_table_init(tab);  // one "thread" of a one-thread block fills every entry
    long long n = 0, exp_bad = 0, fast_bad = 0, sig_bad = 0, sig_far = 0;
#pragma omp parallel for reduction(+ : n, exp_bad, fast_bad, sig_bad, sig_far) schedule(dynamic, 1 << 16)
    for (long long u = 0; u < (1ll << 32); u += stride) {
        const float x = __int_as_float((int)(unsigned)u);
        ++n;
        const float ex = ::expf(x);
        exp_bad += !same(expf_ref(x, tab), ex);
        if (fabsf(x) <= 87.0f) fast_bad += !same(expf_ref_fast(x, tab), ex);
        const float want = 1.0f / (1.0f + ::expf(-x));
        const float got = sigmoid_ref(x, tab);
        if (!same(got, want)) {
            ++sig_bad;
            const long long d = (long long)__float_as_int(got) - __float_as_int(want);
            if (d > 1 || d < -1) ++sig_far;
        }
    }
    volatile float probe = 0x1.04845ep+5f;  // volatile: no compile-time folding of expf
    const int fma_variant = __float_as_int(::expf(probe)) == __float_as_int(0x1.f93e38p+46f);
    std::printf("n=%lld exp_mismatch=%lld fast_mismatch=%lld sig_mismatch=%lld sig_over1ulp=%lld fma_variant=%d\n", n,
                exp_bad, fast_bad, sig_bad, sig_far, fma_variant);
    return 0;
}
