// expf_ref.cuh -- e^x and sigmoid for the element-wise chains and the GEMM
// epilogues, bit for bit as the reference's CPU computes them.
//
// The reference's sigmoid is 1.0f / (1.0f + std::exp(-x)) (README.md:332),
// and std::exp(float) is glibc's expf. On x86-64 hosts with AVX2 and FMA
// (every host of a B200 system) glibc selects the build of its expf compiled
// with FMA contraction (sysdeps/x86_64/fpu/multiarch/e_expf.c), a table-driven
// method published with the source (sysdeps/ieee754/flt-32/e_expf.c, the
// Arm optimized-routines design, glibc 2.27 and later):
//
//   z = x * 32/ln2 in double; k = round-to-nearest-even(z) by adding and
//   subtracting the shifter 1.5 * 2^52; r = z - k in [-1/2, 1/2];
//   s = 2^(k/32) = 2^(k >> 5) * T[k & 31], built by adding k << 47 to the bit
//   pattern of a table entry that has j << 47 subtracted already;
//   y = (C0 r + C1) r^2 + (C2 r + 1), a cubic for 2^(r/32);
//   result = (float)(y * s), one rounding from double.
//
// With FMA contraction the compiler fuses z into both of its uses
// (kd = fma(InvLn2N, x, shift), r = fma(InvLn2N, x, -kd)) and each of
// C0 r + C1, C2 r + 1 and z r2 + y into one fma; r * r and y * s stay plain
// products. The functions below perform exactly that sequence of IEEE double
// operations (every step an explicit correctly rounded intrinsic, so the
// result does not depend on -fmad), hence return glibc's float for every
// input: tests/native/expf_ref_host.cpp compiles this header for the host and
// compares it with the process's own expf on all 2^32 floats, and the GPU
// test compares the device build with the host's expf on all 2^32 floats.
// (glibc's build without FMA, chosen on CPUs without it, differs from this
// one on 2 floats.) The table holds 2^(j/32) rounded to double; the three
// coefficients are glibc's published ones.
//
// For |x| <= 87, the range the element-wise kernels' fast path takes, they
// use expf_ref_fast: the same reduction, then y = s + q (r s) with
// q = (C0 r + C1) r + C2 in Horner form -- one fp64 operation fewer than
// glibc's (C0 r + C1) r^2 + (C2 r + 1) followed by y * s. It is not glibc's
// sequence of roundings, but it returns glibc's float for every one of the
// 2.24e9 floats with |x| <= 87 (tests/native/expf_ref_host.cpp compares the
// two on all of them, and the GPU test compares the kernels' sigmoid with the
// host's on all 2^32 floats).
//
// sigmoid then adds 1 and takes the IEEE reciprocal, both single float
// roundings, so it equals the reference's float for every finite input.
// The reciprocal is Markstein's (P. Markstein, "Computation of elementary
// functions on the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1),
// 1990): y0 = hardware reciprocal approximation, one correction
// y1 = y0 + y0 (1 - d y0) with the residual exact by FMA. On the operand
// range it is used for, d in [1, 2^126), it equals the IEEE reciprocal (the
// GPU tests compare it with __frcp_rn on every float of that range).
//
// Cost per element on the fast path: one f32->f64 conversion, seven fp64
// operations, one shared-memory load (the table is 256 bytes), two integer
// operations and one f64->f32 conversion.
//
// Valid under nvcc and NVRTC (no standard headers; explicit intrinsics).
#pragma once

struct ExpTable {
    double t[32];  // bits(2^(j/32)) - (j << 47), as doubles
};

// 2^(j/32) rounded to double.
static __device__ const double kExp2Of32nds[32] = {
    0x1.0000000000000p+0, 0x1.059b0d3158574p+0, 0x1.0b5586cf9890fp+0, 0x1.11301d0125b51p+0,
    0x1.172b83c7d517bp+0, 0x1.1d4873168b9aap+0, 0x1.2387a6e756238p+0, 0x1.29e9df51fdee1p+0,
    0x1.306fe0a31b715p+0, 0x1.371a7373aa9cbp+0, 0x1.3dea64c123422p+0, 0x1.44e086061892dp+0,
    0x1.4bfdad5362a27p+0, 0x1.5342b569d4f82p+0, 0x1.5ab07dd485429p+0, 0x1.6247eb03a5585p+0,
    0x1.6a09e667f3bcdp+0, 0x1.71f75e8ec5f74p+0, 0x1.7a11473eb0187p+0, 0x1.82589994cce13p+0,
    0x1.8ace5422aa0dbp+0, 0x1.93737b0cdc5e5p+0, 0x1.9c49182a3f090p+0, 0x1.a5503b23e255dp+0,
    0x1.ae89f995ad3adp+0, 0x1.b7f76f2fb5e47p+0, 0x1.c199bdd85529cp+0, 0x1.cb720dcef9069p+0,
    0x1.d5818dcfba487p+0, 0x1.dfc97337b9b5fp+0, 0x1.ea4afa2a490dap+0, 0x1.f50765b6e4540p+0,
};

// Fills the table (the block's threads cooperate; the caller synchronises
// before the first use).
__device__ __forceinline__ void exp_table_init(ExpTable& t) {
    for (int i = threadIdx.x; i < 32; i += blockDim.x)
        t.t[i] = __longlong_as_double(__double_as_longlong(kExp2Of32nds[i]) - ((long long)i << 47));
}

// glibc's main path. Valid for x in (-103.98, 88.73), the range that path
// serves (|x| < 88 always takes it).
__device__ __forceinline__ float expf_ref_main(float x, const ExpTable& tab) {
    const double kInvLn2N = 0x1.71547652b82fep+5;  // 32 / ln2
    const double kShift = 0x1.8p52;
    const double xd = (double)x;
    const double kds = fma(kInvLn2N, xd, kShift);  // shift + round(z)
    const int k = __double2loint(kds);
    const double kd = __dsub_rn(kds, kShift);
    const double r = fma(kInvLn2N, xd, -kd);
    const double t = tab.t[k & 31];
    const double s = __hiloint2double(__double2hiint(t) + (int)((unsigned)k << 15), __double2loint(t));
    const double z = fma(0x1.c6af84b912394p-20, r, 0x1.ebfce50fac4f3p-13);
    const double r2 = __dmul_rn(r, r);
    double y = fma(0x1.62e42ff0c52d6p-6, r, 1.0);
    y = fma(z, r2, y);
    y = __dmul_rn(y, s);
    return __double2float_rn(y);
}

// |x| <= 87: the rearranged form described in the header comment.
__device__ __forceinline__ float expf_ref_fast(float x, const ExpTable& tab) {
    const double kInvLn2N = 0x1.71547652b82fep+5;  // 32 / ln2
    const double kShift = 0x1.8p52;
    const double xd = (double)x;
    const double kds = fma(kInvLn2N, xd, kShift);
    const int k = __double2loint(kds);
    const double kd = __dsub_rn(kds, kShift);
    const double r = fma(kInvLn2N, xd, -kd);
    const double t = tab.t[k & 31];
    const double s = __hiloint2double(__double2hiint(t) + (int)((unsigned)k << 15), __double2loint(t));
    const double q = fma(fma(0x1.c6af84b912394p-20, r, 0x1.ebfce50fac4f3p-13), r, 0x1.62e42ff0c52d6p-6);
    return __double2float_rn(fma(q, __dmul_rn(r, s), s));
}

// Any x, with glibc's exits for |x| >= 88 and NaN.
__device__ __forceinline__ float expf_ref(float x, const ExpTable& tab) {
    if (!(fabsf(x) < 88.0f)) {
        if (x != x) return x + x;
        if (x > 0x1.62e42ep6f) return __int_as_float(0x7f800000);  // overflows to +inf
        if (x < -0x1.9fe368p6f) return 0.0f;                       // below half the smallest subnormal
    }
    return expf_ref_main(x, tab);
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
static __device__ __noinline__ float sigmoid_ref_slow(float x, const ExpTable& t) {
    return __frcp_rn(__fadd_rn(1.0f, expf_ref(-x, t)));
}

// |x| <= 87: e^-x lies in (e^-87, e^87), so 1 + e^-x is in [1, 2^126).
__device__ __forceinline__ float sigmoid_ref_fast(float x, const ExpTable& t) {
    return rcp_rn_ge1(__fadd_rn(1.0f, expf_ref_fast(-x, t)));
}

__device__ __forceinline__ float sigmoid_ref(float x, const ExpTable& t) {
    return fabsf(x) <= 87.0f ? sigmoid_ref_fast(x, t) : sigmoid_ref_slow(x, t);
}

#if defined(__CUDACC__) || defined(__CUDACC_RTC__)
// Packed fp32 pairs (sm_100 f32x2 instructions: two IEEE round-to-nearest
// operations per instruction, the same results as two scalar ones).
__device__ __forceinline__ void f32x2_add(float& a0, float& a1, float b0, float b1) {
    asm("{\n\t.reg .b64 pa, pb;\n\tmov.b64 pa, {%0, %1};\n\tmov.b64 pb, {%2, %3};\n\t"
        "add.rn.f32x2 pa, pa, pb;\n\tmov.b64 {%0, %1}, pa;\n\t}"
        : "+f"(a0), "+f"(a1)
        : "f"(b0), "f"(b1));
}
__device__ __forceinline__ void f32x2_sub(float& a0, float& a1, float b0, float b1) {
    asm("{\n\t.reg .b64 pa, pb;\n\tmov.b64 pa, {%0, %1};\n\tmov.b64 pb, {%2, %3};\n\t"
        "sub.rn.f32x2 pa, pa, pb;\n\tmov.b64 {%0, %1}, pa;\n\t}"
        : "+f"(a0), "+f"(a1)
        : "f"(b0), "f"(b1));
}
__device__ __forceinline__ void f32x2_mul(float& a0, float& a1, float b0, float b1) {
    asm("{\n\t.reg .b64 pa, pb;\n\tmov.b64 pa, {%0, %1};\n\tmov.b64 pb, {%2, %3};\n\t"
        "mul.rn.f32x2 pa, pa, pb;\n\tmov.b64 {%0, %1}, pa;\n\t}"
        : "+f"(a0), "+f"(a1)
        : "f"(b0), "f"(b1));
}
__device__ __forceinline__ void f32x2_fma(float& d0, float& d1, float a0, float a1, float b0, float b1, float c0,
                                          float c1) {
    asm("{\n\t.reg .b64 pa, pb, pc;\n\tmov.b64 pa, {%2, %3};\n\tmov.b64 pb, {%4, %5};\n\t"
        "mov.b64 pc, {%6, %7};\n\tfma.rn.f32x2 pa, pa, pb, pc;\n\tmov.b64 {%0, %1}, pa;\n\t}"
        : "=f"(d0), "=f"(d1)
        : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}

// 1 / (1 + e) for two e >= 0 with 1 + e < 2^126, each equal to
// rcp_rn_ge1(1 + e): the add and Markstein's correction as packed pairs.
// d = 1 + e and -d = -1 - e are roundings of the same exact sum, so
// y0 + y0 (1 - d y0) comes out bit-identical to the scalar form (checked on
// every float e in [0, 2^126) on the device).
__device__ __forceinline__ void rcp_1p_x2(float e0, float e1, float& y0, float& y1) {
    float d0 = 1.0f, d1 = 1.0f, n0 = -1.0f, n1 = -1.0f;
    f32x2_add(d0, d1, e0, e1);
    f32x2_sub(n0, n1, e0, e1);
    float a0, a1;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(a0) : "f"(d0));
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(a1) : "f"(d1));
    float r0, r1;
    f32x2_fma(r0, r1, n0, n1, a0, a1, 1.0f, 1.0f);
    f32x2_fma(y0, y1, a0, a1, r0, r1, a0, a1);
}

__device__ __forceinline__ void sigmoid_ref_fast2(float& x0, float& x1, const ExpTable& t) {
    rcp_1p_x2(expf_ref_fast(-x0, t), expf_ref_fast(-x1, t), x0, x1);
}
#endif

// N values at once: one range test for all of them (the slow path is for
// |x| > 87 only, which ordinary data never reaches).
template <int N>
__device__ __forceinline__ void sigmoid_ref_n(float* v, const ExpTable& t) {
    bool fast = true;
#pragma unroll
    for (int i = 0; i < N; ++i) fast = fast && fabsf(v[i]) <= 87.0f;  // false for NaN too
    if (fast) {
#if defined(__CUDA_ARCH__) || defined(__CUDACC_RTC__)
#pragma unroll
        for (int i = 0; i + 1 < N; i += 2) sigmoid_ref_fast2(v[i], v[i + 1], t);
        if (N & 1) v[N - 1] = sigmoid_ref_fast(v[N - 1], t);
#else
#pragma unroll
        for (int i = 0; i < N; ++i) v[i] = sigmoid_ref_fast(v[i], t);
#endif
    } else {
#pragma unroll
        for (int i = 0; i < N; ++i) v[i] = sigmoid_ref(v[i], t);
    }
}
