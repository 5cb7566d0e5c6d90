// glibc_expf.cuh -- binary32 exp() that returns the same bits as the C
// runtime expf the reference calls.
//
// The reference computes every router softmax / sigmoid and every SiLU with
// MathF.Exp (src/QuantRunner.Core/Runtime/StreamingEngine.cs:645,
// Glm5Ops.cs:19, TransformerOps.cs:112).  .NET 8 implements MathF.Exp by
// calling the C runtime's expf; on Linux x86-64 that is glibc's expf, which
// since glibc 2.27 is the table-driven algorithm published by Szabolcs Nagy in
// ARM's optimized-routines (e_expf.c / e_exp2f_data.c): with N = 32,
//   k = round(x * N/ln2),  r = x * N/ln2 - k,
//   exp(x) = 2^(k/N) * (1 + C2 r + C1 r^2 + C0 r^3),
// evaluated in binary64 and rounded once to binary32.  On CPUs with FMA glibc
// selects the build compiled with FMA contraction, so the range reduction
// (z*InvLn2N + SHIFT and z*InvLn2N - kd) and the three polynomial steps are
// fused multiply-adds.  This restatement, with the table entries
// T[i] = bits(2^(i/N)) - (i << 47) and the published polynomial, reproduces
// glibc 2.39's expf bit for bit on all 2^32 binary32 inputs (checked
// exhaustively by tests/test_expf_restatement.py on the CPU).
//
// Usable from host code (tests) and device code; device code must be compiled
// without --use_fast_math and with denormals preserved.
#pragma once
#include <stdint.h>

#if defined(__CUDACC__)
#define QRM_HD __host__ __device__ __forceinline__
#else
#define QRM_HD inline
#include <math.h>
#include <string.h>
#endif

namespace qrm {

// T[i] = bits(2^(i/32)) - (i << 47), i = 0..31
#define QRM_EXPF_TABLE \
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull, \
    0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull, \
    0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull, \
    0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull, \
    0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull, \
    0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull, \
    0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull, \
    0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull
#if defined(__CUDACC__)
__device__ __constant__ static const uint64_t kExpfTabDev[32] = {QRM_EXPF_TABLE};
#endif
static const uint64_t kExpfTabHost[32] = {QRM_EXPF_TABLE};

QRM_HD uint32_t f32_bits(float f) {
#if defined(__CUDA_ARCH__)
    return __float_as_uint(f);
#else
    uint32_t u; memcpy(&u, &f, 4); return u;
#endif
}
QRM_HD float f32_from(uint32_t u) {
#if defined(__CUDA_ARCH__)
    return __uint_as_float(u);
#else
    float f; memcpy(&f, &u, 4); return f;
#endif
}
QRM_HD uint64_t f64_bits(double d) {
#if defined(__CUDA_ARCH__)
    return (uint64_t)__double_as_longlong(d);
#else
    uint64_t u; memcpy(&u, &d, 8); return u;
#endif
}
QRM_HD double f64_from(uint64_t u) {
#if defined(__CUDA_ARCH__)
    return __longlong_as_double((long long)u);
#else
    double d; memcpy(&d, &u, 8); return d;
#endif
}
QRM_HD double fma64(double a, double b, double c) {
#if defined(__CUDA_ARCH__)
    return __fma_rn(a, b, c);
#else
    return fma(a, b, c);
#endif
}
QRM_HD double mul64(double a, double b) {
#if defined(__CUDA_ARCH__)
    return __dmul_rn(a, b);
#else
    return a * b;
#endif
}
QRM_HD double add64(double a, double b) {
#if defined(__CUDA_ARCH__)
    return __dadd_rn(a, b);
#else
    return a + b;
#endif
}
QRM_HD float to_f32(double y) {
#if defined(__CUDA_ARCH__)
    return __double2float_rn(y);
#else
    return (float)y;
#endif
}

// glibc-identical expf with the table T[] at tab (device code may pass a
// shared-memory copy: lanes index it divergently).
QRM_HD float expf_glibc_t(float x, const uint64_t* tab) {
    const double kInvLn2N = 0x1.71547652b82fep+0 * 32;
    const double kShift = 0x1.8p+52;
    const double kC0 = 0x1.c6af84b912394p-5 / 32 / 32 / 32;
    const double kC1 = 0x1.ebfce50fac4f3p-3 / 32 / 32;
    const double kC2 = 0x1.62e42ff0c52d6p-1 / 32;
    uint32_t ux = f32_bits(x);
    uint32_t abstop = (ux >> 20) & 0x7ff;
    if (abstop >= 0x42b) {                 // |x| >= 88 or NaN
        if (ux == 0xff800000u) return 0.0f;                 // -inf
        if (abstop >= 0x7f8) return x + x;                  // inf or NaN
        if (x > 0x1.62e42ep6f) return f32_from(0x7f800000u); // overflow
        if (x < -0x1.9fe368p6f) return 0.0f;                // underflow
    }
    double xd = (double)x;
    double kd = fma64(kInvLn2N, xd, kShift);
    uint64_t ki = f64_bits(kd);
    kd = add64(kd, -kShift);
    double r = fma64(kInvLn2N, xd, -kd);
    uint64_t t = tab[ki % 32];
    t += ki << (52 - 5);
    double s = f64_from(t);
    double z = fma64(kC0, r, kC1);
    double r2 = mul64(r, r);
    double y = fma64(kC2, r, 1.0);
    y = fma64(z, r2, y);
    y = mul64(y, s);
    return to_f32(y);
}

// glibc-identical expf.
QRM_HD float expf_glibc(float x) {
#if defined(__CUDA_ARCH__)
    return expf_glibc_t(x, kExpfTabDev);
#else
    return expf_glibc_t(x, kExpfTabHost);
#endif
}

}  // namespace qrm
