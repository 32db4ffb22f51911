// expf and tanhf with the results of the host C library the reference runs
// on (GNU libc 2.28 and later on x86-64), for host and device code, so that
// the decoder's softmax, GELU and soft-cap round exactly as the reference's
// f32::exp and f32::tanh do (Rust calls the platform libm). A device's own
// expf/tanhf differ from glibc's in the last bit now and then, and on the
// synthetic E2B model one such bit, through the Q8_0 quantization of the
// next projection's input, is enough to change later greedy tokens.
//
// expf: the method of ARM's optimized-routines (Szabolcs Nagy), which glibc
// uses for expf: k = round(x * 32/ln2), exp(x) = 2^(k/32) * 2^(r/32) with a
// 32-entry table of 2^(i/32) (exponent bits folded out; computed here from
// exact arithmetic) and a cubic in r, all in double, rounded once to float.
// glibc selects a build of it with fused multiply-adds on CPUs that have
// them; the evaluation below follows that build (fma in the polynomial).
// The method and its reduction and polynomial constants come from:
//   Arm Optimized Routines, math/expf.c
//   Copyright (c) 2017-2018, Arm Limited.
//   SPDX-License-Identifier: MIT OR Apache-2.0 WITH LLVM-exception
// under whose MIT terms: "The above copyright notice and this permission
// notice shall be included in all copies or substantial portions of the
// Software." (Permission is hereby granted, free of charge, to any person
// obtaining a copy of this software and associated documentation files, to
// deal in the Software without restriction, including without limitation the
// rights to use, copy, modify, merge, publish, distribute, sublicense, and/or
// sell copies of the Software. THE SOFTWARE IS PROVIDED "AS IS", WITHOUT
// WARRANTY OF ANY KIND, EXPRESS OR IMPLIED.)
//
// tanhf: the single-precision port of Sun's fdlibm tanh/expm1, which glibc
// uses for tanhf:
//   Copyright (C) 1993 by Sun Microsystems, Inc. All rights reserved.
//   Developed at SunPro, a Sun Microsystems, Inc. business.
//   Permission to use, copy, modify, and distribute this
//   software is freely granted, provided that this notice
//   is preserved.
// Every float operation is a separately rounded IEEE operation (no fused
// multiply-add), as in the x86-64 build.
#pragma once

#include <cstdint>
#include <cstring>

#ifndef __CUDACC__
#define __host__
#define __device__
#define __forceinline__ inline
#include <cmath>
#endif

namespace g4a {
namespace glibc {

#ifdef __CUDA_ARCH__
__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }
__device__ __forceinline__ float fsub(float a, float b) { return __fsub_rn(a, b); }
__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fdiv(float a, float b) { return __fdiv_rn(a, b); }
__device__ __forceinline__ double dadd(double a, double b) { return __dadd_rn(a, b); }
__device__ __forceinline__ double dsub(double a, double b) { return __dsub_rn(a, b); }
__device__ __forceinline__ double dmul(double a, double b) { return __dmul_rn(a, b); }
__device__ __forceinline__ double dfma(double a, double b, double c) { return __fma_rn(a, b, c); }
__device__ __forceinline__ uint32_t f2u(float x) { return __float_as_uint(x); }
__device__ __forceinline__ float u2f(uint32_t x) { return __uint_as_float(x); }
__device__ __forceinline__ uint64_t d2u(double x) { return (uint64_t)__double_as_longlong(x); }
__device__ __forceinline__ double u2d(uint64_t x) { return __longlong_as_double((long long)x); }
#else
inline float fadd(float a, float b) { volatile float r = a + b; return r; }
inline float fsub(float a, float b) { volatile float r = a - b; return r; }
inline float fmul(float a, float b) { volatile float r = a * b; return r; }
inline float fdiv(float a, float b) { volatile float r = a / b; return r; }
inline double dadd(double a, double b) { volatile double r = a + b; return r; }
inline double dsub(double a, double b) { volatile double r = a - b; return r; }
inline double dmul(double a, double b) { volatile double r = a * b; return r; }
inline double dfma(double a, double b, double c) { return std::fma(a, b, c); }
inline uint32_t f2u(float x) { uint32_t u; std::memcpy(&u, &x, 4); return u; }
inline float u2f(uint32_t u) { float x; std::memcpy(&x, &u, 4); return x; }
inline uint64_t d2u(double x) { uint64_t u; std::memcpy(&u, &x, 8); return u; }
inline double u2d(uint64_t u) { double x; std::memcpy(&x, &u, 8); return x; }
#endif

// asuint64(2^(i/32)) - (i << 47): 2^(i/32) rounded to double, its exponent
// contribution removed so that k can be added back as an integer. A table at
// file scope (device code reads it through the read-only cache): as a local
// array indexed at run time it would be rebuilt in local memory on every call.
#define G4A_EXP2_32_TABLE \
        0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull, \
        0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull, \
        0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull, \
        0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull, \
        0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull, \
        0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull, \
        0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull, \
        0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull
#ifdef __CUDACC__
static __device__ const unsigned long long kExp2TabDev[32] = {G4A_EXP2_32_TABLE};
#endif
static const uint64_t kExp2TabHost[32] = {G4A_EXP2_32_TABLE};
#undef G4A_EXP2_32_TABLE

__host__ __device__ __forceinline__ uint64_t exp2_32_entry(int i) {
#ifdef __CUDA_ARCH__
    return (uint64_t)__ldg(&kExp2TabDev[i]);
#else
    return kExp2TabHost[i];
#endif
}

__host__ __device__ __forceinline__ float expf(float x) {
    const uint32_t ux = f2u(x);
    const uint32_t abstop = (ux >> 20) & 0x7ff;
    if (abstop >= 0x42b) {                          // |x| >= 88 or x is NaN
        if (ux == 0xff800000u) return 0.0f;         // -inf
        if (abstop >= 0x7f8) return fadd(x, x);     // +inf, NaN
        if (x > 0x1.62e42ep6f) return u2f(0x7f800000u);   // overflow
        if (x < -0x1.9fe368p6f) return 0.0f;               // underflow
    }
    const double N = 32.0;
    const double inv_ln2_n = 0x1.71547652b82fep+0 * N;
    const double shift = 0x1.8p+52;
    const double c0 = 0x1.c6af84b912394p-5 / N / N / N, c1 = 0x1.ebfce50fac4f3p-3 / N / N,
                 c2 = 0x1.62e42ff0c52d6p-1 / N;
    const double xd = (double)x;
    const double kd0 = dfma(inv_ln2_n, xd, shift);  // round(x * 32 / ln2) by the shift
    const uint64_t ki = d2u(kd0);
    const double kd = dsub(kd0, shift);
    const double r = dfma(inv_ln2_n, xd, -kd);
    uint64_t t = exp2_32_entry((int)(ki % 32));
    t += ki << 47;
    const double s = u2d(t);
    const double z = dfma(c0, r, c1);
    const double r2 = dmul(r, r);
    double y = dfma(c2, r, 1.0);
    y = dfma(z, r2, y);
    y = dmul(y, s);
    return (float)y;
}

// fdlibm expm1f (float port)
__host__ __device__ __forceinline__ float expm1f(float x) {
    const float huge = 1.0e+30f, tiny = 1.0e-30f, one = 1.0f;
    const float o_threshold = 8.8721679688e+01f, ln2_hi = 6.9313812256e-01f, ln2_lo = 9.0580006145e-06f,
                invln2 = 1.4426950216e+00f;
    const float Q1 = -3.3333335072e-02f, Q2 = 1.5873016091e-03f, Q3 = -7.9365076090e-05f, Q4 = 4.0082177293e-06f,
                Q5 = -2.0109921195e-07f;
    float y, hi, lo, c = 0.0f, t, e, hxs, hfx, r1;
    int32_t k;
    uint32_t hx = f2u(x);
    const uint32_t xsb = hx & 0x80000000u;
    y = xsb == 0 ? x : -x;
    hx &= 0x7fffffffu;
    if (hx >= 0x4195b844u) {        // |x| >= 27 ln2
        if (hx >= 0x42b17218u) {    // |x| >= 88.72
            if (hx > 0x7f800000u) return fadd(x, x);
            if (hx == 0x7f800000u) return xsb == 0 ? x : -1.0f;
            if (x > o_threshold) return fmul(huge, huge);
        }
        if (xsb != 0) return fsub(tiny, one);
    }
    if (hx > 0x3eb17218u) {         // |x| > 0.5 ln2
        if (hx < 0x3F851592u) {     // and |x| < 1.5 ln2
            if (xsb == 0) {
                hi = fsub(x, ln2_hi);
                lo = ln2_lo;
                k = 1;
            } else {
                hi = fadd(x, ln2_hi);
                lo = -ln2_lo;
                k = -1;
            }
        } else {
            k = (int32_t)fadd(fmul(invln2, x), xsb == 0 ? 0.5f : -0.5f);
            t = (float)k;
            hi = fsub(x, fmul(t, ln2_hi));
            lo = fmul(t, ln2_lo);
        }
        x = fsub(hi, lo);
        c = fsub(fsub(hi, x), lo);
    } else if (hx < 0x33000000u) {  // |x| < 2^-25
        t = fadd(huge, x);
        return fsub(x, fsub(t, fadd(huge, x)));
    } else {
        k = 0;
    }
    hfx = fmul(0.5f, x);
    hxs = fmul(x, hfx);
    r1 = fadd(one, fmul(hxs, fadd(Q1, fmul(hxs, fadd(Q2, fmul(hxs, fadd(Q3, fmul(hxs, fadd(Q4, fmul(hxs, Q5))))))))));
    t = fsub(3.0f, fmul(r1, hfx));
    e = fmul(hxs, fdiv(fsub(r1, t), fsub(6.0f, fmul(x, t))));
    if (k == 0) return fsub(x, fsub(fmul(x, e), hxs));
    e = fsub(fmul(x, fsub(e, c)), c);
    e = fsub(e, hxs);
    if (k == -1) return fsub(fmul(0.5f, fsub(x, e)), 0.5f);
    if (k == 1) {
        if (x < -0.25f) return fmul(-2.0f, fsub(e, fadd(x, 0.5f)));
        return fadd(one, fmul(2.0f, fsub(x, e)));
    }
    if (k <= -2 || k > 56) {
        y = fsub(one, fsub(e, x));
        if (k == 128) {
            y = fmul(fmul(y, 2.0f), 0x1p127f);
        } else {
            y = u2f(f2u(y) + ((uint32_t)k << 23));
        }
        return fsub(y, one);
    }
    if (k < 23) {
        t = u2f(0x3f800000u - (0x1000000u >> k));  // 1 - 2^-k
        y = fsub(t, fsub(e, x));
        y = u2f(f2u(y) + ((uint32_t)k << 23));
    } else {
        t = u2f((uint32_t)(0x7f - k) << 23);  // 2^-k
        y = fsub(x, fadd(e, t));
        y = fadd(y, one);
        y = u2f(f2u(y) + ((uint32_t)k << 23));
    }
    return y;
}

// fdlibm tanhf (float port)
__host__ __device__ __forceinline__ float tanhf(float x) {
    const float one = 1.0f, two = 2.0f, tiny = 1.0e-30f;
    const uint32_t jx = f2u(x), ix = jx & 0x7fffffffu;
    float z;
    if (ix >= 0x7f800000u) {  // inf or NaN
        if ((int32_t)jx >= 0) return fadd(fdiv(one, x), one);
        return fsub(fdiv(one, x), one);
    }
    if (ix < 0x41b00000u) {   // |x| < 22
        if (ix == 0) return x;
        if (ix < 0x24000000u) return fmul(x, fadd(one, x));  // |x| < 2^-55
        const float ax = u2f(ix);
        if (ix >= 0x3f800000u) {  // |x| >= 1
            const float t = expm1f(fmul(two, ax));
            z = fsub(one, fdiv(two, fadd(t, two)));
        } else {
            const float t = expm1f(fmul(-two, ax));
            z = fdiv(-t, fadd(t, two));
        }
    } else {
        z = fsub(one, tiny);
    }
    return (int32_t)jx >= 0 ? z : -z;
}

}  // namespace glibc
}  // namespace g4a
