/* expf with the exact rounding of the C library the reference runs on.
 *
 * The reference's scalar attention calls expf (vendor/embeddinggemma.c/src/
 * gemma2_fast.c scalar branch of attention_rows) from glibc >= 2.27, whose
 * single-precision exp is the published ARM optimized-routines algorithm
 * (Szabolcs Nagy): x * 32/ln2 split into an integer k and a remainder r,
 * 2^(k/32) from a 32-entry table of 2^(i/32) with the integer part folded into
 * the exponent, and a degree-3 polynomial for 2^(r/32), all in double, then
 * one rounding to float.  It is not correctly rounded (about 1 in 2000
 * arguments in [-8, 0] differ by one ulp from the correctly rounded value), so
 * an exact-order attention has to evaluate this algorithm, not any other exp.
 * glibc dispatches an FMA build on x86-64 CPUs with FMA; the multiply-adds
 * below are therefore fused.  Checked against glibc's expf on every float in
 * (-inf, 0] (tests/test_cpu_oracle.py samples that check; the arguments here
 * are always <= 0: scores minus their maximum).
 *
 * The table holds bits(2^(i/32) rounded to double) - (i << 47).
 *
 * Licence of the restated algorithm and its table: ARM optimized-routines,
 * Copyright (c) 2017-2018, Arm Limited, distributed under the MIT licence
 * (SPDX-License-Identifier: MIT OR Apache-2.0 WITH LLVM-exception), which
 * permits use, copying, modification and distribution provided this notice is
 * kept; the code here is this project's own restatement.
 */
#ifndef EG2_REF_EXPF_H
#define EG2_REF_EXPF_H
#include <stdint.h>
#include <string.h>
#include <math.h>

#define EG2_EXP2_TAB                                                                                    \
    0x3ff0000000000000ull, 0x3fefd9b0d3158574ull, 0x3fefb5586cf9890full, 0x3fef9301d0125b51ull,        \
        0x3fef72b83c7d517bull, 0x3fef54873168b9aaull, 0x3fef387a6e756238ull, 0x3fef1e9df51fdee1ull,    \
        0x3fef06fe0a31b715ull, 0x3feef1a7373aa9cbull, 0x3feedea64c123422ull, 0x3feece086061892dull,    \
        0x3feebfdad5362a27ull, 0x3feeb42b569d4f82ull, 0x3feeab07dd485429ull, 0x3feea47eb03a5585ull,    \
        0x3feea09e667f3bcdull, 0x3fee9f75e8ec5f74ull, 0x3feea11473eb0187ull, 0x3feea589994cce13ull,    \
        0x3feeace5422aa0dbull, 0x3feeb737b0cdc5e5ull, 0x3feec49182a3f090ull, 0x3feed503b23e255dull,    \
        0x3feee89f995ad3adull, 0x3feeff76f2fb5e47ull, 0x3fef199bdd85529cull, 0x3fef3720dcef9069ull,    \
        0x3fef5818dcfba487ull, 0x3fef7c97337b9b5full, 0x3fefa4afa2a490daull, 0x3fefd0765b6e4540ull

#define EG2_EXPF_SHIFT 0x1.8p+52
#define EG2_EXPF_INVLN2N (0x1.71547652b82fep+0 * 32)
#define EG2_EXPF_C0 (0x1.c6af84b912394p-5 / 32 / 32 / 32)
#define EG2_EXPF_C1 (0x1.ebfce50fac4f3p-3 / 32 / 32)
#define EG2_EXPF_C2 (0x1.62e42ff0c52d6p-1 / 32)

#ifdef __CUDACC__
#define EG2_EXPF_QUAL __host__ __device__ __forceinline__
#else
#define EG2_EXPF_QUAL static inline
#endif

/* For x <= 0 (and any x below the overflow threshold).  tab: EG2_EXP2_TAB. */
EG2_EXPF_QUAL float eg2_ref_expf(float x, const uint64_t *tab) {
    if (x < -0x1.9fe368p6f) return 0.0f; /* underflows to +0 */
    const double xd = (double)x;
    double kd = fma(EG2_EXPF_INVLN2N, xd, EG2_EXPF_SHIFT);
    uint64_t ki;
    memcpy(&ki, &kd, 8);
    kd -= EG2_EXPF_SHIFT;
    const double r = fma(EG2_EXPF_INVLN2N, xd, -kd);
    const uint64_t t = tab[ki % 32] + (ki << 47);
    double s;
    memcpy(&s, &t, 8);
    const double p = fma(EG2_EXPF_C0, r, EG2_EXPF_C1);
    const double r2 = r * r;
    double y = fma(EG2_EXPF_C2, r, 1.0);
    y = fma(p, r2, y);
    return (float)(y * s);
}

#endif
