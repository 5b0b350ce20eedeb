/* tanhf with the exact rounding of the C library the reference runs on.
 *
 * The reference's scalar CPU tier evaluates the GELU-tanh gate with tanhf
 * (vendor/embeddinggemma.c/src/kernels.c:367-371), from glibc 2.39, whose
 * single-precision tanh and expm1 are the classic Sun fdlibm algorithms
 * (s_tanhf.c / s_expm1f.c): tanh(x) = sign(x) (1 - 2/(expm1(2|x|) + 2)) for
 * 1 <= |x| < 22, -expm1(-2|x|)/(expm1(-2|x|) + 2) below 1, x(1 + x) below
 * 2^-55, +-1 above; expm1 by argument reduction with ln2 split in hi/lo and a
 * degree-5 rational correction in x^2/2, with a result reconstruction that
 * depends on the reduction step k.  Neither is correctly rounded (about 5 % of
 * tanhf results differ from the correctly rounded value), so the GPU has to
 * evaluate these exact steps.  The library's build has no fused multiply-add
 * here; the EG2_F* macros give IEEE operations that are never contracted, on
 * the host and on the device.  Checked against glibc on every finite float.
 *
 * Notice of the restated algorithms (fdlibm, as carried by glibc):
 * Copyright (C) 1993 by Sun Microsystems, Inc. All rights reserved.
 * Developed at SunPro, a Sun Microsystems, Inc. business.  Permission to use,
 * copy, modify, and distribute this software is freely granted, provided that
 * this notice is preserved.  (The float versions were converted by Ian Lance
 * Taylor, Cygnus Support.)  The code here is this project's own restatement.
 */
#ifndef EG2_REF_TANHF_H
#define EG2_REF_TANHF_H
#include <stdint.h>
#include <string.h>

#ifdef __CUDACC__
#define EG2_TANHF_QUAL __host__ __device__ __forceinline__
#else
#define EG2_TANHF_QUAL static inline
#endif
#if defined(__CUDA_ARCH__)
#define EG2_FADD(a, b) __fadd_rn((a), (b))
#define EG2_FSUB(a, b) __fsub_rn((a), (b))
#define EG2_FMUL(a, b) __fmul_rn((a), (b))
#define EG2_FDIV(a, b) __fdiv_rn((a), (b))
#else
#define EG2_FADD(a, b) ((a) + (b))
#define EG2_FSUB(a, b) ((a) - (b))
#define EG2_FMUL(a, b) ((a) * (b))
#define EG2_FDIV(a, b) ((a) / (b))
#endif

EG2_TANHF_QUAL uint32_t eg2_fbits(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
}
EG2_TANHF_QUAL float eg2_bitsf(uint32_t u) {
    float f;
    memcpy(&f, &u, 4);
    return f;
}

EG2_TANHF_QUAL float eg2_ref_expm1f(float x) {
    const float one = 1.0f, huge = 1.0e+30f, tiny = 1.0e-30f, o_threshold = 8.8721679688e+01f,
                ln2_hi = 6.9313812256e-01f, ln2_lo = 9.0580006145e-06f, invln2 = 1.4426950216e+00f,
                Q1 = -3.3333335072e-02f, Q2 = 1.5873016091e-03f, Q3 = -7.9365076090e-05f, Q4 = 4.0082177293e-06f,
                Q5 = -2.0109921195e-07f;
    float y, hi, lo, c = 0.0f, t, e, hxs, hfx, r1;
    int32_t k;
    uint32_t hx = eg2_fbits(x);
    const uint32_t xsb = hx & 0x80000000u;
    hx &= 0x7fffffffu;
    if (hx >= 0x4195b844u) { /* |x| >= 27 ln2 */
        if (hx >= 0x42b17218u) {
            if (hx > 0x7f800000u) return EG2_FADD(x, x);
            if (hx == 0x7f800000u) return xsb == 0 ? x : -1.0f;
            if (x > o_threshold) return EG2_FMUL(huge, huge);
        }
        if (xsb != 0) return EG2_FSUB(tiny, one);
    }
    if (hx > 0x3eb17218u) { /* |x| > ln2 / 2 */
        if (hx < 0x3F851592u) {
            if (xsb == 0) {
                hi = EG2_FSUB(x, ln2_hi), lo = ln2_lo, k = 1;
            } else {
                hi = EG2_FADD(x, ln2_hi), lo = -ln2_lo, k = -1;
            }
        } else {
            k = (int32_t)EG2_FADD(EG2_FMUL(invln2, x), xsb == 0 ? 0.5f : -0.5f);
            t = (float)k;
            hi = EG2_FSUB(x, EG2_FMUL(t, ln2_hi));
            lo = EG2_FMUL(t, ln2_lo);
        }
        x = EG2_FSUB(hi, lo);
        c = EG2_FSUB(EG2_FSUB(hi, x), lo);
    } else if (hx < 0x33000000u) { /* |x| < 2^-25 */
        t = EG2_FADD(huge, x);
        return EG2_FSUB(x, EG2_FSUB(t, EG2_FADD(huge, x)));
    } else {
        k = 0;
    }
    hfx = EG2_FMUL(0.5f, x);
    hxs = EG2_FMUL(x, hfx);
    r1 = EG2_FADD(one, EG2_FMUL(hxs, EG2_FADD(Q1, EG2_FMUL(hxs, EG2_FADD(Q2, EG2_FMUL(hxs, EG2_FADD(Q3, EG2_FMUL(hxs, EG2_FADD(Q4, EG2_FMUL(hxs, Q5))))))))));
    t = EG2_FSUB(3.0f, EG2_FMUL(r1, hfx));
    e = EG2_FMUL(hxs, EG2_FDIV(EG2_FSUB(r1, t), EG2_FSUB(6.0f, EG2_FMUL(x, t))));
    if (k == 0) return EG2_FSUB(x, EG2_FSUB(EG2_FMUL(x, e), hxs));
    e = EG2_FSUB(EG2_FMUL(x, EG2_FSUB(e, c)), c);
    e = EG2_FSUB(e, hxs);
    if (k == -1) return EG2_FSUB(EG2_FMUL(0.5f, EG2_FSUB(x, e)), 0.5f);
    if (k == 1) {
        if (x < -0.25f) return EG2_FMUL(-2.0f, EG2_FSUB(e, EG2_FADD(x, 0.5f)));
        return EG2_FADD(one, EG2_FMUL(2.0f, EG2_FSUB(x, e)));
    }
    if (k <= -2 || k > 56) {
        y = EG2_FSUB(one, EG2_FSUB(e, x));
        y = eg2_bitsf(eg2_fbits(y) + ((uint32_t)k << 23));
        return EG2_FSUB(y, one);
    }
    if (k < 23) {
        t = eg2_bitsf(0x3f800000u - (0x1000000u >> k)); /* 1 - 2^-k */
        y = EG2_FSUB(t, EG2_FSUB(e, x));
        y = eg2_bitsf(eg2_fbits(y) + ((uint32_t)k << 23));
    } else {
        t = eg2_bitsf((uint32_t)(0x7f - k) << 23); /* 2^-k */
        y = EG2_FSUB(x, EG2_FADD(e, t));
        y = EG2_FADD(y, one);
        y = eg2_bitsf(eg2_fbits(y) + ((uint32_t)k << 23));
    }
    return y;
}

EG2_TANHF_QUAL float eg2_ref_tanhf(float x) {
    const float one = 1.0f, two = 2.0f, tiny = 1.0e-30f;
    float t, z;
    const uint32_t jx = eg2_fbits(x), ix = jx & 0x7fffffffu;
    if (ix >= 0x7f800000u) return (jx >> 31) ? EG2_FSUB(EG2_FDIV(one, x), one) : EG2_FADD(EG2_FDIV(one, x), one);
    if (ix < 0x41b00000u) { /* |x| < 22 */
        if (ix == 0) return x;
        if (ix < 0x24000000u) return EG2_FMUL(x, EG2_FADD(one, x)); /* |x| < 2^-55 */
        const float ax = eg2_bitsf(ix);
        if (ix >= 0x3f800000u) { /* |x| >= 1 */
            t = eg2_ref_expm1f(EG2_FMUL(two, ax));
            z = EG2_FSUB(one, EG2_FDIV(two, EG2_FADD(t, two)));
        } else {
            t = eg2_ref_expm1f(EG2_FMUL(-two, ax));
            z = EG2_FDIV(-t, EG2_FADD(t, two));
        }
    } else {
        z = EG2_FSUB(one, tiny);
    }
    return (jx >> 31) ? -z : z;
}

#endif
