// The host C library's single-precision expf, log1pf, expm1f and tanhf as
// glibc 2.39 computes them, restated so a kernel reproduces the bits the
// reference's scalar code gets from the host library (the Diffusion Policy's
// spatial softmax calls expf; the scalar tail of its Mish, v * tanh(log1p(exp(v)))
// at src/hal/common/eltwise.cpp:244-248, calls all three). The same source
// compiles as device code (nvcc) and as host C (the oracle's exhaustive check
// against the host library, oracle/libm_check.c): every float operation goes
// through LF_* so nvcc cannot contract or reassociate it, and the host build
// uses -ffp-contract=off.
//
// Published methods restated:
//   expf   - glibc's table-driven expf (Szabolcs Nagy, 2017): x = (k + r)/32 ln2
//            with k rounded to an integer, 2^(k/32) from a 32-entry table of
//            doubles, a degree-3 polynomial for 2^(r/32) in double.
//   log1pf - fdlibm's s_log1pf (Sun Microsystems, 1993): 1+x = 2^k (1+f) with
//            sqrt(2)/2 < 1+f < sqrt(2), a correction term for the rounding of
//            1+x, log(1+f) = f - s(f - R(s^2)) with s = f/(2+f) and a degree-7
//            polynomial R; ln2 split in a high part with trailing zeros and a
//            low part.
//   expm1f - fdlibm's s_expm1f: x = k ln2 + r, |r| <= ln2/2, expm1(r) from a
//            rational form r + r^2/2 + r^3/2 * (3 - (r1 + r1 r/2)) / (6 - r (3 - r1 r/2))
//            with r1 a degree-5 polynomial in r^2/2, then scaled by 2^k with
//            the exponent added to the bits.
//   tanhf  - fdlibm's s_tanhf: for |x| < 1, -expm1(-2|x|)/(expm1(-2|x|)+2);
//            for 1 <= |x| < 22, 1 - 2/(expm1(2|x|)+2); 1 beyond; odd symmetry.
// The polynomial and splitting constants are those methods' published
// coefficients (needed for the same bits); the code is this library's own.
#pragma once
#include <stdint.h>

#if defined(__CUDACC__)
#define LF_FN static __device__ __forceinline__
#define LF_ADD(a, b) __fadd_rn((a), (b))
#define LF_SUB(a, b) __fsub_rn((a), (b))
#define LF_MUL(a, b) __fmul_rn((a), (b))
#define LF_DIV(a, b) __fdiv_rn((a), (b))
#define LF_DFMA(a, b, c) __fma_rn((a), (b), (c))
#define LF_DSUB(a, b) __dsub_rn((a), (b))
#define LF_DMUL(a, b) __dmul_rn((a), (b))
#define LF_D2F(d) __double2float_rn(d)
#define LF_DCONST __device__
LF_FN int32_t lf_bits(float x) { return __float_as_int(x); }
LF_FN float lf_float(int32_t i) { return __int_as_float(i); }
LF_FN uint64_t lf_dbits(double x) { return static_cast<uint64_t>(__double_as_longlong(x)); }
LF_FN double lf_double(uint64_t i) { return __longlong_as_double(static_cast<long long>(i)); }
#else
#include <math.h>
#include <string.h>
#define LF_FN static inline
#define LF_ADD(a, b) ((a) + (b))
#define LF_SUB(a, b) ((a) - (b))
#define LF_MUL(a, b) ((a) * (b))
#define LF_DIV(a, b) ((a) / (b))
#define LF_DFMA(a, b, c) fma((a), (b), (c))
#define LF_DSUB(a, b) ((a) - (b))
#define LF_DMUL(a, b) ((a) * (b))
#define LF_D2F(d) ((float)(d))
#define LF_DCONST
LF_FN int32_t lf_bits(float x) { int32_t i; memcpy(&i, &x, 4); return i; }
LF_FN float lf_float(int32_t i) { float x; memcpy(&x, &i, 4); return x; }
LF_FN uint64_t lf_dbits(double x) { uint64_t i; memcpy(&i, &x, 8); return i; }
LF_FN double lf_double(uint64_t i) { double x; memcpy(&x, &i, 8); return x; }
#endif

// 2^(i/32) for i = 0..31 with the table index's exponent bits taken out
// (bits - (i << 47)), as the table-driven expf stores them.
static LF_DCONST const uint64_t kLfExp2Tab32[32] = {
    0x3ff0000000000000ULL, 0x3fefd9b0d3158574ULL, 0x3fefb5586cf9890fULL, 0x3fef9301d0125b51ULL,
    0x3fef72b83c7d517bULL, 0x3fef54873168b9aaULL, 0x3fef387a6e756238ULL, 0x3fef1e9df51fdee1ULL,
    0x3fef06fe0a31b715ULL, 0x3feef1a7373aa9cbULL, 0x3feedea64c123422ULL, 0x3feece086061892dULL,
    0x3feebfdad5362a27ULL, 0x3feeb42b569d4f82ULL, 0x3feeab07dd485429ULL, 0x3feea47eb03a5585ULL,
    0x3feea09e667f3bcdULL, 0x3fee9f75e8ec5f74ULL, 0x3feea11473eb0187ULL, 0x3feea589994cce13ULL,
    0x3feeace5422aa0dbULL, 0x3feeb737b0cdc5e5ULL, 0x3feec49182a3f090ULL, 0x3feed503b23e255dULL,
    0x3feee89f995ad3adULL, 0x3feeff76f2fb5e47ULL, 0x3fef199bdd85529cULL, 0x3fef3720dcef9069ULL,
    0x3fef5818dcfba487ULL, 0x3fef7c97337b9b5fULL, 0x3fefa4afa2a490daULL, 0x3fefd0765b6e4540ULL};

LF_FN float lf_expf(float x) {
    if (x != x) return LF_ADD(x, x);
    if (x > 0x1.62e42ep6f) return lf_float(0x7f800000);   // overflow: +inf
    if (x < -0x1.9fe368p6f) return 0.0f;                  // underflow
    const double xd = (double)x;
    const double inv_ln2_32 = 0x1.71547652b82fep+5, shift = 0x1.8p+52;
    double kd = LF_DFMA(inv_ln2_32, xd, shift);
    const uint64_t ki = lf_dbits(kd);
    kd = LF_DSUB(kd, shift);
    const double r = LF_DFMA(inv_ln2_32, xd, -kd);
    const double s = lf_double(kLfExp2Tab32[ki & 31] + (ki << 47));
    const double z = LF_DFMA(0x1.c6af84b912394p-20, r, 0x1.ebfce50fac4f3p-13);
    const double r2 = LF_DMUL(r, r);
    double y = LF_DFMA(0x1.62e42ff0c52d6p-6, r, 1.0);
    y = LF_DFMA(z, r2, y);
    return LF_D2F(LF_DMUL(y, s));
}

// ln 2 split: the high part has its low mantissa bits clear, so k * ln2_hi is exact
#define LF_LN2_HI 6.9313812256e-01f   /* 0x3f317180 */
#define LF_LN2_LO 9.0580006145e-06f   /* 0x3717f7d1 */

LF_FN float lf_log1pf(float x) {
    const int32_t hx = lf_bits(x);
    const int32_t ax = hx & 0x7fffffff;
    int32_t k = 1, hu = 0;
    float f = 0.0f, c = 0.0f;
    if (hx < 0x3ed413d7) {                         // x < 0.41422 (sqrt(2) - 1), negatives included
        if (ax >= 0x3f800000) {                    // x <= -1
            if (x == -1.0f) return LF_DIV(-33554432.0f, 0.0f);   // -inf
            return LF_DIV(LF_SUB(x, x), LF_SUB(x, x));           // NaN
        }
        if (ax < 0x31000000) {                     // |x| < 2^-29
            if (LF_ADD(33554432.0f, x) > 0.0f && ax < 0x24800000) return x;   // |x| < 2^-54
            return LF_SUB(x, LF_MUL(LF_MUL(x, x), 0.5f));
        }
        if (hx > 0 || hx <= (int32_t)0xbe95f61f) { // -0.2929 < x < 0.41422: no reduction
            k = 0;
            f = x;
            hu = 1;
        }
    }
    if (hx >= 0x7f800000) return LF_ADD(x, x);     // +inf, NaN
    if (k != 0) {
        float u;
        if (hx < 0x5a000000) {                     // 1 + x rounds: keep a correction term
            u = LF_ADD(1.0f, x);
            hu = lf_bits(u);
            k = (hu >> 23) - 127;
            c = k > 0 ? LF_SUB(1.0f, LF_SUB(u, x)) : LF_SUB(x, LF_SUB(u, 1.0f));
            c = LF_DIV(c, u);
        } else {                                   // 1 + x == x
            u = x;
            hu = lf_bits(u);
            k = (hu >> 23) - 127;
            c = 0.0f;
        }
        hu &= 0x007fffff;
        if (hu < 0x3504f7) {                       // mantissa below sqrt(2): u in [1, sqrt(2))
            u = lf_float(hu | 0x3f800000);
        } else {                                   // else halve it: u in [sqrt(2)/2, 1)
            k += 1;
            u = lf_float(hu | 0x3f000000);
            hu = (0x00800000 - hu) >> 2;
        }
        f = LF_SUB(u, 1.0f);
    }
    const float hfsq = LF_MUL(LF_MUL(0.5f, f), f);
    const float kf = (float)k;
    if (hu == 0) {                                 // |f| < 2^-20
        if (f == 0.0f) {
            if (k == 0) return 0.0f;
            c = LF_ADD(c, LF_MUL(kf, LF_LN2_LO));
            return LF_ADD(LF_MUL(kf, LF_LN2_HI), c);
        }
        const float R = LF_MUL(hfsq, LF_SUB(1.0f, LF_MUL(0.66666666666666666f, f)));
        if (k == 0) return LF_SUB(f, R);
        return LF_SUB(LF_MUL(kf, LF_LN2_HI), LF_SUB(LF_SUB(R, LF_ADD(LF_MUL(kf, LF_LN2_LO), c)), f));
    }
    const float s = LF_DIV(f, LF_ADD(2.0f, f));
    const float z = LF_MUL(s, s);
    float R = LF_MUL(z, 1.4798198640e-01f);        // Lp7
    R = LF_MUL(z, LF_ADD(1.5313838422e-01f, R));   // Lp6
    R = LF_MUL(z, LF_ADD(1.8183572590e-01f, R));   // Lp5
    R = LF_MUL(z, LF_ADD(2.2222198546e-01f, R));   // Lp4
    R = LF_MUL(z, LF_ADD(2.8571429849e-01f, R));   // Lp3
    R = LF_MUL(z, LF_ADD(4.0000000596e-01f, R));   // Lp2
    R = LF_MUL(z, LF_ADD(6.6666668653e-01f, R));   // Lp1
    if (k == 0) return LF_SUB(f, LF_SUB(hfsq, LF_MUL(s, LF_ADD(hfsq, R))));
    return LF_SUB(LF_MUL(kf, LF_LN2_HI),
                  LF_SUB(LF_SUB(hfsq, LF_ADD(LF_MUL(s, LF_ADD(hfsq, R)), LF_ADD(LF_MUL(kf, LF_LN2_LO), c))), f));
}

LF_FN float lf_expm1f(float x) {
    int32_t hx = lf_bits(x);
    const int neg = (hx & (int32_t)0x80000000) != 0;
    hx &= 0x7fffffff;
    if (hx >= 0x4195b844) {                        // |x| >= 27 ln2
        if (hx >= 0x42b17218) {                    // |x| >= 88.72
            if (hx > 0x7f800000) return LF_ADD(x, x);          // NaN
            if (hx == 0x7f800000) return neg ? -1.0f : x;      // exp(+-inf) - 1
            if (x > 8.8721679688e+01f) return LF_MUL(1.0e+30f, 1.0e+30f);   // overflow
        }
        if (neg) return LF_SUB(1.0e-30f, 1.0f);   // -1 (inexact)
    }
    int32_t k;
    float c = 0.0f;
    if (hx > 0x3eb17218) {                         // |x| > ln2 / 2: reduce
        float hi, lo;
        if (hx < 0x3F851592) {                     // and |x| < 1.5 ln2: k = +-1
            if (!neg) { hi = LF_SUB(x, LF_LN2_HI); lo = LF_LN2_LO; k = 1; }
            else { hi = LF_ADD(x, LF_LN2_HI); lo = -LF_LN2_LO; k = -1; }
        } else {
            k = (int32_t)LF_ADD(LF_MUL(1.4426950216e+00f, x), neg ? -0.5f : 0.5f);   // truncation
            const float t = (float)k;
            hi = LF_SUB(x, LF_MUL(t, LF_LN2_HI));  // exact
            lo = LF_MUL(t, LF_LN2_LO);
        }
        x = LF_SUB(hi, lo);
        c = LF_SUB(LF_SUB(hi, x), lo);
    } else if (hx < 0x33000000) {                  // |x| < 2^-25: expm1(x) = x
        const float t = LF_ADD(1.0e+30f, x);
        return LF_SUB(x, LF_SUB(t, LF_ADD(1.0e+30f, x)));
    } else {
        k = 0;
    }
    const float hfx = LF_MUL(0.5f, x);
    const float hxs = LF_MUL(x, hfx);
    float r1 = LF_MUL(hxs, -2.0109921195e-07f);          // Q5
    r1 = LF_MUL(hxs, LF_ADD(4.0082177293e-06f, r1));      // Q4
    r1 = LF_MUL(hxs, LF_ADD(-7.9365076090e-05f, r1));     // Q3
    r1 = LF_MUL(hxs, LF_ADD(1.5873016091e-03f, r1));      // Q2
    r1 = LF_ADD(1.0f, LF_MUL(hxs, LF_ADD(-3.3333335072e-02f, r1)));   // Q1
    const float t = LF_SUB(3.0f, LF_MUL(r1, hfx));
    float e = LF_MUL(hxs, LF_DIV(LF_SUB(r1, t), LF_SUB(6.0f, LF_MUL(x, t))));
    if (k == 0) return LF_SUB(x, LF_SUB(LF_MUL(x, e), hxs));
    e = LF_SUB(LF_MUL(x, LF_SUB(e, c)), c);
    e = LF_SUB(e, hxs);
    if (k == -1) return LF_SUB(LF_MUL(0.5f, LF_SUB(x, e)), 0.5f);
    if (k == 1) {
        if (x < -0.25f) return LF_MUL(-2.0f, LF_SUB(e, LF_ADD(x, 0.5f)));
        return LF_ADD(1.0f, LF_MUL(2.0f, LF_SUB(x, e)));
    }
    if (k <= -2 || k > 56) {                       // exp(x) - 1 = 2^k (1 - (e - x)) - 1
        float y = LF_SUB(1.0f, LF_SUB(e, x));
        y = lf_float(lf_bits(y) + (k << 23));
        return LF_SUB(y, 1.0f);
    }
    float y;
    if (k < 23) {
        const float tk = lf_float(0x3f800000 - (0x1000000 >> k));   // 1 - 2^-k
        y = LF_SUB(tk, LF_SUB(e, x));
    } else {
        const float tk = lf_float((0x7f - k) << 23);                // 2^-k
        y = LF_SUB(x, LF_ADD(e, tk));
        y = LF_ADD(y, 1.0f);
    }
    return lf_float(lf_bits(y) + (k << 23));
}

LF_FN float lf_tanhf(float x) {
    const int32_t jx = lf_bits(x);
    const int32_t ix = jx & 0x7fffffff;
    if (ix >= 0x7f800000) {                        // inf, NaN
        return jx >= 0 ? LF_ADD(LF_DIV(1.0f, x), 1.0f) : LF_SUB(LF_DIV(1.0f, x), 1.0f);
    }
    float z;
    if (ix < 0x41b00000) {                         // |x| < 22
        if (ix == 0) return x;                     // +-0
        if (ix < 0x24000000) return LF_MUL(x, LF_ADD(1.0f, x));   // |x| < 2^-55
        const float ax = lf_float(ix);
        if (ix >= 0x3f800000) {                    // |x| >= 1
            const float t = lf_expm1f(LF_MUL(2.0f, ax));
            z = LF_SUB(1.0f, LF_DIV(2.0f, LF_ADD(t, 2.0f)));
        } else {
            const float t = lf_expm1f(LF_MUL(-2.0f, ax));
            z = LF_DIV(-t, LF_ADD(t, 2.0f));
        }
    } else {                                       // |x| >= 22: +-1 (inexact)
        z = LF_SUB(1.0f, 1.0e-30f);
    }
    return jx >= 0 ? z : -z;
}

// The reference's scalar Mish tail: v * tanh(softplus(v)) with softplus the
// identity above 20 (src/hal/common/eltwise.cpp:244-248).
LF_FN float lf_mish(float v) {
    const float sp = v > 20.0f ? v : lf_log1pf(lf_expf(v));
    return LF_MUL(v, lf_tanhf(sp));
}
