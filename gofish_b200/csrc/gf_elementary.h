// Elementary functions shared, bit for bit, by the sm_100a kernels and the CPU
// oracle.
//
// The tile binning (atan2 of the fisheye projection, log of the opacity power)
// and the per-pixel hit test (exp of the Gaussian response) decide integer
// outputs: sort keys, tile counts and per-pixel hit counts.  Those must be
// identical between the GPU and the CPU restatement, so neither side may use
// its platform's expf/logf/atan2f (CUDA's and glibc's differ in the last ulp).
// Both sides call the functions below, written only with IEEE-754 single
// precision +, -, *, /, correctly rounded fused multiply-add and integer bit
// operations, which give the same bits on an x86-64 host (-ffp-contract=off)
// and on the GPU (-fmad=false, -prec-div=true, -prec-sqrt=true, no -ftz).
//
// Methods (all from the mathematics, constants derived in the comments):
//   gf_expf   : Cody & Waite argument reduction x = k ln2 + r, |r| <= ln2/2,
//               exp(r) by its Taylor series to degree 8, scaled by 2^k.
//               (W. J. Cody, W. Waite, "Software Manual for the Elementary
//               Functions", 1980.)
//   gf_logf   : x = m 2^e, m in [sqrt(1/2), sqrt(2)), log m = 2 atanh(s),
//               s = (m-1)/(m+1), atanh by its Taylor series to s^15.
//   gf_atan2f : octant reduction to t in [0,1], then t > tan(pi/8) is mapped
//               by atan t = pi/4 + atan((t-1)/(t+1)); atan by its Taylor
//               series to u^19 on |u| <= tan(pi/8).
// Measured error against IEEE double references is <= 2 ulp for exp and
// log and <= 2.5 ulp for atan2 (see
// tests/test_elementary.py).
#pragma once

#include <stdint.h>
#include <string.h>

#if defined(__CUDACC__)
#define GF_HD __host__ __device__ __forceinline__
#else
#include <math.h>
#define GF_HD static inline
#endif

namespace gf {

GF_HD uint32_t f2u(float f) {
#if defined(__CUDA_ARCH__)
    return __float_as_uint(f);
#else
    uint32_t u;
    memcpy(&u, &f, 4);
    return u;
#endif
}

GF_HD float u2f(uint32_t u) {
#if defined(__CUDA_ARCH__)
    return __uint_as_float(u);
#else
    float f;
    memcpy(&f, &u, 4);
    return f;
#endif
}

// Correctly rounded fused multiply-add on both sides.
GF_HD float fmaf_rn(float a, float b, float c) {
#if defined(__CUDA_ARCH__)
    return __fmaf_rn(a, b, c);
#else
    return fmaf(a, b, c);
#endif
}

GF_HD bool isnan_f(float x) { return x != x; }
GF_HD bool isfinite_f(float x) { return (f2u(x) & 0x7f800000u) != 0x7f800000u; }
GF_HD float abs_f(float x) { return u2f(f2u(x) & 0x7fffffffu); }
GF_HD float copysign_f(float mag, float sgn) {
    return u2f((f2u(mag) & 0x7fffffffu) | (f2u(sgn) & 0x80000000u));
}
GF_HD float inf_f() { return u2f(0x7f800000u); }
GF_HD float nan_f() { return u2f(0x7fc00000u); }
// IEEE minNum / maxNum with the operand order of CUDA's fminf/fmaxf (a NaN
// operand yields the other operand).
GF_HD float min_f(float a, float b) {
    if (isnan_f(a)) return b;
    if (isnan_f(b)) return a;
    return a < b ? a : b;
}
GF_HD float max_f(float a, float b) {
    if (isnan_f(a)) return b;
    if (isnan_f(b)) return a;
    return a > b ? a : b;
}
// Round half to even, for |x| < 2^22.
GF_HD float rint_small(float x) {
    const float magic = 12582912.0f;  // 1.5 * 2^23
    const float r = (x + magic) - magic;
    return r;
}

// 2^k for -149 <= k <= 127 as an exactly representable float.
GF_HD float pow2i(int k) {
    if (k >= -126) return u2f(uint32_t(k + 127) << 23);
    return u2f(1u << (k + 149));
}

// exp(x).
GF_HD float gf_expf(float x) {
    if (isnan_f(x)) return x;
    if (x > 88.72283935546875f) return inf_f();   // > log(FLT_MAX)
    if (x < -103.97208404541016f) return 0.0f;      // < log(2^-150)
    // ln 2 = LN2_HI + LN2_LO; LN2_HI keeps 16 significant bits (0x3f317200)
    // so k * LN2_HI is exact for |k| <= 150.
    const float LN2_HI = 0.693145751953125f;
    const float LN2_LO = 1.4286067653301870e-06f;
    const float INV_LN2 = 1.44269502162933349609375f;
    const float k = rint_small(x * INV_LN2);
    const float r = (x - k * LN2_HI) - k * LN2_LO;
    // Taylor coefficients 1/n!, n = 8 .. 0.
    float p = 2.4801587301587302e-05f;          // 1/8!
    p = fmaf_rn(p, r, 1.9841269841269841e-04f);  // 1/7!
    p = fmaf_rn(p, r, 1.3888888888888889e-03f);  // 1/6!
    p = fmaf_rn(p, r, 8.3333333333333332e-03f);  // 1/5!
    p = fmaf_rn(p, r, 4.1666666666666664e-02f);  // 1/4!
    p = fmaf_rn(p, r, 1.6666666666666666e-01f);  // 1/3!
    p = fmaf_rn(p, r, 0.5f);
    p = fmaf_rn(p, r, 1.0f);
    p = fmaf_rn(p, r, 1.0f);
    const int ki = int(k);
    const int k1 = ki / 2;
    const int k2 = ki - k1;
    return (p * pow2i(k1)) * pow2i(k2);
}

// log(x), natural logarithm.
GF_HD float gf_logf(float x) {
    if (isnan_f(x)) return x;
    if (x < 0.0f) return nan_f();
    if (x == 0.0f) return -inf_f();
    if (!isfinite_f(x)) return x;
    int e = 0;
    uint32_t u = f2u(x);
    if (u < 0x00800000u) {  // subnormal: scale by 2^23 first
        x = x * 8388608.0f;
        u = f2u(x);
        e = -23;
    }
    e += int(u >> 23) - 127;
    float m = u2f((u & 0x007fffffu) | 0x3f800000u);  // [1, 2)
    if (m > 1.41421353816986083984375f) {             // float(sqrt 2)
        m = m * 0.5f;
        e += 1;
    }
    const float s = (m - 1.0f) / (m + 1.0f);
    const float s2 = s * s;
    // atanh(s)/s = sum s^(2n)/(2n+1), n = 7 .. 1.
    float p = 6.6666666666666667e-02f;           // 1/15
    p = fmaf_rn(p, s2, 7.6923076923076927e-02f);  // 1/13
    p = fmaf_rn(p, s2, 9.0909090909090912e-02f);  // 1/11
    p = fmaf_rn(p, s2, 1.1111111111111111e-01f);  // 1/9
    p = fmaf_rn(p, s2, 1.4285714285714285e-01f);  // 1/7
    p = fmaf_rn(p, s2, 2.0000000000000001e-01f);  // 1/5
    p = fmaf_rn(p, s2, 3.3333333333333331e-01f);  // 1/3
    const float twoS = s + s;
    const float logm = fmaf_rn(twoS * s2, p, twoS);
    const float LN2_HI = 0.693145751953125f;
    const float LN2_LO = 1.4286067653301870e-06f;
    const float ef = float(e);
    return fmaf_rn(ef, LN2_HI, fmaf_rn(ef, LN2_LO, logm));
}

// atan(u) for |u| <= tan(pi/8).
GF_HD float atan_reduced(float u) {
    const float q = u * u;
    // atan(u) = u - u q S(q), S(q) = 1/3 - q/5 + q^2/7 - ... + q^8/19,
    // evaluated by Horner from the q^8 coefficient down.
    float p = 5.2631578947368418e-02f;            // +1/19
    p = fmaf_rn(p, q, -5.8823529411764705e-02f);  // -1/17
    p = fmaf_rn(p, q, 6.6666666666666666e-02f);   // +1/15
    p = fmaf_rn(p, q, -7.6923076923076927e-02f);  // -1/13
    p = fmaf_rn(p, q, 9.0909090909090912e-02f);   // +1/11
    p = fmaf_rn(p, q, -1.1111111111111111e-01f);  // -1/9
    p = fmaf_rn(p, q, 1.4285714285714285e-01f);   // +1/7
    p = fmaf_rn(p, q, -2.0000000000000001e-01f);  // -1/5
    p = fmaf_rn(p, q, 3.3333333333333331e-01f);   // +1/3
    return fmaf_rn(-(u * q), p, u);
}

// atan2(y, x) in (-pi, pi].
GF_HD float gf_atan2f(float y, float x) {
    if (isnan_f(x) || isnan_f(y)) return x + y;
    const float PI = 3.14159274101257324219f;
    const float PI_2 = 1.57079637050628662109f;
    const float PI_4 = 0.78539818525314331055f;
    const float ax = abs_f(x);
    const float ay = abs_f(y);
    const bool xneg = (f2u(x) & 0x80000000u) != 0u;
    if (ax == 0.0f && ay == 0.0f) {
        return copysign_f(xneg ? PI : 0.0f, y);
    }
    float a;
    if (!isfinite_f(ax) || !isfinite_f(ay)) {
        if (!isfinite_f(ax) && !isfinite_f(ay)) {
            a = PI_4;
            if (xneg) a = PI - a;
            return copysign_f(a, y);
        }
        a = isfinite_f(ax) ? PI_2 : 0.0f;
        if (xneg) a = PI - a;
        return copysign_f(a, y);
    }
    // pi, pi/2, pi/4 as float head + float tail (the tail is the rounding error of the head).
    const float PI_LO = -8.742277657347586e-08f;
    const float PI_2_LO = -4.371138828673793e-08f;
    const float PI_4_LO = -2.1855694143368964e-08f;
    const bool swap = ay > ax;
    const float mx = swap ? ay : ax;
    const float mn = swap ? ax : ay;
    const float t = mn / mx;  // [0, 1]
    if (t > 0.41421356237309503f) {  // tan(pi/8)
        const float u = (t - 1.0f) / (t + 1.0f);
        a = PI_4 + (atan_reduced(u) + PI_4_LO);
    } else {
        a = atan_reduced(t);
    }
    if (swap) a = (PI_2 - a) + PI_2_LO;
    if (xneg) a = (PI - a) + PI_LO;
    return copysign_f(a, y);
}

// ---------------------------------------------------------------- double
// Double-precision atan2 for the physical-mip search, shared by the oracle
// and the sm_100a kernel so both round identically.  |y|/|x| (or its
// reciprocal) lies in [0, 1]; with c = k/8 the nearest eighth,
// atan(t) = atan(c) + atan((t - c) / (1 + t c)), |(t - c)/(1 + t c)| <= 1/16,
// and the odd Taylor series of atan to the u^21 term leaves a truncation
// error below 1e-27 of u.  atan(k/8), pi/2 and pi are double head + tail
// pairs (the tail is the rounding error of the head).
GF_HD double atan_unit_d(double t) {
    const double HI[9] = {0.0, 0.12435499454676144, 0.24497866312686414, 0.35877067027057225, 0.4636476090008061,
                          0.5585993153435624, 0.6435011087932844, 0.7188299996216245, 0.7853981633974483};
    const double LO[9] = {0.0, -3.1253241424539383e-18, 1.0698755618734451e-17, -2.4623815582638635e-17,
                          2.2698777452961687e-17, -5.4556305485916264e-18, 1.5834785051444286e-17,
                          -2.1478388444456983e-17, 3.061616997868383e-17};
    const int k = int(t * 8.0 + 0.5);
    const double c = double(k) * 0.125;
    const double u = (t - c) / (1.0 + t * c);
    const double q = u * u;
    // S(q) = 1/3 - q/5 + q^2/7 - ... - q^9/21, atan(u) = u - u q S(q).
    double p = -1.0 / 21.0;
    p = p * q + 1.0 / 19.0;
    p = p * q - 1.0 / 17.0;
    p = p * q + 1.0 / 15.0;
    p = p * q - 1.0 / 13.0;
    p = p * q + 1.0 / 11.0;
    p = p * q - 1.0 / 9.0;
    p = p * q + 1.0 / 7.0;
    p = p * q - 1.0 / 5.0;
    p = p * q + 1.0 / 3.0;
    return HI[k] + (LO[k] + (u - (u * q) * p));
}

GF_HD bool isnan_d(double x) { return x != x; }
GF_HD bool isfinite_d(double x) { return x - x == 0.0; }

// atan2(y, x) in [-pi, pi] for finite arguments; NaN in, NaN out.
GF_HD double gf_atan2d(double y, double x) {
    if (isnan_d(x) || isnan_d(y)) return x + y;
    const double PI_HI = 3.141592653589793, PI_LO = 1.2246467991473532e-16;
    const double PI_2_HI = 1.5707963267948966, PI_2_LO = 6.123233995736766e-17;
    const double ax = x < 0.0 ? -x : x;
    const double ay = y < 0.0 ? -y : y;
    const bool xneg = x < 0.0 || (x == 0.0 && 1.0 / x < 0.0);
    const bool yneg = y < 0.0 || (y == 0.0 && 1.0 / y < 0.0);
    double a;
    if (ax == 0.0 && ay == 0.0) {
        a = xneg ? PI_HI : 0.0;
    } else if (!isfinite_d(ax) || !isfinite_d(ay)) {
        if (!isfinite_d(ax) && !isfinite_d(ay)) a = 0.5 * PI_2_HI;
        else a = isfinite_d(ax) ? PI_2_HI : 0.0;
        if (xneg) a = PI_HI - a;
    } else {
        const bool swap = ay > ax;
        const double t = swap ? ax / ay : ay / ax;  // [0, 1]
        a = atan_unit_d(t);
        if (swap) a = (PI_2_HI - a) + PI_2_LO;
        if (xneg) a = (PI_HI - a) + PI_LO;
    }
    return yneg ? -a : a;
}

// sqrt(x^2 + y^2) in this operation order (no rescaling: the physical-mip
// arguments are far from the overflow and underflow ranges).
GF_HD double gf_hypotd(double x, double y) { return sqrt(x * x + y * y); }

}  // namespace gf
