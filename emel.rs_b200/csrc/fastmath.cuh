// Binary64 exponential family for the f32 libm calls of the reference
// (expf, expm1f, tanhf), built for throughput on sm_100a.
//
// Method: Tang's table-driven exponential (P. T. P. Tang, "Table-driven
// implementation of the exponential function in IEEE floating-point
// arithmetic", ACM TOMS 15(2), 1989).  For a binary64 argument z:
//     n = nearest(z * 64/ln2),  n = 64 k + j  (0 <= j < 64)
//     r = z - n * ln2/64        (two-constant reduction, |r| <= ln2/128)
//     exp(z) = 2^k * T[j] * (1 + p),  T[j] = 2^(j/64),
//     p = expm1(r) by its Taylor polynomial to degree 5.
// Truncation error |r|^6/6! < 2^-54 and the binary64 rounding errors keep
// the relative error of exp near 2^-51, far inside binary32's 2^-24: after
// one rounding to binary32 the result is the correctly rounded value except
// when exp(z) lies within ~2^-51 of a rounding boundary.  The constants come
// from gen_exp_table.py (computed in 60-digit decimal, rounded once).
//
// expm1 and tanh reuse the split: expm1(z) = (s - 1) + s*p with
// s = 2^k T[j]; s - 1 is exact when s is in [1/2, 2] (Sterbenz), so there is
// no cancellation near 0 (there s = 1 and expm1 = p).  tanh(y) = -e/(e + 2)
// with e = expm1(-2|y|), sign restored; the division uses a binary32
// reciprocal estimate refined by two binary64 Newton steps (relative error
// below 2^-52 for a denominator in (1, 2]).
//
// Range handling is done once on the binary32 argument by the f32 entry
// points, so the binary64 core runs without clamps or special cases.
//
// The header also compiles as plain C++ (host) so the same arithmetic can be
// unit-tested on the CPU: fma is IEEE on both sides.
#pragma once

#include <cmath>
#include <cstdint>
#include <cstring>

#if defined(__CUDACC__)
#define EMEL_HD __host__ __device__ __forceinline__
#else
#define EMEL_HD inline
#endif

namespace emel {

#include "exp_table.inc"

#if defined(__CUDACC__)
static __device__ const double kExpT[64] = {EMEL_EXP_TABLE_VALUES};
#endif
static const double kExpTHost[64] = {EMEL_EXP_TABLE_VALUES};

EMEL_HD int lo_word(double x) {
#if defined(__CUDA_ARCH__)
    return __double2loint(x);
#else
    unsigned long long u;
    std::memcpy(&u, &x, 8);
    return (int)(unsigned)(u & 0xffffffffull);
#endif
}

EMEL_HD int hi_word(double x) {
#if defined(__CUDA_ARCH__)
    return __double2hiint(x);
#else
    unsigned long long u;
    std::memcpy(&u, &x, 8);
    return (int)(unsigned)(u >> 32);
#endif
}

EMEL_HD double from_words(int hi, int lo) {
#if defined(__CUDA_ARCH__)
    return __hiloint2double(hi, lo);
#else
    const unsigned long long u = ((unsigned long long)(unsigned)hi << 32) | (unsigned)lo;
    double d;
    std::memcpy(&d, &u, 8);
    return d;
#endif
}

EMEL_HD double exp_table(int j) {
#if defined(__CUDA_ARCH__)
    return __ldg(&kExpT[j]);
#else
    return kExpTHost[j];
#endif
}

// Approximate binary32 reciprocal (about 23 correct bits).
EMEL_HD float rcp_estimate(float x) {
#if defined(__CUDA_ARCH__)
    float r;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
    return r;
#else
    return 1.0f / x;
#endif
}

// s = 2^k T[j] and p = expm1(r) for |z| <= 200.  n = nearest(z * 64/ln2)
// comes from adding 1.5 * 2^52 (where the binary64 spacing is 1): the low
// word of the sum is n and subtracting the constant back is exact, so no
// float<->int conversion is issued.  2^k is applied by adding k to the
// exponent field of T[j] (in range for |k| <= 289).
EMEL_HD void exp_split(double z, double& s, double& p) {
    constexpr double kShift = 0x1.8p52;
    const double t = std::fma(z, kExpInvL, kShift);
    const int n = lo_word(t);
    const double nd = t - kShift;
    double r = std::fma(-nd, kExpLhi, z);
    r = std::fma(-nd, kExpLlo, r);
    double q = std::fma(r, 1.0 / 120.0, 1.0 / 24.0);
    q = std::fma(q, r, 1.0 / 6.0);
    q = std::fma(q, r, 0.5);
    q = std::fma(q, r, 1.0);
    p = q * r;
    const double tj = exp_table(n & 63);
    s = from_words((int)((unsigned)hi_word(tj) + ((unsigned)(n >> 6) << 20)), lo_word(tj));
}

EMEL_HD double exp_core(double z) {
    double s, p;
    exp_split(z, s, p);
    return std::fma(s, p, s);
}

EMEL_HD double expm1_core(double z) {
    double s, p;
    exp_split(z, s, p);
    return std::fma(s, p, s - 1.0);
}

// tanh(|y|) for 0 < |y| < 10: -e / (e + 2), e = expm1(-2|y|) in (-1, 0).
EMEL_HD double tanh_abs_core(double ay) {
    const double e = expm1_core(-2.0 * ay);
    const double d = e + 2.0;  // in (1, 2]
    double r = (double)rcp_estimate((float)d);
    r = std::fma(r, std::fma(-d, r, 1.0), r);
    r = std::fma(r, std::fma(-d, r, 1.0), r);
    return -e * r;
}

// binary32 entry points: correctly rounded except within ~2^-51 of a
// rounding boundary.  Out-of-range arguments saturate the way the binary32
// result does (exp: inf / +0, expm1: inf / -1, tanh: +-1); NaN propagates.
// Branch-free: the argument is clamped into the core's range (comparisons
// with NaN are false, so a NaN passes through), the core is evaluated, and
// the saturated cases are selected afterwards.
EMEL_HD float fast_expf(float x) {
    const float xc = x > 89.0f ? 89.0f : (x < -104.0f ? -104.0f : x);
    const float r = (float)exp_core((double)xc);
    return x > 89.0f ? INFINITY : (x < -104.0f ? 0.0f : r);
}

EMEL_HD float fast_expm1f(float x) {
    const float xc = x > 89.0f ? 89.0f : (x < -18.0f ? -18.0f : x);
    const float r = (float)expm1_core((double)xc);
    if (x == 0.0f) return x;  // keeps the sign of zero
    return x > 89.0f ? INFINITY : (x < -18.0f ? -1.0f : r);
}

// tanh(y) rounds to +-1 in binary32 once |y| > 9.02.
EMEL_HD float fast_tanhf(float y) {
    const float ay = std::fabs(y);
    const float ac = ay >= 10.0f ? 10.0f : ay;
    const float t = (float)tanh_abs_core((double)ac);
    const float s = y < 0.0f ? -1.0f : 1.0f;
    const float r = ay >= 10.0f ? s : (y < 0.0f ? -t : t);
    return y == 0.0f ? y : r;
}

}  // namespace emel
