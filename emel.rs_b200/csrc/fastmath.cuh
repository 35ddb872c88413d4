// Binary64 exponential family for the f32 libm calls of the reference
// (expf, expm1f, tanhf), built for throughput on sm_100a.
//
// Method: Tang's table-driven exponential (P. T. P. Tang, "Table-driven
// implementation of the exponential function in IEEE floating-point
// arithmetic", ACM TOMS 15(2), 1989).  For a binary64 argument z:
//     n = nearest(z * 64/ln2),  n = 64 k + j  (0 <= j < 64)
//     r = z - n * ln2/64        (two-constant reduction, |r| <= ln2/128)
//     exp(z) = 2^k * T[j] * (1 + p),  T[j] = 2^(j/64),
//     p = expm1(r) by its Taylor polynomial to degree 6.
// Truncation error |r|^7/7! < 2^-57 and the binary64 rounding errors keep
// the relative error of exp near 2^-51, far inside binary32's 2^-24: after
// one rounding to binary32 the result is the correctly rounded value except
// when exp(z) lies within ~2^-51 of a rounding boundary.  The constants come
// from gen_exp_table.py (computed in 60-digit decimal, rounded once).
//
// expm1 and tanh reuse the split: expm1(z) = (s - 1) + s*p with
// s = 2^k T[j]; s - 1 is exact when s is in [1/2, 2] (Sterbenz), so there is
// no cancellation near 0 (there s = 1 and expm1 = p).  tanh(y) = -e/(e + 2)
// with e = expm1(-2|y|), sign restored.
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

// Low 32 bits of a binary64's encoding.
EMEL_HD int low_word(double x) {
#if defined(__CUDA_ARCH__)
    return __double2loint(x);
#else
    unsigned long long u;
    std::memcpy(&u, &x, 8);
    return (int)(unsigned)(u & 0xffffffffull);
#endif
}

EMEL_HD double bits_to_double(unsigned long long u) {
#if defined(__CUDA_ARCH__)
    return __longlong_as_double((long long)u);
#else
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

// Returns s = 2^k T[j] and p = expm1(r) for |z| <= 200.  n = nearest(z*64/ln2)
// comes from adding 1.5 * 2^52 (where the binary64 spacing is 1): the low
// word of the sum is n and subtracting the constant back is exact, so no
// float<->int conversion is issued.
EMEL_HD void exp_split(double z, double& s, double& p) {
    constexpr double kShift = 0x1.8p52;
    const double t = std::fma(z, kExpInvL, kShift);
    const int n = low_word(t);
    const double nd = t - kShift;
    double r = std::fma(-nd, kExpLhi, z);
    r = std::fma(-nd, kExpLlo, r);
    double q = std::fma(r, 1.0 / 720.0, 1.0 / 120.0);
    q = std::fma(q, r, 1.0 / 24.0);
    q = std::fma(q, r, 1.0 / 6.0);
    q = std::fma(q, r, 0.5);
    q = std::fma(q, r, 1.0);
    p = q * r;
    const int j = n & 63;
    const int k = n >> 6;
    s = exp_table(j) * bits_to_double((unsigned long long)(unsigned)(k + 1023) << 52);
}

// Clamp for the float-valued exponentials: beyond +-200 the binary32 result
// is already inf / 0 / -1.  NaN passes (both comparisons false).
EMEL_HD double exp_arg(double z) { return z > 200.0 ? 200.0 : (z < -200.0 ? -200.0 : z); }

EMEL_HD double exp_d(double z) {
    double s, p;
    exp_split(exp_arg(z), s, p);
    return std::fma(s, p, s);
}

EMEL_HD double expm1_d(double z) {
    if (z == 0.0) return z;  // keeps the sign of zero
    double s, p;
    exp_split(exp_arg(z), s, p);
    return std::fma(s, p, s - 1.0);
}

// tanh for |y| < 10 (callers saturate beyond): -e / (e + 2), e = expm1(-2|y|).
EMEL_HD double tanh_d(double y) {
    if (y == 0.0) return y;
    const double e = expm1_d(-2.0 * std::fabs(y));
    const double t = -e / (e + 2.0);
    return y < 0.0 ? -t : t;
}

EMEL_HD float fast_expf(float x) { return (float)exp_d((double)x); }
EMEL_HD float fast_expm1f(float x) { return (float)expm1_d((double)x); }

// tanh(y) rounds to +-1 in binary32 once |y| > 9.02.
EMEL_HD float fast_tanhf(float y) {
    if (std::fabs(y) >= 10.0f) return y < 0.0f ? -1.0f : 1.0f;
    return (float)tanh_d((double)y);
}

}  // namespace emel
