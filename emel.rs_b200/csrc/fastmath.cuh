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


// ===========================================================================
// Binary32 exponential family: the default for the activation, soft_max and
// GLU kernels.  The reference's tolerance for transcendental unary ops is
// 2 ulp, so the correctly rounded binary64 evaluation above is more than the
// path needs; this one runs entirely in binary32 FMAs.
//
// Method (Cody-Waite reduction, W. J. Cody and W. Waite, "Software Manual
// for the Elementary Functions", 1980, with a Taylor polynomial):
//     k = nearest(x / ln2)                       (1.5 * 2^23 shift)
//     r = x - k * Ln2Hi     exact: Ln2Hi is ln2 rounded to binary32, so
//                           k * Ln2Hi is a multiple of 2^-24 and the
//                           difference (|r| < 0.35) fits 24 bits; the FMA
//                           forms it without intermediate rounding
//     c = -k * Ln2Lo        (Ln2Lo = ln2 - Ln2Hi, |c| < 3e-7)
//     e^(r + c) - 1 = r + t,  t = r^2 (1/2! + r/3! + ... + r^5/7!) + c (1 + r)
//     exp(x) = 2^k (1 + r + t)
// Taylor truncation at degree 7 is below 2^-27 relative for |r| <= 0.35;
// the constants are generated by gen_exp_table.py (1/ln2, the ln2 split and
// 1/k!, each rounded once to binary32).  The power of two is applied as
// 2^k1 * 2^k2 (k1 kept in the normal range) so results near overflow and
// in the subnormal range need no special case.
//
// expm1(x) = (2^k - 1) + 2^k r + 2^k t: the first two terms are formed with
// one rounding (2^k r is exact and 2^k - 1 is exact for |k| <= 24), so there
// is no cancellation; with k = 0 it is r + t.
// tanh(|y|) = e / (e + 2) with e = expm1(2|y|) > 0 below 0.625 (no
// cancellation; the quotient's sensitivity to e stays below one), and
// 1 - 2 / (exp(2|y|) + 1) above, where the subtracted term is small and its
// relative error becomes a far smaller absolute one: near +-1 the result is
// the correctly rounded value unless it lies next to a rounding boundary.
// Over every binary32 input, against binary64 libm rounded once: exp and
// expm1 within 1 ulp, tanh within 2 (tests/cpp/fastmath_check.cpp).
// ===========================================================================

EMEL_HD float fma32(float a, float b, float c) {
#if defined(__CUDA_ARCH__)
    return __fmaf_rn(a, b, c);
#else
    return std::fma(a, b, c);
#endif
}

EMEL_HD uint32_t f32_to_bits(float f) {
#if defined(__CUDA_ARCH__)
    return __float_as_uint(f);
#else
    uint32_t u;
    std::memcpy(&u, &f, 4);
    return u;
#endif
}

EMEL_HD float bits_to_f32(uint32_t u) {
#if defined(__CUDA_ARCH__)
    return __uint_as_float(u);
#else
    float f;
    std::memcpy(&f, &u, 4);
    return f;
#endif
}

// 2^e for -126 <= e <= 127.
EMEL_HD float pow2i(int e) { return bits_to_f32((uint32_t)(e + 127) << 23); }

// k, r and t with e^(x - k ln2) - 1 = r + t for |x| <= 104: r is the exact
// reduced argument, t = r^2 (1/2! + ... + r^5/7!) + c (1 + r) carries the
// rest (|t| < 0.07).
EMEL_HD void f32_exp_split(float x, int& k, float& r, float& t) {
    constexpr float kShift = 0x1.8p23f;
    const float tk = fma32(x, kF32InvLn2, kShift);
    k = (int)(f32_to_bits(tk) - f32_to_bits(kShift));
    const float kd = tk - kShift;  // exact
    r = fma32(-kd, kF32Ln2Hi, x);
    const float c = -kd * kF32Ln2Lo;
    float q = fma32(r, kF32InvFact7, kF32InvFact6);
    q = fma32(q, r, kF32InvFact5);
    q = fma32(q, r, kF32InvFact4);
    q = fma32(q, r, kF32InvFact3);
    q = fma32(q, r, kF32InvFact2);
    t = fma32(c, r, fma32(r * r, q, c));
}

// exp(x) within one ulp, any x.  Saturates like the binary32 result (inf
// above 89, +0 below -104); NaN propagates (every comparison is false).
EMEL_HD float exp32_general(float x) {
    const float xc = x > 89.0f ? 89.0f : (x < -104.0f ? -104.0f : x);
    int k;
    float r, t;
    f32_exp_split(xc, k, r, t);
    const int k1 = k > 127 ? 127 : (k < -100 ? -100 : k);
    const float s1 = pow2i(k1), s2 = pow2i(k - k1);
    const float y = fma32(s1, r + t, s1) * s2;
    return x > 89.0f ? INFINITY : (x < -104.0f ? 0.0f : y);
}

// exp(x): where the result is a normal binary32 number (-86 <= x <= 88.72)
// 2^k is one exponent-field value -- 2^(k-1) scaled by 2 keeps k = 128 in
// range -- and no saturation is needed; everything else (subnormal results,
// overflow, NaN) takes the general routine.  The same bits either way.
EMEL_HD float exp32(float x) {
    if (!(x >= -86.0f && x <= 88.72f)) return exp32_general(x);
    int k;
    float r, t;
    f32_exp_split(x, k, r, t);
    const float sh = bits_to_f32((uint32_t)(k + 126) << 23);  // 2^(k-1), -125 <= k - 1 <= 127
    return fma32(sh, r + t, sh) * 2.0f;
}

// expm1(x) within one ulp; saturates to -1 below -18 and to inf above 89;
// keeps -0.
EMEL_HD float expm1_32(float x) {
    const float xc = x > 89.0f ? 89.0f : (x < -18.0f ? -18.0f : x);
    int k;
    float r, t;
    f32_exp_split(xc, k, r, t);
    const int k1 = k > 127 ? 127 : k;  // k >= -26 here
    const int k2 = k - k1;             // 0, or 1 right below the overflow threshold
    const float s1 = pow2i(k1);
    // (2^k1 - 2^-k2) + 2^k1 r is formed with one rounding (2^k1 r is exact),
    // then the small tail 2^k1 t is added
    const float y = fma32(s1, t, fma32(s1, r, s1 - pow2i(-k2))) * pow2i(k2);
    if (x == 0.0f) return x;
    return x > 89.0f ? INFINITY : (x < -18.0f ? -1.0f : y);
}

// tanh(y) within two ulp; +-1 once |y| >= 10 (binary32 tanh rounds to +-1
// above 9.02).
EMEL_HD float tanh32(float y) {
    const float ay = std::fabs(y);
    const float ac = ay >= 10.0f ? 10.0f : ay;
    float t;
    if (ac < 0.625f) {
        const float e = expm1_32(2.0f * ac);
        t = e / (e + 2.0f);
    } else {
        t = 1.0f - 2.0f / (exp32(2.0f * ac) + 1.0f);
    }
    const float s = y < 0.0f ? -1.0f : 1.0f;
    const float r = ay >= 10.0f ? s : (y < 0.0f ? -t : t);
    return y == 0.0f ? y : r;
}

// exp(x) inside a gate 1 + exp(x) (sigmoid, silu and the GLU gates, whose
// quotient is then taken).  From x > 15.9 on exp(x) >= 2^23, where the sum
// 1 + exp(x) rounds and a one-ulp difference in exp(x) can become several
// ulp of the quotient; there the correctly rounded binary64 evaluation is
// used, so the gate is the correctly rounded formula's.  Below, exp32.
constexpr float kExpGateCr = 15.9f;
EMEL_HD float exp32_gate(float x) { return x > kExpGateCr ? fast_expf(x) : exp32(x); }

#if defined(__CUDACC__)
// exp32 (GATE: exp32_gate) on a pair of arguments.  When both lie in the
// one-scale packed range the two lanes run exp32's operations packed two to
// an instruction (__ffma2_rn / __fadd2_rn / __fmul2_rn round each lane
// exactly like the scalar operation), so each lane gets the scalar bits at
// about half the instructions; otherwise each lane calls the scalar form.
template <bool GATE = false>
__device__ __forceinline__ float2 exp32x2(float2 x) {
    constexpr float kTop = GATE ? kExpGateCr : 88.72f;
    if (!(x.x >= -86.0f && x.x <= kTop && x.y >= -86.0f && x.y <= kTop))
        return GATE ? make_float2(exp32_gate(x.x), exp32_gate(x.y)) : make_float2(exp32(x.x), exp32(x.y));
    constexpr float kShift = 0x1.8p23f;
    auto sp = [](float v) { return make_float2(v, v); };
    const float2 tk = __ffma2_rn(x, sp(kF32InvLn2), sp(kShift));
    const float2 kd = __fadd2_rn(tk, sp(-kShift));  // exact
    const float2 nkd = make_float2(-kd.x, -kd.y);
    const float2 r = __ffma2_rn(nkd, sp(kF32Ln2Hi), x);
    const float2 c = __fmul2_rn(nkd, sp(kF32Ln2Lo));
    float2 q = __ffma2_rn(r, sp(kF32InvFact7), sp(kF32InvFact6));
    q = __ffma2_rn(q, r, sp(kF32InvFact5));
    q = __ffma2_rn(q, r, sp(kF32InvFact4));
    q = __ffma2_rn(q, r, sp(kF32InvFact3));
    q = __ffma2_rn(q, r, sp(kF32InvFact2));
    const float2 t = __ffma2_rn(c, r, __ffma2_rn(__fmul2_rn(r, r), q, c));
    // 2^(k - 1) with k = bits(tk) - bits(kShift), as in exp32
    const uint32_t kb = f32_to_bits(kShift) - 126u;
    const float2 sh = make_float2(bits_to_f32((f32_to_bits(tk.x) - kb) << 23), bits_to_f32((f32_to_bits(tk.y) - kb) << 23));
    return __fmul2_rn(__ffma2_rn(sh, __fadd2_rn(r, t), sh), sp(2.0f));
}
#endif

}  // namespace emel
