// Device-side numeric helpers shared by every kernel of the device op table.
//
// Bit-exactness contract: results must equal the reference's x86-64 CPU
// loops (IEEE binary32, round-to-nearest-even, no FMA contraction, subnormals
// kept).  The translation units are compiled with -fmad=false -ftz=false
// -prec-div=true -prec-sqrt=true, and every formula spells out the
// reference's operation order.  Two things differ between SSE and the GPU
// and are handled here explicitly:
//   * NaN results: SSE returns the first NaN operand, quietened, or the
//     "indefinite" QNaN 0xFFC00000 for an invalid operation; the GPU returns
//     a canonical NaN.  `x86_nan2`/`x86_nan1` rebuild the SSE bits.
//   * sign/abs: PTX neg/abs leave NaN payloads unspecified, so they are
//     done on the integer bits.
// exp / expm1 / tanh run on the binary32 core of fastmath.cuh (within 1 / 1
// / 2 ulp of the correctly rounded value over every binary32 input; the
// tolerance for transcendental unary ops is 2 ulp); log, log1p, sin and cos
// are evaluated in binary64 and rounded once.
#pragma once

#include <cuda_fp16.h>
#include <cstdint>

#include "fastmath.cuh"
#include "plan.hpp"

namespace emel {

constexpr uint32_t kIndefiniteNaN = 0xFFC00000u;

__device__ __forceinline__ uint32_t fbits(float f) { return __float_as_uint(f); }
__device__ __forceinline__ float bitsf(uint32_t u) { return __uint_as_float(u); }
__device__ __forceinline__ bool is_nan(float f) { return (fbits(f) & 0x7fffffffu) > 0x7f800000u; }
__device__ __forceinline__ float quiet(float f) { return bitsf(fbits(f) | 0x00400000u); }

// Result of an SSE binary operation whose GPU result `r` was computed from
// operands (a, b) in that source order.
__device__ __forceinline__ float x86_nan2(float r, float a, float b) {
    if (!is_nan(r)) return r;
    if (is_nan(a)) return quiet(a);
    if (is_nan(b)) return quiet(b);
    return bitsf(kIndefiniteNaN);
}

// Result of a fused multiply-add (a * b + c): the first NaN operand in
// source order, quietened, or the invalid-operation QNaN.
__device__ __forceinline__ float x86_nan3(float r, float a, float b, float c) {
    if (!is_nan(r)) return r;
    if (is_nan(a)) return quiet(a);
    if (is_nan(b)) return quiet(b);
    if (is_nan(c)) return quiet(c);
    return bitsf(kIndefiniteNaN);
}

// Result of a one-input libm/SSE operation: a NaN input comes back quietened,
// a NaN produced from a number is the invalid-operation QNaN.
__device__ __forceinline__ float x86_nan1(float r, float a) {
    if (!is_nan(r)) return r;
    if (is_nan(a)) return quiet(a);
    return bitsf(kIndefiniteNaN);
}

__device__ __forceinline__ float f_add(float a, float b) { return x86_nan2(__fadd_rn(a, b), a, b); }
__device__ __forceinline__ float f_sub(float a, float b) { return x86_nan2(__fsub_rn(a, b), a, b); }
__device__ __forceinline__ float f_mul(float a, float b) { return x86_nan2(__fmul_rn(a, b), a, b); }
__device__ __forceinline__ float f_div(float a, float b) { return x86_nan2(__fdiv_rn(a, b), a, b); }
__device__ __forceinline__ float f_neg(float a) { return bitsf(fbits(a) ^ 0x80000000u); }
__device__ __forceinline__ float f_abs(float a) { return bitsf(fbits(a) & 0x7fffffffu); }
__device__ __forceinline__ float f_sqrt(float a) { return x86_nan1(__fsqrt_rn(a), a); }

// binary32 <-> binary16 with the reference's NaN behaviour: a NaN becomes the
// quiet half 0x7E00 with the input's sign (unary.rs:546-570); a half NaN
// widens with its payload shifted up and quietened (unary.rs:572-586).  For
// every other value both directions are exact IEEE conversions (RNE when
// narrowing), which the hardware cvt instructions implement.
__device__ __forceinline__ uint16_t f32_to_f16_bits(float v) {
    if (is_nan(v)) return (uint16_t)(((fbits(v) >> 16) & 0x8000u) | 0x7e00u);
    return __half_as_ushort(__float2half_rn(v));
}

__device__ __forceinline__ float f16_bits_to_f32(uint16_t h) {
    if ((h & 0x7fffu) > 0x7c00u) return bitsf(((uint32_t)(h & 0x8000u) << 16) | 0x7fc00000u | ((uint32_t)(h & 0x3ffu) << 13));
    return __half2float(__ushort_as_half(h));
}

// ---------------------------------------------------------------------------
// Binary formulas (binary.rs:386-409).
// ---------------------------------------------------------------------------

template <int OP>
__device__ __forceinline__ float binary_apply(float a, float b) {
    if constexpr (OP == kAdd) return f_add(a, b);
    if constexpr (OP == kSub) return f_sub(a, b);
    if constexpr (OP == kMul) return f_mul(a, b);
    return f_div(a, b);
}

// ---------------------------------------------------------------------------
// Unary formulas (unary.rs:474-672, power.rs:315/397-412,
// reductions.rs:640-668, activation.rs:366-521, elementwise.rs:280-291).
// Codes match emel_cuda_unary_op; parameterised ops use codes >= 128.
// ---------------------------------------------------------------------------

struct UnaryParams {
    float a;
    float b;
};

// The reference's libm calls (f32::exp, exp_m1, tanh) on binary32 results:
// the binary32 core of fastmath.cuh (exp and expm1 within 1 ulp of the
// correctly rounded value over every binary32 input, tanh within 2), with
// the x86 NaN rules.  The _cr forms evaluate in binary64 and round once
// (correctly rounded but for rare double-rounding ties): the standalone tanh
// op (glibc's tanhf is itself up to 2 ulp from the correctly rounded value,
// so a 2-ulp tanh could sit 4 ulp from it) and the paths whose parity is
// pinned bit for bit on the reference's golden vectors (single-query
// attention's binary16 recurrence, RoPE frequencies, silu_back).
__device__ __forceinline__ float lm_exp(float x) { return x86_nan1(exp32(x), x); }
__device__ __forceinline__ float lm_exp_gate(float x) { return x86_nan1(exp32_gate(x), x); }
__device__ __forceinline__ float lm_expm1(float x) { return x86_nan1(expm1_32(x), x); }
__device__ __forceinline__ float lm_tanh(float x) { return x86_nan1(tanh32(x), x); }
__device__ __forceinline__ float lm_exp_cr(float x) { return x86_nan1(fast_expf(x), x); }
__device__ __forceinline__ float lm_tanh_cr(float x) { return x86_nan1(fast_tanhf(x), x); }
// exp(z) for the fast soft_max passes (z = v - max <= 0, or NaN), whose bar
// is 1e-5 relative on the outputs: 2^(z log2 e) with z log2 e carried as a
// binary32 pair, hi = RN(z * L) and lo = z * L - hi (exact through the FMA)
// + z * Llo, L + Llo = log2 e; 2^hi from the SFU's ex2 and 2^lo applied as
// 1 + lo ln 2 (|lo| < 2^-17, so the next term is below 2^-35).  Measured over
// every binary32 z in [-87.33, 0]: relative error at most 2.4e-7 (3 ulp; 14
// arguments above 2 ulp).  Below -87 -- results in binary32's subnormal
// range, which the SFU flushes -- and for NaN, the binary32 core.
__device__ __forceinline__ float softmax_exp(float z) {
    if (!(z >= -87.0f)) return exp32(z);
    constexpr float kLog2e = 0x1.715476p0f, kLog2eLo = 0x1.4ae0cp-26f, kLn2 = 0x1.62e43p-1f;
    const float hi = __fmul_rn(z, kLog2e);
    const float lo = __fmaf_rn(z, kLog2eLo, __fmaf_rn(z, kLog2e, -hi));
    float r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(hi));
    return __fmaf_rn(r, __fmul_rn(lo, kLn2), r);
}

// Packed binary32 pairs.  sm_100a executes add / mul / fma on two binary32
// lanes in one instruction (__fadd2_rn, __fmul2_rn, __ffma2_rn), each lane
// rounded exactly like the scalar operation, so the pair forms below give
// the scalar forms' bits at half the instruction count.  x - y is written
// x + (-y), which IEEE 754 defines it to be.
__device__ __forceinline__ float2 lo2(float4 v) { return make_float2(v.x, v.y); }
__device__ __forceinline__ float2 hi2(float4 v) { return make_float2(v.z, v.w); }
__device__ __forceinline__ float4 cat2(float2 a, float2 b) { return make_float4(a.x, a.y, b.x, b.y); }
__device__ __forceinline__ float2 splat2(float x) { return make_float2(x, x); }

// Three-operand maximum / minimum (sm_100a): fmaxf / fminf of three values,
// NaN operands skipped the same way.
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}
__device__ __forceinline__ float fmin3(float a, float b, float c) {
    float d;
    asm("min.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// exp(z) for a pair of soft_max terms with -41 <= z <= 0 (the callers test
// the range; NaN and anything below go to softmax_exp): Cody-Waite reduction
// against base 2, hi = RN(z log2 e), lo = z - hi ln2 with ln2 split in two
// binary32 constants (two FMAs, each rounding once at |lo| < 2^-17), then
// exp(z) = 2^hi e^lo = ex2(hi) (1 + lo), the dropped lo^2 / 2 below 2^-35.
// The error is the SFU's ex2 (a few units of 2^-24), the bar softmax_exp
// is held to.
__device__ __forceinline__ float2 softmax_exp2(float2 z) {
    constexpr float kLog2e = 0x1.715476p0f, kLn2Hi = 0x1.62e43p-1f, kLn2Lo = -0x1.05c610p-29f;
    const float2 hi = __fmul2_rn(z, splat2(kLog2e));
    float2 lo = __ffma2_rn(hi, splat2(-kLn2Hi), z);
    lo = __ffma2_rn(hi, splat2(-kLn2Lo), lo);
    float2 r;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r.x) : "f"(hi.x));
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r.y) : "f"(hi.y));
    return __ffma2_rn(r, lo, r);
}

// e / d rounded once for 0 <= e <= 1 and a finite d >= 1, given
// inv = RN(1 / d): q0 = RN(e * inv) is within one ulp of e / d, the FMA
// residual e - d * q0 is exact, and RN(q0 + residual * inv) is the
// correctly rounded quotient (Markstein's theorem on reciprocal-based
// division).  e = 0 gives +0 through the same steps; 0 < e < 2^-60, whose
// quotient could leave the normal range, uses the divider (softmax_div).
__device__ __forceinline__ float markstein_div(float e, float d, float inv) {
    const float q0 = __fmul_rn(e, inv);
    return __fmaf_rn(__fmaf_rn(-d, q0, e), inv, q0);
}

// markstein_div on a pair (same bits per lane), d2 = (d, d), inv2 = (inv, inv).
__device__ __forceinline__ float2 markstein_div2(float2 e, float2 d2, float2 inv2) {
    const float2 q0 = __fmul2_rn(e, inv2);
    return __ffma2_rn(__ffma2_rn(make_float2(-d2.x, -d2.y), q0, e), inv2, q0);
}

// a / b inside the transcendental formulas (sigmoid, silu and the GLU
// gates, denominators 1 + exp(...) >= 1): the reciprocal estimate refined
// by one residual step, q0 = a * rcp(b), q = q0 + (a - b * q0) * rcp(b), the
// residual exact through the FMA.  Within one ulp of a / b in general, and
// bit-identical to the IEEE quotient for every binary32 argument of
// silu's x / (1 + exp(-x)) and sigmoid's 1 / (1 + exp(-x)) (checked
// exhaustively on the device), at a third of the divider's instructions.
// A NaN residual (an infinite operand) leaves
// q0, which is already the IEEE limit there: x / inf = +-0, inf / 1 = inf,
// inf / inf = NaN.
__device__ __forceinline__ float div_refined(float a, float b) {
    float y;
    asm("rcp.approx.f32 %0, %1;" : "=f"(y) : "f"(b));
    const float q0 = __fmul_rn(a, y);
    const float r = __fmaf_rn(-b, q0, a);
    const float q = __fmaf_rn(r, y, q0);
    // a zero quotient keeps q0's sign (-0 / 2 = -0: the residual step would add +0)
    return r != r ? q0 : copysignf(q, q0);
}

// div_refined on a pair: the same operations lane for lane, the multiply and
// the two FMAs packed.
__device__ __forceinline__ float2 div_refined2(float2 a, float2 b) {
    float2 y;
    asm("rcp.approx.f32 %0, %1;" : "=f"(y.x) : "f"(b.x));
    asm("rcp.approx.f32 %0, %1;" : "=f"(y.y) : "f"(b.y));
    const float2 q0 = __fmul2_rn(a, y);
    const float2 r = __ffma2_rn(make_float2(-b.x, -b.y), q0, a);
    const float2 q = __ffma2_rn(r, y, q0);
    return make_float2(r.x != r.x ? q0.x : copysignf(q.x, q0.x), r.y != r.y ? q0.y : copysignf(q.y, q0.y));
}

__device__ __forceinline__ float softmax_div(float e, float d, float inv) {
    const float q = markstein_div(e, d, inv);
    if (e < 0x1p-60f && e != 0.0f) return __fdiv_rn(e, d);
    return q;
}

// While every v - max of a soft_max row is >= kSoftmaxPlainDivFloor, each
// e is at least e^-41 > 2^-60 (or exactly 1), so markstein_div needs no
// range check.
constexpr float kSoftmaxPlainDivFloor = -41.0f;

__device__ __forceinline__ float lm_log(float x) { return x86_nan1((float)log((double)x), x); }
__device__ __forceinline__ float lm_log1p(float x) { return x86_nan1((float)log1p((double)x), x); }
__device__ __forceinline__ float lm_sin(float x) { return x86_nan1((float)sin((double)x), x); }
__device__ __forceinline__ float lm_cos(float x) { return x86_nan1((float)cos((double)x), x); }

// f32::clamp: both comparisons false for NaN, which passes through with its
// payload.  The NaN test is on the integer bits so the compiler cannot fold
// the selection into a NaN-canonicalising min/max.
__device__ __forceinline__ float clamp_rs(float v, float lo, float hi) {
    if (is_nan(v)) return v;
    if (v < lo) return lo;
    if (v > hi) return hi;
    return v;
}

// Arithmetic policies for the formulas.
//   kFast   plain IEEE binary32 operations and the binary32 exponential core;
//   kExact  the same values with the reference's x86 NaN semantics on every
//           operation.  The two agree bit for bit on every non-NaN result
//           (a selection on a NaN intermediate does not depend on its
//           payload), so the heavy formulas run kFast and recompute kExact
//           only when the result is NaN;
//   kHalf   for results rounded to binary16 (binary16 storage, and GELU,
//           whose formula rounds its output through binary16): CUDA's
//           exponential and division intrinsics (__expf, __fdividef: a few
//           binary32 ulp) where binary16's half-ulp of 2^-12 relative
//           absorbs them.  expm1 stays on the binary32 core (a small
//           negative argument would lose relative accuracy to exp - 1), and
//           tanh is 1 - 2 / (exp(2|y|) + 1): its error is absolute and tiny
//           near +-1, where GELU's 1 + tanh cancels.
enum ArithMode : int { kFast = 0, kExact = 1, kHalf = 2 };

template <int MODE>
struct Arith {
    static constexpr bool EXACT = MODE == kExact;
    static __device__ __forceinline__ float add(float a, float b) { return EXACT ? f_add(a, b) : __fadd_rn(a, b); }
    static __device__ __forceinline__ float sub(float a, float b) { return EXACT ? f_sub(a, b) : __fsub_rn(a, b); }
    static __device__ __forceinline__ float mul(float a, float b) { return EXACT ? f_mul(a, b) : __fmul_rn(a, b); }
    static __device__ __forceinline__ float div(float a, float b) { return EXACT ? f_div(a, b) : __fdiv_rn(a, b); }
    // division inside a transcendental formula (a few ulp allowed)
    static __device__ __forceinline__ float tdiv(float a, float b) { return EXACT ? f_div(a, b) : div_refined(a, b); }
    static __device__ __forceinline__ float exp(float x) { return EXACT ? lm_exp(x) : exp32(x); }
    // exp inside a gate 1 + exp(x) (exp32_gate)
    static __device__ __forceinline__ float exp_gate(float x) { return EXACT ? lm_exp_gate(x) : exp32_gate(x); }
    static __device__ __forceinline__ float expm1(float x) { return EXACT ? lm_expm1(x) : expm1_32(x); }
    static __device__ __forceinline__ float tanh(float x) { return EXACT ? lm_tanh(x) : tanh32(x); }
    // the standalone tanh op (unary.rs OpUnary Tanh): correctly rounded
    static __device__ __forceinline__ float tanh_op(float x) { return EXACT ? lm_tanh_cr(x) : fast_tanhf(x); }
    static __device__ __forceinline__ float log1p(float x) { return EXACT ? lm_log1p(x) : (float)::log1p((double)x); }
    // fp16_to_f32(fp32_to_fp16(v)) (unary.rs:533,539)
    static __device__ __forceinline__ float round_f16(float v) {
        return EXACT ? f16_bits_to_f32(f32_to_f16_bits(v)) : __half2float(__float2half_rn(v));
    }
    static __device__ __forceinline__ float fma(float a, float b, float c) {
        return EXACT ? x86_nan3(__fmaf_rn(a, b, c), a, b, c) : __fmaf_rn(a, b, c);
    }
    // Fast keeps "NaN in, NaN out" (any payload) so the exact recompute triggers.
    static __device__ __forceinline__ float clamp(float v, float lo, float hi) {
        return EXACT ? clamp_rs(v, lo, hi) : (v < lo ? lo : (v > hi ? hi : v));
    }
};

template <>
struct Arith<kHalf> {
    static constexpr bool EXACT = false;
    static __device__ __forceinline__ float add(float a, float b) { return __fadd_rn(a, b); }
    static __device__ __forceinline__ float sub(float a, float b) { return __fsub_rn(a, b); }
    static __device__ __forceinline__ float mul(float a, float b) { return __fmul_rn(a, b); }
    static __device__ __forceinline__ float div(float a, float b) { return __fdividef(a, b); }
    static __device__ __forceinline__ float tdiv(float a, float b) { return __fdividef(a, b); }
    static __device__ __forceinline__ float exp(float x) { return __expf(x); }
    static __device__ __forceinline__ float exp_gate(float x) { return __expf(x); }
    static __device__ __forceinline__ float expm1(float x) { return expm1_32(x); }
    static __device__ __forceinline__ float tanh(float x) {
        const float ay = fabsf(x);
        const float t = __fsub_rn(1.0f, __fdividef(2.0f, __fadd_rn(__expf(__fmul_rn(2.0f, ay)), 1.0f)));
        const float r = ay >= 10.0f ? 1.0f : t;
        return x == 0.0f ? x : (x < 0.0f ? -r : r);
    }
    static __device__ __forceinline__ float tanh_op(float x) { return tanh32(x); }
    static __device__ __forceinline__ float log1p(float x) { return (float)::log1p((double)x); }
    static __device__ __forceinline__ float round_f16(float v) { return __half2float(__float2half_rn(v)); }
    static __device__ __forceinline__ float fma(float a, float b, float c) { return __fmaf_rn(a, b, c); }
    static __device__ __forceinline__ float clamp(float v, float lo, float hi) {
        return v < lo ? lo : (v > hi ? hi : v);
    }
};

// GELU's tanh approximation of an already binary16-rounded input q
// (unary.rs:533-539, between the two binary16 round trips).
template <int MODE>
__device__ __forceinline__ float gelu_tanh_core(float q) {
    using A = Arith<MODE>;
    const float cube = A::mul(A::mul(A::mul(0.044715f, q), q), q);
    const float inner = A::mul(0.7978846f, A::add(q, cube));
    return A::mul(A::mul(0.5f, q), A::add(1.0f, A::tanh(inner)));
}

template <int OP, int MODE, bool IN_F16 = false>
__device__ __forceinline__ float unary_formula(float v, UnaryParams p) {
    using A = Arith<MODE>;
    constexpr bool EXACT = MODE == kExact;
    if constexpr (OP == kAbs) return f_abs(v);
    if constexpr (OP == kSgn) return is_nan(v) ? bitsf(0x7fc00000u) : bitsf((fbits(v) & 0x80000000u) | 0x3f800000u);
    if constexpr (OP == kNeg) return f_neg(v);
    if constexpr (OP == kStep) return v > 0.0f ? 1.0f : 0.0f;
    if constexpr (OP == kTanh) return A::tanh_op(v);
    if constexpr (OP == kElu) return v >= 0.0f ? v : A::expm1(v);
    if constexpr (OP == kRelu) return v > 0.0f ? v : 0.0f;
    if constexpr (OP == kSigmoid) return A::tdiv(1.0f, A::add(1.0f, A::exp_gate(f_neg(v))));
    if constexpr (OP == kGelu) {
        if (v <= -10.0f) return 0.0f;
        if (v >= 10.0f) return v;
        // an f16 input is already binary16, and an f16 store rounds the
        // output the same way: the fast path skips both round trips
        const float q = (IN_F16 && !EXACT) ? v : A::round_f16(v);
        const float approx = gelu_tanh_core<MODE>(q);
        return (IN_F16 && !EXACT) ? approx : A::round_f16(approx);
    }
    if constexpr (OP == kGeluGeneric) {
        // generic.rs:1330-1337: no binary16 rounding (the "rounded" value is
        // the input's own bits), no +-10 clamp, and the cubic term fused:
        // 0.5 * v * (1 + tanh(0.7978846 * fma(0.044715 * v * v, v, v)))
        const float cubic = A::fma(A::mul(A::mul(0.044715f, v), v), v, v);
        return A::mul(A::mul(0.5f, v), A::add(1.0f, A::tanh(A::mul(0.7978846f, cubic))));
    }
    if constexpr (OP == kGeluQuick) {
        const float inner = A::mul(A::mul(0.7978846f, v), A::add(1.0f, A::mul(A::mul(0.044715f, v), v)));
        return A::mul(A::mul(0.5f, v), A::add(1.0f, A::tanh(inner)));
    }
    if constexpr (OP == kSilu) return A::tdiv(v, A::add(1.0f, A::exp_gate(f_neg(v))));
    if constexpr (OP == kHardswish) return A::div(A::mul(v, A::clamp(A::add(v, 3.0f), 0.0f, 6.0f)), 6.0f);
    if constexpr (OP == kHardsigmoid) return A::div(A::clamp(A::add(v, 3.0f), 0.0f, 6.0f), 6.0f);
    if constexpr (OP == kExp) return A::exp(v);
    if constexpr (OP == kExpm1) return A::expm1(v);
    if constexpr (OP == kSoftplus) return A::log1p(A::exp(v));
    if constexpr (OP == kGeluErf) {
        const float sign = v < 0.0f ? -1.0f : 1.0f;
        const float x = A::div(f_abs(v), 1.41421356237309504880f);
        const float t = A::div(1.0f, A::add(1.0f, A::mul(0.3275911f, x)));
        float poly = A::sub(A::mul(1.0614054f, t), 1.4531521f);
        poly = A::add(A::mul(poly, t), 1.4214138f);
        poly = A::sub(A::mul(poly, t), 0.28449672f);
        poly = A::add(A::mul(poly, t), 0.2548296f);
        poly = A::mul(poly, t);
        const float erf = A::mul(sign, A::sub(1.0f, A::mul(poly, A::exp(A::mul(f_neg(x), x)))));
        return A::mul(A::mul(0.5f, v), A::add(1.0f, erf));
    }
    if constexpr (OP == kFloor) return x86_nan1(floorf(v), v);
    if constexpr (OP == kCeil) return x86_nan1(ceilf(v), v);
    if constexpr (OP == kRound) return x86_nan1(roundf(v), v);
    if constexpr (OP == kTrunc) return x86_nan1(truncf(v), v);
    if constexpr (OP == kSqr) return f_mul(v, v);
    if constexpr (OP == kSqrt) return f_sqrt(v);
    if constexpr (OP == kLog) return lm_log(v);
    if constexpr (OP == kSin) return lm_sin(v);
    if constexpr (OP == kCos) return lm_cos(v);
    if constexpr (OP == kScale) return f_mul(v, p.a);
    if constexpr (OP == kClamp) return clamp_rs(v, p.a, p.b);
    if constexpr (OP == kLeakyRelu) return is_nan(v) ? v : (v < 0.0f ? f_mul(v, p.a) : v);
    if constexpr (OP == kAdd1) return f_add(v, p.a);
    if constexpr (OP == kCopy) return v;
    return v;
}

// Pair forms of heavy formulas on binary32 storage: the fast pass of
// unary_formula (kFast policy; GELU's kHalf) on two elements, lane for lane
// the scalar formula's operations with the binary32 multiplies, adds and
// FMAs packed two to an instruction (exp32x2, div_refined2), so each lane
// has the scalar pass's bits.  CUDA's own intrinsics (__expf, __fdividef)
// are still called per lane.
template <int OP>
constexpr bool kPairFormula = OP == kSilu || OP == kSigmoid || OP == kExp || OP == kGelu;

template <int OP>
__device__ __forceinline__ float2 unary_formula2(float2 v) {
    if constexpr (OP == kExp) return exp32x2(v);
    if constexpr (OP == kSilu || OP == kSigmoid) {
        const float2 d = __fadd2_rn(splat2(1.0f), exp32x2<true>(make_float2(f_neg(v.x), f_neg(v.y))));
        return div_refined2(OP == kSilu ? v : splat2(1.0f), d);
    }
    if constexpr (OP == kGelu) {
        // unary_formula<kGelu, kHalf>: q = v through binary16, the tanh
        // approximation, the result through binary16, +-10 clamps last
        const float2 q = __half22float2(__floats2half2_rn(v.x, v.y));
        const float2 cube = __fmul2_rn(__fmul2_rn(__fmul2_rn(splat2(0.044715f), q), q), q);
        const float2 inner = __fmul2_rn(splat2(0.7978846f), __fadd2_rn(q, cube));
        const float2 ay = make_float2(fabsf(inner.x), fabsf(inner.y));
        const float2 d = __fadd2_rn(make_float2(__expf(__fmul_rn(2.0f, ay.x)), __expf(__fmul_rn(2.0f, ay.y))),
                                    splat2(1.0f));
        const float2 t = __fadd2_rn(splat2(1.0f), make_float2(-__fdividef(2.0f, d.x), -__fdividef(2.0f, d.y)));
        const float rx = ay.x >= 10.0f ? 1.0f : t.x, ry = ay.y >= 10.0f ? 1.0f : t.y;
        const float2 th = make_float2(inner.x == 0.0f ? inner.x : (inner.x < 0.0f ? -rx : rx),
                                      inner.y == 0.0f ? inner.y : (inner.y < 0.0f ? -ry : ry));
        const float2 g = __fmul2_rn(__fmul2_rn(splat2(0.5f), q), __fadd2_rn(splat2(1.0f), th));
        const float2 o = __half22float2(__floats2half2_rn(g.x, g.y));
        return make_float2(v.x <= -10.0f ? 0.0f : (v.x >= 10.0f ? v.x : o.x),
                           v.y <= -10.0f ? 0.0f : (v.y >= 10.0f ? v.y : o.y));
    }
    return v;
}

template <int OP>
constexpr bool kHeavyFormula = OP == kTanh || OP == kElu || OP == kSigmoid || OP == kGelu || OP == kGeluQuick ||
                               OP == kGeluGeneric ||
                               OP == kSilu || OP == kHardswish || OP == kHardsigmoid || OP == kExp || OP == kExpm1 ||
                               OP == kSoftplus || OP == kGeluErf;

// The exact (NaN-payload) recompute is rare; keeping it out of line keeps
// the hot loop small.
template <int OP, bool IN_F16>
__device__ __noinline__ float unary_exact_slow(float v, UnaryParams p) {
    return unary_formula<OP, kExact, IN_F16>(v, p);
}

// IN_F16: the value came from, and the result goes to, binary16 storage.
// Results that end in binary16 (binary16 storage; GELU, which rounds its
// output through binary16 itself) take the kHalf policy.
template <int OP, bool IN_F16 = false>
__device__ __forceinline__ float unary_apply(float v, UnaryParams p) {
    if constexpr (kHeavyFormula<OP>) {
        constexpr int M = (IN_F16 || OP == kGelu) ? kHalf : kFast;
        const float r = unary_formula<OP, M, IN_F16>(v, p);
        if (!is_nan(r)) return r;
        return unary_exact_slow<OP, IN_F16>(v, p);
    } else {
        return unary_formula<OP, kExact, IN_F16>(v, p);
    }
}

// ---------------------------------------------------------------------------
// Gated linear units (glu.rs:99-127, 264-277): out = value * gate(g).
// Rust's f32::max(0.0) / f32::min(7.0) against a constant compile on x86-64
// to maxss / minss with the constant as the second operand, which returns
// that constant for a NaN input and for a tie: relu(-0.0) = +0.0.
// ---------------------------------------------------------------------------
template <int MODE>
__device__ __forceinline__ float glu_silu(float v) {
    using A = Arith<MODE>;
    return A::tdiv(v, A::add(1.0f, A::exp_gate(f_neg(v))));
}

template <int SUB, int MODE>
__device__ __forceinline__ float glu_formula(float value, float g) {
    using A = Arith<MODE>;
    if constexpr (SUB == kReGlu) return A::mul(value, g > 0.0f ? g : 0.0f);
    if constexpr (SUB == kGeGlu) return A::mul(value, unary_formula<kGeluQuick, MODE>(g, UnaryParams{}));
    if constexpr (SUB == kSwiGlu) return A::mul(value, glu_silu<MODE>(g));
    if constexpr (SUB == kSwiGluOai) {
        const float gate = g < 7.0f ? g : 7.0f;
        const float v = value < 7.0f ? value : 7.0f;
        return A::mul(A::div(glu_silu<MODE>(A::mul(1.702f, gate)), 1.702f), A::add(v, 1.0f));
    }
    if constexpr (SUB == kGeGluErf) return A::mul(value, unary_formula<kGeluErf, MODE>(g, UnaryParams{}));
    // kGeGluQuick: value * (1 / (1 + exp(-1.702 * g)))
    return A::mul(value, A::tdiv(1.0f, A::add(1.0f, A::exp_gate(A::mul(-1.702f, g)))));
}

// Pair forms of the exp-based gates (kFast policy), lane for lane the
// scalar glu_formula's operations with the binary32 ones packed.
template <int SUB>
constexpr bool kGluPairFormula = SUB == kSwiGlu || SUB == kSwiGluOai || SUB == kGeGluQuick;

__device__ __forceinline__ float2 glu_silu2(float2 v) {
    return div_refined2(v, __fadd2_rn(splat2(1.0f), exp32x2<true>(make_float2(f_neg(v.x), f_neg(v.y)))));
}

template <int SUB>
__device__ __forceinline__ float2 glu_formula2(float2 value, float2 g) {
    if constexpr (SUB == kSwiGlu) return __fmul2_rn(value, glu_silu2(g));
    if constexpr (SUB == kSwiGluOai) {
        const float2 gate = make_float2(g.x < 7.0f ? g.x : 7.0f, g.y < 7.0f ? g.y : 7.0f);
        const float2 v = make_float2(value.x < 7.0f ? value.x : 7.0f, value.y < 7.0f ? value.y : 7.0f);
        const float2 s = glu_silu2(__fmul2_rn(splat2(1.702f), gate));
        return __fmul2_rn(make_float2(__fdiv_rn(s.x, 1.702f), __fdiv_rn(s.y, 1.702f)), __fadd2_rn(v, splat2(1.0f)));
    }
    if constexpr (SUB == kGeGluQuick)
        return __fmul2_rn(value, div_refined2(splat2(1.0f), __fadd2_rn(splat2(1.0f),
                                                                     exp32x2<true>(__fmul2_rn(splat2(-1.702f), g)))));
    return value;
}

template <int SUB>
__device__ __noinline__ float glu_exact_slow(float value, float g) {
    return glu_formula<SUB, kExact>(value, g);
}

template <int SUB>
__device__ __forceinline__ float glu_apply(float value, float g) {
    const float r = glu_formula<SUB, kFast>(value, g);
    if (!is_nan(r)) return r;
    return glu_exact_slow<SUB>(value, g);
}

// ---------------------------------------------------------------------------
// Element access for the two floating storage types.
// ---------------------------------------------------------------------------
template <typename T>
struct Elem;

template <>
struct Elem<float> {
    static __device__ __forceinline__ float load(const float* p) { return *p; }
    static __device__ __forceinline__ void store(float* p, float v) { *p = v; }
};

template <>
struct Elem<uint16_t> {
    static __device__ __forceinline__ float load(const uint16_t* p) { return f16_bits_to_f32(*p); }
    static __device__ __forceinline__ void store(uint16_t* p, float v) { *p = f32_to_f16_bits(v); }
};

// 16-byte vector of T.
template <typename T>
struct alignas(16) Vec16 {
    static constexpr int N = 16 / sizeof(T);
    T v[N];
};

// binary16 lanes held as four 32-bit words (lane 2i in the low half of word
// i): the vector stays in four registers from the load to the store instead
// of being split into eight 16-bit values and packed again.
template <>
struct alignas(16) Vec16<uint16_t> {
    static constexpr int N = 8;
    uint32_t w[4];
};

template <typename T>
__device__ __forceinline__ Vec16<T> ld_stream(const T* p) {
    Vec16<T> r;
    uint4 u;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(u.x), "=r"(u.y), "=r"(u.z), "=r"(u.w)
                 : "l"(p));
    *reinterpret_cast<uint4*>(&r) = u;
    return r;
}

template <typename T>
__device__ __forceinline__ Vec16<T> ld_keep(const T* p) {
    Vec16<T> r;
    *reinterpret_cast<uint4*>(&r) = __ldg(reinterpret_cast<const uint4*>(p));
    return r;
}

template <typename T>
__device__ __forceinline__ void st_stream(T* p, const Vec16<T>& v) {
    const uint4 u = *reinterpret_cast<const uint4*>(&v);
    asm volatile("st.global.L1::no_allocate.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(u.x), "r"(u.y), "r"(u.z),
                 "r"(u.w)
                 : "memory");
}

__device__ __forceinline__ float vget(const Vec16<float>& v, int i) { return v.v[i]; }
__device__ __forceinline__ float vget(const Vec16<uint16_t>& v, int i) {
    return f16_bits_to_f32((uint16_t)(v.w[i >> 1] >> (16 * (i & 1))));
}
__device__ __forceinline__ void vset(Vec16<float>& v, int i, float x) { v.v[i] = x; }
__device__ __forceinline__ void vset(Vec16<uint16_t>& v, int i, float x) {
    const int sh = 16 * (i & 1);
    v.w[i >> 1] = (v.w[i >> 1] & ~(0xffffu << sh)) | ((uint32_t)f32_to_f16_bits(x) << sh);
}

// 32-bit unsigned division by a run-time constant (round-up multiply-shift,
// Granlund-Montgomery), used to decode logical ordinals into coordinates.
struct FastDiv {
    uint32_t d;
    uint32_t mul;
    uint32_t shift;
};

__host__ __device__ inline FastDiv make_fastdiv(uint32_t d) {
    FastDiv f{d, 0, 0};
    if (d <= 1) return f;
    uint32_t s = 0;
    while ((1ull << s) < d) ++s;
    f.shift = s;
    f.mul = (uint32_t)(((1ull << 32) * ((1ull << s) - d)) / d + 1);
    return f;
}

__device__ __forceinline__ uint32_t fdiv(uint32_t n, const FastDiv& f) {
    if (f.d == 1) return n;
    const uint32_t t = __umulhi(n, f.mul);
    return (t + ((n - t) >> 1)) >> (f.shift - 1);
}

}  // namespace emel
