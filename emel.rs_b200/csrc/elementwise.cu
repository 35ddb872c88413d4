// Elementwise kernels: unary, binary, row broadcast and repeat broadcast.
//
// All of them are HBM-streaming: one read of each input element, one write
// of each output element.  Four shapes of the same loop body:
//   ew_flat    dense operands with identical extents: a grid-stride stream
//              of 16-byte vectors (4 x f32 / 8 x f16), two in flight per
//              thread, loads marked no-allocate in L1, one resident wave of
//              CTAs;
//   ew_rows    every operand has unit stride in dim0: "row workers" of G
//              threads (a warp for short rows, a whole CTA for long ones)
//              walk rows of the iteration space, 16-byte vectors within a
//              row.  This covers row broadcast (src1 = one row), the ggml
//              repeat broadcast and permuted / padded views whose rows are
//              contiguous (e.g. dims 1 and 2 swapped);
//   ew_generic arbitrary strides: one element per thread, coordinates
//              decoded from the ordinal with 32-bit fast division;
//   ew_ordinal equal element counts with different extents: every operand
//              decodes the ordinal with its own extents (binary.rs:411-424).
// Grids are sized in multiples of the SM count (148 on B200).
#include <type_traits>

#include "common.cuh"
#include "launch.hpp"
#include "pdl.cuh"
#include "tma.cuh"

namespace emel {

namespace {

constexpr int kThreads = 256;

// Formula functors.  operator() is the full per-element evaluation (a fast
// pass and, for a NaN result, the exact recompute with the x86 NaN rules);
// fast() is the fast pass alone, for vector paths that check a whole vector
// for NaN results and redo only such vectors lane by lane (kHeavy: the
// formula has a separate fast pass).
template <int OP, bool IN_F16>
struct UnaryFn {
    UnaryParams p;
    static constexpr bool kBinary = false;
    static constexpr bool kHeavy = kHeavyFormula<OP>;
    // two vectors in flight per thread; with 32-bit indexing most ops fit 32
    // registers without spilling (eight CTAs, 2048 threads per SM), the
    // longer formulas 51
    static constexpr int kUnroll = 2;
    static constexpr int kMinBlocks = (OP == kTanh || OP == kExpm1 || OP == kSoftplus || OP == kGeluErf) ? 5 : 8;
    __device__ __forceinline__ float operator()(float a, float) const { return unary_apply<OP, IN_F16>(a, p); }
    __device__ __forceinline__ float fast(float a, float) const {
        if constexpr (kHeavy) return unary_formula<OP, (IN_F16 || OP == kGelu) ? kHalf : kFast, IN_F16>(a, p);
        else return unary_apply<OP, IN_F16>(a, p);
    }
    // fast() on two binary32 elements at once (same bits per lane)
    static constexpr bool kPair = !IN_F16 && kPairFormula<OP>;
    __device__ __forceinline__ float2 fast2(float2 a, float2) const { return unary_formula2<OP>(a); }
    // binary16 ops computed on two packed lanes, bit for bit the reference's
    // f16 -> f32 -> op -> f16 for NaN-free inputs: sign-bit operations, the
    // signed 16-bit compare (positive binary16 values are exactly the lanes
    // > 0 as int16), and x * x, exact in binary32 and rounded once either way
    static constexpr bool kPacked = IN_F16 && (OP == kAbs || OP == kNeg || OP == kRelu || OP == kStep || OP == kSqr);
    static constexpr bool kPackedMayNan = false;
    __device__ __forceinline__ uint32_t packed(uint32_t w, uint32_t) const {
        if constexpr (OP == kAbs) return w & 0x7fff7fffu;
        if constexpr (OP == kNeg) return w ^ 0x80008000u;
        if constexpr (OP == kRelu) return w & __vcmpgts2(w, 0u);
        if constexpr (OP == kStep) return __vcmpgts2(w, 0u) & 0x3c003c00u;
        if constexpr (OP == kSqr) {
            const __half2 h = *reinterpret_cast<const __half2*>(&w);
            const __half2 r = __hmul2(h, h);
            return *reinterpret_cast<const uint32_t*>(&r);
        }
        return w;
    }
};

template <int OP>
struct BinaryFn {
    static constexpr bool kBinary = true;
    static constexpr bool kHeavy = false;
    static constexpr int kUnroll = 2;
    static constexpr int kMinBlocks = 6;  // two operands of two vectors each: 40 registers
    __device__ __forceinline__ float operator()(float a, float b) const { return binary_apply<OP>(a, b); }
    __device__ __forceinline__ float fast(float a, float b) const { return binary_apply<OP>(a, b); }
    // binary16 multiply on packed lanes: the product of two binary16 values
    // is exact in binary32, so one binary16 rounding either way; 0 * inf
    // gives a NaN whose encoding the lane path supplies
    static constexpr bool kPacked = OP == kMul;
    static constexpr bool kPackedMayNan = true;
    __device__ __forceinline__ uint32_t packed(uint32_t wa, uint32_t wb) const {
        const __half2 r = __hmul2(*reinterpret_cast<const __half2*>(&wa), *reinterpret_cast<const __half2*>(&wb));
        return *reinterpret_cast<const uint32_t*>(&r);
    }
};

// activation.rs:467-481, silu_back as a two-input formula: grad * silu'(x).
struct SiluBackFn {
    static constexpr bool kBinary = true;
    static constexpr bool kHeavy = false;
    static constexpr int kUnroll = 2;
    static constexpr int kMinBlocks = 4;
    __device__ __forceinline__ float operator()(float x, float grad) const {
        const float sigmoid = f_div(1.0f, f_add(1.0f, lm_exp_cr(f_neg(x))));
        const float derivative = f_mul(sigmoid, f_add(1.0f, f_mul(x, f_sub(1.0f, sigmoid))));
        return f_mul(grad, derivative);
    }
};

// glu.rs: (value, gate) pairs from the two halves of the input.
template <int SUB>
struct GluFn {
    static constexpr bool kBinary = true;
    static constexpr bool kHeavy = SUB != kReGlu;
    static constexpr int kUnroll = SUB == kReGlu ? 4 : 2;
    static constexpr int kMinBlocks = 3;
    __device__ __forceinline__ float operator()(float value, float g) const { return glu_apply<SUB>(value, g); }
    __device__ __forceinline__ float fast(float value, float g) const {
        if constexpr (kHeavy) return glu_formula<SUB, kFast>(value, g);
        else return glu_apply<SUB>(value, g);
    }
    // fast() on two (value, gate) pairs at once (same bits per lane)
    static constexpr bool kPair = kGluPairFormula<SUB>;
    __device__ __forceinline__ float2 fast2(float2 value, float2 g) const { return glu_formula2<SUB>(value, g); }
};

// Per-lane path (binary16 vectors with a NaN in or out take it rarely; f32
// vectors always).  Out of line for binary16 so the packed loop stays small.
template <typename T, typename F>
__device__ __noinline__ Vec16<T> apply_vec_lanes(const F& f, const Vec16<T>& a, const Vec16<T>& b) {
    Vec16<T> r;
#pragma unroll
    for (int k = 0; k < Vec16<T>::N; ++k) vset(r, k, f(vget(a, k), F::kBinary ? vget(b, k) : 0.0f));
    return r;
}

// Functors with a pair form of their fast pass (kPair, fast2).
template <typename F, typename = void>
struct PairOp : std::false_type {};
template <typename F>
struct PairOp<F, std::void_t<decltype(F::kPair)>> : std::bool_constant<F::kPair> {};

template <typename T, typename F>
__device__ __forceinline__ Vec16<T> apply_vec_scalar(const F& f, const Vec16<T>& a, const Vec16<T>& b) {
    if constexpr (sizeof(T) == 2) {
        return apply_vec_lanes<T>(f, a, b);
    } else if constexpr (F::kHeavy) {
        // fast pass on every lane (in pairs where the formula has a pair
        // form); a vector with a NaN result is redone lane by lane with the
        // exact recompute (one out-of-line call site)
        Vec16<T> r;
        bool nan_out = false;
        if constexpr (PairOp<F>::value) {
#pragma unroll
            for (int k = 0; k < Vec16<T>::N; k += 2) {
                const float2 x = make_float2(vget(a, k), vget(a, k + 1));
                const float2 y = F::kBinary ? make_float2(vget(b, k), vget(b, k + 1)) : make_float2(0.0f, 0.0f);
                const float2 v = f.fast2(x, y);
                nan_out |= is_nan(v.x) | is_nan(v.y);
                vset(r, k, v.x);
                vset(r, k + 1, v.y);
            }
        } else {
#pragma unroll
            for (int k = 0; k < Vec16<T>::N; ++k) {
                const float v = f.fast(vget(a, k), F::kBinary ? vget(b, k) : 0.0f);
                nan_out |= is_nan(v);
                vset(r, k, v);
            }
        }
        if (nan_out) return apply_vec_lanes<T>(f, a, b);
        return r;
    } else {
        Vec16<T> r;
#pragma unroll
        for (int k = 0; k < Vec16<T>::N; ++k) vset(r, k, f(vget(a, k), F::kBinary ? vget(b, k) : 0.0f));
        return r;
    }
}

// True when any of the eight binary16 lanes of `v` is a NaN.
__device__ __forceinline__ bool any_nan_h8(const Vec16<uint16_t>& v) {
    const uint4 u = *reinterpret_cast<const uint4*>(&v);
    const unsigned m = __vcmpgtu2(u.x & 0x7fff7fffu, 0x7c007c00u) | __vcmpgtu2(u.y & 0x7fff7fffu, 0x7c007c00u) |
                       __vcmpgtu2(u.z & 0x7fff7fffu, 0x7c007c00u) | __vcmpgtu2(u.w & 0x7fff7fffu, 0x7c007c00u);
    return m != 0;
}

// Functors with a packed binary16 form (kPacked).
template <typename F, typename = void>
struct PackedOp : std::false_type {};
template <typename F>
struct PackedOp<F, std::void_t<decltype(F::kPacked)>> : std::bool_constant<F::kPacked> {};

template <typename T, typename F>
__device__ __forceinline__ Vec16<T> apply_vec(const F& f, const Vec16<T>& a, const Vec16<T>& b) {
    if constexpr (sizeof(T) == 2) {
        // binary16: NaN-free vectors convert lanes in pairs (cvt.f32.f16 /
        // cvt.rn.f16x2.f32); any NaN in or out takes the per-lane path that
        // applies the reference's NaN encodings.
        if (!any_nan_h8(a) && !(F::kBinary && any_nan_h8(b))) {
            const uint4 ua = *reinterpret_cast<const uint4*>(&a);
            const uint4 ub = *reinterpret_cast<const uint4*>(&b);
            if constexpr (PackedOp<F>::value) {
                Vec16<T> r;
                *reinterpret_cast<uint4*>(&r) = make_uint4(f.packed(ua.x, ub.x), f.packed(ua.y, ub.y),
                                                           f.packed(ua.z, ub.z), f.packed(ua.w, ub.w));
                if (!F::kPackedMayNan || !any_nan_h8(r)) return r;
                return apply_vec_lanes<T>(f, a, b);
            }
            const unsigned wa[4] = {ua.x, ua.y, ua.z, ua.w};
            const unsigned wb[4] = {ub.x, ub.y, ub.z, ub.w};
            unsigned wr[4];
            bool nan_out = false;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float2 xa = __half22float2(*reinterpret_cast<const __half2*>(&wa[k]));
                float2 xb = make_float2(0.0f, 0.0f);
                if constexpr (F::kBinary) xb = __half22float2(*reinterpret_cast<const __half2*>(&wb[k]));
                const float r0 = f.fast(xa.x, xb.x);
                const float r1 = f.fast(xa.y, xb.y);
                nan_out |= is_nan(r0) | is_nan(r1);
                const __half2 h = __floats2half2_rn(r0, r1);
                wr[k] = *reinterpret_cast<const unsigned*>(&h);
            }
            if (!nan_out) {
                Vec16<T> r;
                *reinterpret_cast<uint4*>(&r) = make_uint4(wr[0], wr[1], wr[2], wr[3]);
                return r;
            }
        }
    }
    return apply_vec_scalar<T>(f, a, b);
}

// I: the index type -- 32-bit when the vector count and the grid stride
// leave headroom below 2^31 (every realistic tensor), which keeps the loop's
// registers low enough for eight CTAs per SM on the cheap ops.
//
// early: the inputs do not overlap anything the previous kernel on the
// stream writes (the host's stream record), so each thread issues its first
// batch of loads before waiting for that kernel (pdl_enter); stores always
// come after the wait.  Under programmatic dependent launch the CTAs start
// while the previous kernel drains, and these loads overlap its tail.
template <typename T, typename F, typename I>
__device__ __forceinline__ void flat_load(const T* __restrict__ a, const T* __restrict__ b, I at, I stride,
                                          Vec16<T> (&a0)[F::kUnroll], Vec16<T> (&b0)[F::kUnroll]) {
#pragma unroll
    for (int k = 0; k < F::kUnroll; ++k) {
        a0[k] = ld_stream(a + (uint64_t)(at + k * stride) * Vec16<T>::N);
        if constexpr (F::kBinary) b0[k] = ld_stream(b + (uint64_t)(at + k * stride) * Vec16<T>::N);
        else b0[k] = Vec16<T>{};
    }
}

template <typename T, typename F, typename I>
__device__ __forceinline__ void flat_store(T* __restrict__ dst, I at, I stride, const F& f,
                                           const Vec16<T> (&a0)[F::kUnroll], const Vec16<T> (&b0)[F::kUnroll]) {
#pragma unroll
    for (int k = 0; k < F::kUnroll; ++k)
        st_stream(dst + (uint64_t)(at + k * stride) * Vec16<T>::N, apply_vec<T>(f, a0[k], b0[k]));
}

template <typename T, typename F, typename I>
__global__ void __launch_bounds__(kThreads, F::kMinBlocks) ew_flat(T* __restrict__ dst, const T* __restrict__ a,
                                                    const T* __restrict__ b, uint64_t n, F f, int early) {
    constexpr int N = Vec16<T>::N;
    constexpr int U = F::kUnroll;  // vectors in flight per thread
    const I nvec = (I)(n / N);
    const I stride = (I)gridDim.x * blockDim.x;
    const I gid = (I)blockIdx.x * blockDim.x + threadIdx.x;
    I i = gid;
    if (early && i + (U - 1) * stride < nvec) {
        Vec16<T> a0[U], b0[U];
        flat_load<T, F, I>(a, b, i, stride, a0, b0);
        pdl_enter();
        flat_store<T, F, I>(dst, i, stride, f, a0, b0);
        i += U * stride;
    } else {
        pdl_enter();
    }
    for (; i + (U - 1) * stride < nvec; i += U * stride) {
        Vec16<T> a0[U], b0[U];
        flat_load<T, F, I>(a, b, i, stride, a0, b0);
        flat_store<T, F, I>(dst, i, stride, f, a0, b0);
    }
    if (i < nvec) {
        // this thread's last (fewer than U) vectors, their loads issued together
        Vec16<T> a0[U], b0[U];
#pragma unroll
        for (int k = 0; k < U; ++k) {
            a0[k] = Vec16<T>{};
            b0[k] = Vec16<T>{};
            if (i + k * stride < nvec) {
                a0[k] = ld_stream(a + (uint64_t)(i + k * stride) * N);
                if constexpr (F::kBinary) b0[k] = ld_stream(b + (uint64_t)(i + k * stride) * N);
            }
        }
#pragma unroll
        for (int k = 0; k < U; ++k)
            if (i + k * stride < nvec) st_stream(dst + (uint64_t)(i + k * stride) * N, apply_vec<T>(f, a0[k], b0[k]));
    }
    const uint64_t t = (uint64_t)nvec * N + gid;
    if (t < n) {
        const float x = Elem<T>::load(a + t);
        const float y = F::kBinary ? Elem<T>::load(b + t) : 0.0f;
        Elem<T>::store(dst + t, f(x, y));
    }
}

template <typename T>
__device__ __forceinline__ T* at(const Operand& o, int64_t elems) {
    return reinterpret_cast<T*>(o.ptr) + elems;
}

// Row workers: G = 1 << gshift threads per row.
template <typename T, typename F>
__global__ void __launch_bounds__(kThreads) ew_rows(EwPlan p, F f, int gshift) {
    pdl_enter();
    constexpr int N = Vec16<T>::N;
    const uint32_t G = 1u << gshift;
    const uint32_t lane = threadIdx.x & (G - 1);
    const uint64_t group = ((uint64_t)blockIdx.x * blockDim.x + threadIdx.x) >> gshift;
    const uint64_t ngroups = ((uint64_t)gridDim.x * blockDim.x) >> gshift;
    const uint64_t ne0 = p.ne[0], ne1 = p.ne[1], ne2 = p.ne[2];
    const uint64_t rows = p.count / ne0;
    const bool col_bcast = F::kBinary && p.src1.ne[0] == 1;
    for (uint64_t r = group; r < rows; r += ngroups) {
        const uint64_t i1 = r % ne1, q = r / ne1, i2 = q % ne2, i3 = q / ne2;
        T* drow = at<T>(p.dst, i1 * p.dst.st[1] + i2 * p.dst.st[2] + i3 * p.dst.st[3]);
        const T* arow = at<T>(p.src0, i1 * p.src0.st[1] + i2 * p.src0.st[2] + i3 * p.src0.st[3]);
        const T* brow = nullptr;
        if constexpr (F::kBinary) {
            const uint64_t j1 = p.src1_bcast ? i1 % p.src1.ne[1] : i1;
            const uint64_t j2 = p.src1_bcast ? i2 % p.src1.ne[2] : i2;
            const uint64_t j3 = p.src1_bcast ? i3 % p.src1.ne[3] : i3;
            brow = at<T>(p.src1, j1 * p.src1.st[1] + j2 * p.src1.st[2] + j3 * p.src1.st[3]);
        }
        if (p.vec && !col_bcast) {
            const uint64_t nv = ne0 / N;
            for (uint64_t c = lane; c < nv; c += G) {
                const Vec16<T> a0 = ld_stream(arow + c * N);
                Vec16<T> b0{};
                if constexpr (F::kBinary) b0 = ld_keep(brow + c * N);
                st_stream(drow + c * N, apply_vec<T>(f, a0, b0));
            }
        } else {
            for (uint64_t c = lane; c < ne0; c += G) {
                const float x = Elem<T>::load(arow + c);
                float y = 0.0f;
                if constexpr (F::kBinary) y = Elem<T>::load(brow + (col_bcast ? 0 : (int64_t)(c % p.src1.ne[0]) * p.src1.st[0]));
                Elem<T>::store(drow + c, f(x, y));
            }
        }
    }
}

// Vector walk over rows whose every operand has unit dim-0 stride and
// 16-byte aligned starts (row broadcast, the repeat broadcast, permuted or
// padded views): grid-stride over the 16-byte vectors of the logical order,
// U independent vectors per thread per iteration; each vector's row and the
// broadcast operand's wrapped row come from 32-bit magic-number divisions.
struct RowsWalk {
    FastDiv dv, d1, d2;  // vectors per row, ne1, ne2
    FastDiv m1, m2, m3;  // src1 extents (broadcast wrap)
    uint32_t vpr, ne1, ne2;
    uint32_t nvec;
};

// No early loads here: holding the first batch across the wait, or
// prefetching it into L2 before the wait, both measured slower on this
// kernel than waiting first (359 vs 363 us on cfg5's full repeat).
template <typename T, typename F>
__global__ void __launch_bounds__(kThreads) ew_rows_vec(EwPlan p, F f, RowsWalk w) {
    constexpr int N = Vec16<T>::N;
    constexpr int U = 4;
    const uint32_t stride = gridDim.x * blockDim.x;
    pdl_enter();
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < w.nvec; i += U * stride) {
        Vec16<T> a[U], b[U];
        T* d[U];
#pragma unroll
        for (int k = 0; k < U; ++k) {
            const uint32_t v = i + k * stride;
            d[k] = nullptr;
            if (v >= w.nvec) continue;
            const uint32_t row = fdiv(v, w.dv), c = (v - row * w.vpr) * N;
            const uint32_t q = fdiv(row, w.d1), i1 = row - q * w.ne1;
            const uint32_t i3 = fdiv(q, w.d2), i2 = q - i3 * w.ne2;
            d[k] = at<T>(p.dst, (int64_t)i1 * p.dst.st[1] + (int64_t)i2 * p.dst.st[2] + (int64_t)i3 * p.dst.st[3]) + c;
            a[k] = ld_stream(at<T>(p.src0, (int64_t)i1 * p.src0.st[1] + (int64_t)i2 * p.src0.st[2] +
                                               (int64_t)i3 * p.src0.st[3]) + c);
            if constexpr (F::kBinary) {
                uint32_t j1 = i1, j2 = i2, j3 = i3;
                if (p.src1_bcast) {
                    j1 = i1 - fdiv(i1, w.m1) * w.m1.d;
                    j2 = i2 - fdiv(i2, w.m2) * w.m2.d;
                    j3 = i3 - fdiv(i3, w.m3) * w.m3.d;
                }
                b[k] = ld_keep(at<T>(p.src1, (int64_t)j1 * p.src1.st[1] + (int64_t)j2 * p.src1.st[2] +
                                                 (int64_t)j3 * p.src1.st[3]) + c);
            } else {
                b[k] = Vec16<T>{};
            }
        }
#pragma unroll
        for (int k = 0; k < U; ++k)
            if (d[k] != nullptr) st_stream(d[k], apply_vec<T>(f, a[k], b[k]));
    }
}

// A dense tensor with one broadcast row (the row-broadcast event,
// broadcast.rs:352-390: src1 ne == [ne0, 1, 1, 1]): vector i of dst and src0
// is i, and src1's vector is i modulo the row's vector count -- one
// magic-number division per vector instead of the row walk's four.
template <typename T, typename F>
__global__ void __launch_bounds__(kThreads) ew_row_broadcast(EwPlan p, F f, FastDiv dv, uint32_t nvec, int early) {
    constexpr int N = Vec16<T>::N;
    constexpr int U = 4;
    const T* a = reinterpret_cast<const T*>(p.src0.ptr);
    const T* b = reinterpret_cast<const T*>(p.src1.ptr);
    T* d = reinterpret_cast<T*>(p.dst.ptr);
    const uint32_t stride = gridDim.x * blockDim.x;
    uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    bool first = early && i < nvec;  // this thread's first batch loads before the wait (as ew_flat's)
    if (!first) pdl_enter();
    for (; i < nvec; i += U * stride) {
        Vec16<T> av[U], bv[U];
#pragma unroll
        for (int k = 0; k < U; ++k) {
            const uint32_t v = i + k * stride;
            if (v >= nvec) continue;
            av[k] = ld_stream(a + (size_t)v * N);
            bv[k] = ld_keep(b + (size_t)(v - fdiv(v, dv) * dv.d) * N);
        }
        if (first) {
            pdl_enter();
            first = false;
        }
#pragma unroll
        for (int k = 0; k < U; ++k) {
            const uint32_t v = i + k * stride;
            if (v < nvec) st_stream(d + (size_t)v * N, apply_vec<T>(f, av[k], bv[k]));
        }
    }
}

// dst and src0 dense (rows of ne0 back to back), src1 a single contiguous row.
bool dense_row_broadcast(const EwPlan& p) {
    if (!p.vec || !p.src1_bcast || p.src1.st[0] != 1) return false;
    if (p.src1.ne[1] != 1 || p.src1.ne[2] != 1 || p.src1.ne[3] != 1 || p.src1.ne[0] != p.ne[0]) return false;
    const uint64_t N = p.dtype == DType::F16 ? 8 : 4;
    if (p.ne[0] % N != 0 || p.count / N >= (1ull << 31) || p.ne[0] / N >= (1ull << 31)) return false;
    const Operand* ops[2] = {&p.dst, &p.src0};
    for (const Operand* o : ops) {
        int64_t expect = 1;
        for (int d = 0; d < 4; ++d) {
            if (p.ne[d] > 1 && o->st[d] != expect) return false;
            expect *= (int64_t)p.ne[d];
        }
    }
    return true;
}

bool rows_walk(const EwPlan& p, RowsWalk* w) {
    const uint64_t N = p.dtype == DType::F16 ? 8 : 4;
    const uint64_t nvec = p.count / N;
    if (!p.vec || p.ne[0] % N != 0 || nvec >= (1ull << 31) || p.ne[1] >= (1ull << 31) || p.ne[2] >= (1ull << 31))
        return false;
    if (p.src1_bcast && p.src1.ne[0] != p.ne[0]) return false;
    w->vpr = (uint32_t)(p.ne[0] / N);
    w->ne1 = (uint32_t)p.ne[1];
    w->ne2 = (uint32_t)p.ne[2];
    w->nvec = (uint32_t)nvec;
    w->dv = make_fastdiv(w->vpr);
    w->d1 = make_fastdiv(w->ne1);
    w->d2 = make_fastdiv(w->ne2);
    const uint64_t b1 = p.src1.ne[1] ? p.src1.ne[1] : 1, b2 = p.src1.ne[2] ? p.src1.ne[2] : 1,
                   b3 = p.src1.ne[3] ? p.src1.ne[3] : 1;
    if (b1 >= (1ull << 31) || b2 >= (1ull << 31) || b3 >= (1ull << 31)) return false;
    w->m1 = make_fastdiv((uint32_t)b1);
    w->m2 = make_fastdiv((uint32_t)b2);
    w->m3 = make_fastdiv((uint32_t)b3);
    return true;
}

template <typename T, typename F>
__global__ void __launch_bounds__(kThreads) ew_generic(EwPlan p, F f, FastDiv d0, FastDiv d1, FastDiv d2) {
    pdl_enter();
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < p.count; i += stride) {
        const uint32_t o = (uint32_t)i;
        const uint32_t q0 = fdiv(o, d0), c0 = o - q0 * d0.d;
        const uint32_t q1 = fdiv(q0, d1), c1 = q0 - q1 * d1.d;
        const uint32_t c3 = fdiv(q1, d2), c2 = q1 - c3 * d2.d;
        const uint32_t c[4] = {c0, c1, c2, c3};
        int64_t od = 0, oa = 0, ob = 0;
#pragma unroll
        for (int d = 0; d < 4; ++d) {
            od += (int64_t)c[d] * p.dst.st[d];
            oa += (int64_t)c[d] * p.src0.st[d];
            if constexpr (F::kBinary) ob += (int64_t)(p.src1_bcast ? c[d] % p.src1.ne[d] : c[d]) * p.src1.st[d];
        }
        const float x = Elem<T>::load(at<T>(p.src0, oa));
        const float y = F::kBinary ? Elem<T>::load(at<T>(p.src1, ob)) : 0.0f;
        Elem<T>::store(at<T>(p.dst, od), f(x, y));
    }
}

__device__ __forceinline__ int64_t ordinal_elems(const Operand& o, uint64_t ordinal) {
    int64_t off = 0;
#pragma unroll
    for (int d = 0; d < 4; ++d) {
        off += (int64_t)(ordinal % o.ne[d]) * o.st[d];
        ordinal /= o.ne[d];
    }
    return off;
}

// src1 of a repeat broadcast: decode with the iteration extents, wrap each
// coordinate into src1's extents (generic.rs:1652-1660).
__device__ __forceinline__ int64_t repeat_elems(const EwPlan& p, uint64_t ordinal) {
    int64_t off = 0;
#pragma unroll
    for (int d = 0; d < 4; ++d) {
        off += (int64_t)((ordinal % p.ne[d]) % p.src1.ne[d]) * p.src1.st[d];
        ordinal /= p.ne[d];
    }
    return off;
}

template <typename T, typename F>
__global__ void __launch_bounds__(kThreads) ew_ordinal(EwPlan p, F f) {
    pdl_enter();
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < p.count; i += stride) {
        const float x = Elem<T>::load(at<T>(p.src0, ordinal_elems(p.src0, i)));
        float y = 0.0f;
        if constexpr (F::kBinary)
            y = Elem<T>::load(at<T>(p.src1, p.src1_bcast ? repeat_elems(p, i) : ordinal_elems(p.src1, i)));
        Elem<T>::store(at<T>(p.dst, ordinal_elems(p.dst, i)), f(x, y));
    }
}

// The generic envelope's repeat (generic.rs:1641-1665): dst ordinal o ->
// coordinates in dst's extents -> each taken modulo src's extent -> src
// element; copied as raw 32-bit words (NaN payloads kept).  32-bit
// magic-number decode when every extent and the count fit, else 64-bit.
struct RepeatArgs {
    FastDiv d0, d1, d2;      // dst extents
    FastDiv m0, m1, m2, m3;  // src extents (modulo)
    bool small;
};

__global__ void __launch_bounds__(kThreads) repeat_copy(EwPlan p, RepeatArgs r) {
    pdl_enter();
    const uint32_t* src = reinterpret_cast<const uint32_t*>(p.src0.ptr);
    uint32_t* dst = reinterpret_cast<uint32_t*>(p.dst.ptr);
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    for (uint64_t i = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; i < p.count; i += stride) {
        uint64_t c[4];
        if (r.small) {
            const uint32_t o = (uint32_t)i;
            const uint32_t q0 = fdiv(o, r.d0), q1 = fdiv(q0, r.d1), q2 = fdiv(q1, r.d2);
            c[0] = o - q0 * r.d0.d;
            c[1] = q0 - q1 * r.d1.d;
            c[2] = q1 - q2 * r.d2.d;
            c[3] = q2;
        } else {
            uint64_t o = i;
            for (int d = 0; d < 4; ++d) {
                c[d] = o % p.ne[d];
                o /= p.ne[d];
            }
        }
        int64_t od = 0, os = 0;
#pragma unroll
        for (int d = 0; d < 4; ++d) {
            od += (int64_t)c[d] * p.dst.st[d];
            os += (int64_t)(c[d] % p.src0.ne[d]) * p.src0.st[d];
        }
        dst[od] = src[os];
    }
}

// resident: CTAs of the kernel that fit on one SM (8 x 256 threads = 2048,
// the SM's thread limit, unless registers allow fewer); the grid never
// exceeds one resident wave, so no CTA waits for another to finish.
uint32_t grid_for(const LaunchEnv& env, uint64_t work_items, int per_thread, uint32_t resident = 8) {
    const uint64_t want = (work_items + (uint64_t)kThreads * per_thread - 1) / ((uint64_t)kThreads * per_thread);
    const uint64_t cap = (uint64_t)env.sm_count * (resident < 8 ? resident : 8);
    uint64_t g = want < cap ? want : cap;
    return (uint32_t)(g == 0 ? 1 : g);
}

// CTAs of `kernel` resident per SM at kThreads threads, cached per device
// (one cache per kernel instantiation).
template <typename K>
uint32_t resident_ctas(DeviceKeyedValue& cache, const LaunchEnv& env, K kernel) {
    uint32_t n = 0;
    if (cache.get(env.device, 0u, &n)) return n;
    int r = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&r, kernel, kThreads, 0) != cudaSuccess || r < 1) r = 1;
    cache.put(env.device, 0u, (uint32_t)r);
    return (uint32_t)r;
}

template <typename T, typename F>
cudaError_t launch_ew(const LaunchEnv& env, const EwPlan& p, const F& f) {
    switch (p.kind) {
    case EwKind::Flat: {
        const uint64_t nvec = p.count / Vec16<T>::N;
        const uint64_t bytes = p.count * sizeof(T);
        const int early = reads_clear(env, p.src0.ptr, bytes) && (!F::kBinary || reads_clear(env, p.src1.ptr, bytes));
        static DeviceKeyedValue resident32, resident64;
        cudaError_t err;
        if (nvec < (1ull << 31) - (uint64_t)(F::kUnroll + 1) * env.sm_count * 8 * kThreads) {
            auto* kernel = ew_flat<T, F, uint32_t>;
            err = launch_dependent(kernel, dim3(grid_for(env, nvec, F::kUnroll, resident_ctas(resident32, env, kernel))),
                                   dim3(kThreads), 0, env.stream, reinterpret_cast<T*>(p.dst.ptr),
                                   reinterpret_cast<const T*>(p.src0.ptr), reinterpret_cast<const T*>(p.src1.ptr),
                                   p.count, f, early);
        } else {
            auto* kernel = ew_flat<T, F, uint64_t>;
            err = launch_dependent(kernel, dim3(grid_for(env, nvec, F::kUnroll, resident_ctas(resident64, env, kernel))),
                                   dim3(kThreads), 0, env.stream, reinterpret_cast<T*>(p.dst.ptr),
                                   reinterpret_cast<const T*>(p.src0.ptr), reinterpret_cast<const T*>(p.src1.ptr),
                                   p.count, f, early);
        }
        if (err != cudaSuccess) return err;
        stream_wrote(env.stream, p.dst.ptr, bytes);
        break;
    }
    case EwKind::Rows: {
        if constexpr (F::kBinary) {
            if (dense_row_broadcast(p)) {
                const uint32_t n = (uint32_t)(p.count / Vec16<T>::N);
                static DeviceKeyedValue resident;
                auto* kernel = ew_row_broadcast<T, F>;
                const uint64_t bytes = p.count * sizeof(T);
                const int early = reads_clear(env, p.src0.ptr, bytes) && reads_clear(env, p.src1.ptr, p.ne[0] * sizeof(T));
                const cudaError_t err = launch_dependent(
                    kernel, dim3(grid_for(env, n, 4, resident_ctas(resident, env, kernel))), dim3(kThreads), 0,
                    env.stream, p, f, make_fastdiv((uint32_t)(p.ne[0] / Vec16<T>::N)), n, early);
                if (err != cudaSuccess) return err;
                stream_wrote(env.stream, p.dst.ptr, bytes);
                break;
            }
        }
        RowsWalk w;
        if (rows_walk(p, &w)) {
            static DeviceKeyedValue resident;
            auto* kernel = ew_rows_vec<T, F>;
            const Span sd = span_of(p.dst, sizeof(T));
            const cudaError_t err = launch_dependent(kernel, dim3(grid_for(env, w.nvec, 4, resident_ctas(resident, env, kernel))),
                                                     dim3(kThreads), 0, env.stream, p, f, w);
            if (err != cudaSuccess) return err;
            stream_wrote(env.stream, sd);
            break;
        }
        const uint64_t per_row = p.vec ? p.ne[0] / Vec16<T>::N : p.ne[0];
        int gshift = 5;
        while (gshift < 8 && (1ull << gshift) < per_row) ++gshift;
        const uint64_t rows = p.count / p.ne[0];
        const uint64_t threads = rows << gshift;
        const cudaError_t err =
            launch_dependent(ew_rows<T, F>, dim3(grid_for(env, threads, 1)), dim3(kThreads), 0, env.stream, p, f, gshift);
        if (err != cudaSuccess) return err;
        break;
    }
    case EwKind::Generic: {
        const cudaError_t err = launch_dependent(ew_generic<T, F>, dim3(grid_for(env, p.count, 1)), dim3(kThreads), 0,
                                                 env.stream, p, f, make_fastdiv((uint32_t)p.ne[0]),
                                                 make_fastdiv((uint32_t)p.ne[1]), make_fastdiv((uint32_t)p.ne[2]));
        if (err != cudaSuccess) return err;
        break;
    }
    case EwKind::Ordinal: {
        const cudaError_t err =
            launch_dependent(ew_ordinal<T, F>, dim3(grid_for(env, p.count, 1)), dim3(kThreads), 0, env.stream, p, f);
        if (err != cudaSuccess) return err;
        break;
    }
        break;
    }
    ++*env.launches;
    return cudaGetLastError();
}

// ---------------------------------------------------------------------------
// binary16 unary ops through context-resident domain tables.
//
// A binary16 operand has 65,536 possible values, far fewer than the
// elements of a large tensor.  When a context is created, one kernel
// evaluates each table op's formula -- the same unary_apply<OP, true> and
// reference conversions the direct kernels use -- for every binary16 input
// into a 128 KB table per op, and the tables stay with the context.  A large
// dense binary16 tensor then streams through a shared-memory copy of its
// op's table: no per-element arithmetic, identical bits to the direct path.
// ---------------------------------------------------------------------------
// The ops whose direct binary16 evaluation costs more than the table stream
// (about 10 us for configuration 2's 7.3 M elements): the three GELUs,
// softplus and the binary64 libm calls.  exp, silu, sigmoid, tanh, elu and
// the rest run faster directly on the binary32 core.
constexpr int kTableOpCodes[kDomainTableSlots] = {kGelu, kGeluQuick, kGeluErf, kSoftplus, kSqrt, kLog, kSin, kCos};

template <int OP>
constexpr bool kTableOp = OP == kGelu || OP == kGeluQuick || OP == kGeluErf || OP == kSoftplus || OP == kSqrt ||
                          OP == kLog || OP == kSin || OP == kCos;

constexpr int table_slot(int op) {
    for (int k = 0; k < kDomainTableSlots; ++k)
        if (kTableOpCodes[k] == op) return k;
    return -1;
}

// the build kernel's case labels follow kTableOpCodes
static_assert(table_slot(kGelu) == 0, "slot order");
static_assert(table_slot(kGeluQuick) == 1, "slot order");
static_assert(table_slot(kGeluErf) == 2, "slot order");
static_assert(table_slot(kSoftplus) == 3, "slot order");
static_assert(table_slot(kSqrt) == 4, "slot order");
static_assert(table_slot(kLog) == 5, "slot order");
static_assert(table_slot(kSin) == 6, "slot order");
static_assert(table_slot(kCos) == 7, "slot order");

constexpr uint64_t kTableMinCount = 1ull << 20;  // below this the 128 KB table copy costs more than it saves
constexpr int kTableThreads = 1024;              // one stream CTA per SM
constexpr uint32_t kTableBytes = 65536u * 2u;

template <int OP>
__device__ __forceinline__ void fill_entry(uint16_t* t, uint32_t h) {
    t[h] = f32_to_f16_bits(unary_apply<OP, true>(f16_bits_to_f32((uint16_t)h), UnaryParams{}));
}

__global__ void __launch_bounds__(256) domain_tables_build(uint16_t* __restrict__ tables) {
    const uint32_t h = blockIdx.x * 256u + threadIdx.x;
    uint16_t* t = tables + (uint64_t)blockIdx.y * 65536u;
    switch (blockIdx.y) {
    case 0: fill_entry<kGelu>(t, h); break;
    case 1: fill_entry<kGeluQuick>(t, h); break;
    case 2: fill_entry<kGeluErf>(t, h); break;
    case 3: fill_entry<kSoftplus>(t, h); break;
    case 4: fill_entry<kSqrt>(t, h); break;
    case 5: fill_entry<kLog>(t, h); break;
    case 6: fill_entry<kSin>(t, h); break;
    case 7: fill_entry<kCos>(t, h); break;
    default: break;
    }
}

__device__ __forceinline__ uint32_t lookup2(const uint16_t* tab, uint32_t w) {
    return (uint32_t)tab[w & 0xffffu] | ((uint32_t)tab[w >> 16] << 16);
}

__device__ __forceinline__ uint4 ld_u4(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ void st_u4(void* p, uint4 v) {
    asm volatile("st.global.L1::no_allocate.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
                 "r"(v.w)
                 : "memory");
}

template <int U>
__device__ __forceinline__ void table_first_loads(uint4 (&cur)[U], const uint16_t* __restrict__ src, uint64_t gid,
                                                  uint64_t stride, uint64_t nvec) {
#pragma unroll
    for (int k = 0; k < U; ++k) {
        const uint64_t i = gid + k * stride;
        cur[k] = i < nvec ? ld_u4(src + i * 8) : make_uint4(0, 0, 0, 0);
    }
}

// One CTA of 1024 threads per SM.  Thread 0 has the TMA engine copy the
// op's 128 KB table into shared memory -- the tables are written once at
// context creation, before any operator, so the copy starts before the wait
// for the previous kernel -- while every thread issues its first 8 vector
// loads (128 KB per SM in flight): before that wait too when `early` (the
// input is clear of the previous kernel's writes), after it otherwise; then
// grid-strided 16-byte vectors stream through the table, 8 per iteration.
__global__ void __launch_bounds__(kTableThreads, 1) table_stream(uint16_t* __restrict__ dst,
                                                                 const uint16_t* __restrict__ src, uint64_t n,
                                                                 const uint16_t* __restrict__ table, uint32_t* fault,
                                                                 int early) {
    extern __shared__ __align__(128) uint16_t tab[];
    __shared__ __align__(8) uint64_t bar;
    constexpr int L = 8;  // halves per 16-byte vector
    constexpr int U = 8;
    const uint64_t nvec = n / L;
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t gid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        mbar_init_fence();
        mbar_expect_tx(&bar, kTableBytes);
        bulk_load(tab, table, kTableBytes, &bar);
    }
    uint4 cur[U];
    if (early) {
        table_first_loads<U>(cur, src, gid, stride, nvec);
        pdl_enter();
    } else {
        pdl_enter();
        table_first_loads<U>(cur, src, gid, stride, nvec);
    }
    __syncthreads();  // the barrier is initialised before any thread waits on it
    const bool ok = mbar_wait(&bar, 0);
    if (!__syncthreads_and(ok)) {
        if (threadIdx.x == 0) {
            atomicExch(fault, 1u);
            mbar_wait(&bar, 0);
        }
        return;
    }
    uint64_t base = gid;
    for (;;) {
#pragma unroll
        for (int k = 0; k < U; ++k) {
            const uint64_t i = base + k * stride;
            if (i < nvec)
                st_u4(dst + i * L, make_uint4(lookup2(tab, cur[k].x), lookup2(tab, cur[k].y), lookup2(tab, cur[k].z),
                                              lookup2(tab, cur[k].w)));
        }
        base += U * stride;
        if (base >= nvec) break;
#pragma unroll
        for (int k = 0; k < U; ++k) {
            const uint64_t i = base + k * stride;
            cur[k] = i < nvec ? ld_u4(src + i * L) : make_uint4(0, 0, 0, 0);
        }
    }
    const uint64_t t = nvec * L + gid;
    if (t < n) dst[t] = tab[src[t]];
}

cudaError_t launch_table_stream(const LaunchEnv& env, const EwPlan& p, int slot) {
    static DeviceFlags configured;  // devices with the attribute set
    if (!configured.done(env.device)) {
        const cudaError_t err =
            cudaFuncSetAttribute(table_stream, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTableBytes);
        if (err != cudaSuccess) return err;
        configured.mark(env.device);
    }
    const uint16_t* table = static_cast<const uint16_t*>(env.tables) + (uint64_t)slot * 65536u;
    uint32_t* fault = reinterpret_cast<uint32_t*>(static_cast<char*>(env.workspace) + kFaultWordOffset);
    const int early = reads_clear(env, p.src0.ptr, p.count * 2);
    const cudaError_t err = launch_dependent(table_stream, dim3((unsigned)env.sm_count), dim3(kTableThreads),
                                             (size_t)kTableBytes, env.stream, reinterpret_cast<uint16_t*>(p.dst.ptr),
                                             reinterpret_cast<const uint16_t*>(p.src0.ptr), p.count, table, fault, early);
    if (err == cudaSuccess) stream_wrote(env.stream, p.dst.ptr, p.count * 2);
    ++*env.launches;
    return err != cudaSuccess ? err : cudaGetLastError();
}

template <int OP>
cudaError_t unary_typed(const LaunchEnv& env, const EwPlan& p, float pa, float pb) {
    if (p.dtype == DType::F16) {
        if constexpr (kTableOp<OP>) {
            if (p.kind == EwKind::Flat && p.vec && p.count >= kTableMinCount && env.tables != nullptr)
                return launch_table_stream(env, p, table_slot(OP));
        }
        return launch_ew<uint16_t>(env, p, UnaryFn<OP, true>{UnaryParams{pa, pb}});
    }
    return launch_ew<float>(env, p, UnaryFn<OP, false>{UnaryParams{pa, pb}});
}

template <int OP>
cudaError_t binary_typed(const LaunchEnv& env, const EwPlan& p) {
    BinaryFn<OP> f;
    if (p.dtype == DType::F16) return launch_ew<uint16_t>(env, p, f);
    return launch_ew<float>(env, p, f);
}

}  // namespace

cudaError_t build_domain_tables(void* tables, cudaStream_t stream) {
    domain_tables_build<<<dim3(65536 / 256, kDomainTableSlots), 256, 0, stream>>>(static_cast<uint16_t*>(tables));
    return cudaGetLastError();
}

cudaError_t launch_unary(const LaunchEnv& env, const EwPlan& p, int op, float pa, float pb) {
    switch (op) {
#define EMEL_UNARY_CASE(code) \
    case code: return unary_typed<code>(env, p, pa, pb);
        EMEL_UNARY_CASE(kAbs) EMEL_UNARY_CASE(kSgn) EMEL_UNARY_CASE(kNeg) EMEL_UNARY_CASE(kStep)
        EMEL_UNARY_CASE(kTanh) EMEL_UNARY_CASE(kElu) EMEL_UNARY_CASE(kRelu) EMEL_UNARY_CASE(kSigmoid)
        EMEL_UNARY_CASE(kGelu) EMEL_UNARY_CASE(kGeluQuick) EMEL_UNARY_CASE(kSilu) EMEL_UNARY_CASE(kHardswish)
        EMEL_UNARY_CASE(kHardsigmoid) EMEL_UNARY_CASE(kExp) EMEL_UNARY_CASE(kExpm1) EMEL_UNARY_CASE(kSoftplus)
        EMEL_UNARY_CASE(kGeluErf) EMEL_UNARY_CASE(kFloor) EMEL_UNARY_CASE(kCeil) EMEL_UNARY_CASE(kRound)
        EMEL_UNARY_CASE(kTrunc) EMEL_UNARY_CASE(kSqr) EMEL_UNARY_CASE(kSqrt) EMEL_UNARY_CASE(kLog)
        EMEL_UNARY_CASE(kSin) EMEL_UNARY_CASE(kCos) EMEL_UNARY_CASE(kScale) EMEL_UNARY_CASE(kClamp)
        EMEL_UNARY_CASE(kLeakyRelu) EMEL_UNARY_CASE(kAdd1) EMEL_UNARY_CASE(kCopy) EMEL_UNARY_CASE(kGeluGeneric)
#undef EMEL_UNARY_CASE
    default: return cudaErrorInvalidValue;
    }
}

cudaError_t launch_repeat(const LaunchEnv& env, const EwPlan& p) {
    RepeatArgs r{};
    r.small = p.count < (1ull << 32);
    for (int d = 0; d < 4; ++d) r.small = r.small && p.ne[d] < (1ull << 31);
    if (r.small) {
        r.d0 = make_fastdiv((uint32_t)p.ne[0]);
        r.d1 = make_fastdiv((uint32_t)p.ne[1]);
        r.d2 = make_fastdiv((uint32_t)p.ne[2]);
    }
    const cudaError_t err =
        launch_dependent(repeat_copy, dim3(grid_for(env, p.count, 1)), dim3(kThreads), 0, env.stream, p, r);
    ++*env.launches;
    return err != cudaSuccess ? err : cudaGetLastError();
}

cudaError_t launch_binary(const LaunchEnv& env, const EwPlan& p, int op) {
    switch (op) {
    case kAdd: return binary_typed<kAdd>(env, p);
    case kSub: return binary_typed<kSub>(env, p);
    case kMul: return binary_typed<kMul>(env, p);
    case kDiv: return binary_typed<kDiv>(env, p);
    case kSiluBack: return launch_ew<float>(env, p, SiluBackFn{});
    case kGluBase + kReGlu: return launch_ew<float>(env, p, GluFn<kReGlu>{});
    case kGluBase + kGeGlu: return launch_ew<float>(env, p, GluFn<kGeGlu>{});
    case kGluBase + kSwiGlu: return launch_ew<float>(env, p, GluFn<kSwiGlu>{});
    case kGluBase + kSwiGluOai: return launch_ew<float>(env, p, GluFn<kSwiGluOai>{});
    case kGluBase + kGeGluErf: return launch_ew<float>(env, p, GluFn<kGeGluErf>{});
    case kGluBase + kGeGluQuick: return launch_ew<float>(env, p, GluFn<kGeGluQuick>{});
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace emel
