// Launch plans: what the host-side validator hands to the kernel launchers.
// Plain structs, passed to kernels by value.
#pragma once

#include <cstdint>

#include <cuda_runtime.h>

namespace emel {

enum class DType : int { F32 = 0, F16 = 1, I32 = 26, I64 = 27 };

// Binary formula codes (emel_cuda_binary_op); 16 = silu_back (grad * silu'(x)).
enum BinaryOp : int { kAdd = 0, kSub = 1, kMul = 2, kDiv = 3, kSiluBack = 16 };

// Gated linear units (glu.rs:22-38 GluSubOp wire codes), run as two-input
// elementwise ops (value, gate) under BinaryOp code kGluBase + subop.
enum GluSubOp : int { kReGlu = 0, kGeGlu = 1, kSwiGlu = 2, kSwiGluOai = 3, kGeGluErf = 4, kGeGluQuick = 5 };
constexpr int kGluBase = 32;

// Unary formula codes (emel_cuda_unary_op); parameterised ops use codes >= 128.
enum UnaryOp : int {
    kAbs = 0, kSgn = 1, kNeg = 2, kStep = 3, kTanh = 4, kElu = 5, kRelu = 6, kSigmoid = 7, kGelu = 8,
    kGeluQuick = 9, kSilu = 10, kHardswish = 11, kHardsigmoid = 12, kExp = 13, kExpm1 = 14, kSoftplus = 15,
    kGeluErf = 16, kFloor = 18, kCeil = 19, kRound = 20, kTrunc = 21,
    kSqr = 64, kSqrt = 65, kLog = 66, kSin = 67, kCos = 68,
    kScale = 128, kClamp = 129, kLeakyRelu = 130, kAdd1 = 131, kCopy = 132,
    kGeluGeneric = 133  // the generic envelope's GELU (generic.rs:1330-1337)
};

// One operand over the iteration space: base address and element strides per
// dimension (a stride of 0 repeats the element), plus its own extents, which
// the ordinal-order and repeat-broadcast paths need.
struct Operand {
    char* ptr;
    int64_t st[4];
    uint64_t ne[4];
};

enum class EwKind : int {
    Flat = 0,     // every operand dense with identical extents: one 1-D stream
    Rows = 1,     // dim0 unit stride for every operand: row workers, vectorised
    Generic = 2,  // shared iteration extents, arbitrary strides
    Ordinal = 3   // equal counts, different extents: per-operand ordinal decode
};

// Elementwise plan (unary, binary, broadcast).  For binary ops src1's extents
// may be divisors of the iteration extents (repeat broadcast).
struct EwPlan {
    EwKind kind;
    DType dtype;
    int ndim;
    uint64_t ne[4];
    uint64_t count;
    bool vec;        // 16-byte vector path legal (alignment and extents checked)
    bool src1_bcast; // src1 extents differ from the iteration extents
    Operand dst;
    Operand src0;
    Operand src1;
};

// Row plan: a tensor viewed as rows of ne0 elements over (ne1, ne2, ne3).
struct RowOperand {
    char* ptr;
    int64_t st[4];  // element strides
    uint64_t ne[4];
};

struct RowPlan {
    uint64_t ne[4];
    uint64_t rows;
    bool contiguous_rows;  // every operand: dim0 stride 1
    bool vec;              // 16-byte vectors legal for every operand
    bool dense;            // softmax: src and dst dense (f64 sum) or not (f32 sum)
    bool flat;             // src is one dense run of rows * ne0 elements, 16-byte aligned
    bool dst_ordinal;      // dst has other extents: address it by ordinal (dst.ne, dst.st)
    RowOperand src;
    RowOperand dst;
    RowOperand aux;        // weight (rms_norm_mul) or mask (soft_max_ext)
    int aux_dtype;         // DType of aux
    bool has_aux;
};

struct LaunchEnv {
    cudaStream_t stream;
    int sm_count;
    int device;
    uint64_t* launches;
    void* workspace;         // device scratch owned by the context
    uint64_t workspace_bytes;
    const void* tables;      // the context's binary16 domain tables (kDomainTableSlots x 128 KB)
    // The device bytes [prev_lo, prev_hi) written by the library's previous
    // launch on `stream`, when known (prev_known; stream_wrote).  A kernel
    // whose inputs lie outside them may read before that launch finishes.
    uintptr_t prev_lo, prev_hi;
    bool prev_known;
};

// Per-stream record of the bytes the library's last launch wrote (host.cpp).
// stream_take returns the stream's record and clears it (every entry point
// that launches anything takes it first, so an unreported launch leaves the
// record unknown); stream_wrote records a finished launch's output range.
void stream_take(cudaStream_t stream, uintptr_t* lo, uintptr_t* hi, bool* known);
void stream_wrote(cudaStream_t stream, const void* p, uint64_t bytes);

// The bytes a view (Operand or RowOperand: ptr, element strides st, extents
// ne) can touch: from its base to the last element of the last row.
struct Span {
    uintptr_t lo, hi;
};
template <typename O>
inline Span span_of(const O& o, uint64_t elem_bytes) {
    uint64_t last = 0;
    for (int d = 0; d < 4; ++d)
        if (o.ne[d] > 0) last += (o.ne[d] - 1) * (uint64_t)(o.st[d] < 0 ? -o.st[d] : o.st[d]);
    const uintptr_t lo = reinterpret_cast<uintptr_t>(o.ptr);
    return Span{lo, lo + (last + 1) * elem_bytes};
}

// True when the span lies outside what the previous launch on the stream
// wrote (and that range is known).
inline bool reads_clear(const LaunchEnv& env, const Span& s) {
    if (!env.prev_known) return false;
    return s.hi <= env.prev_lo || s.lo >= env.prev_hi;
}
inline bool reads_clear(const LaunchEnv& env, const void* p, uint64_t bytes) {
    const uintptr_t lo = reinterpret_cast<uintptr_t>(p);
    return reads_clear(env, Span{lo, lo + bytes});
}
inline void stream_wrote(cudaStream_t stream, const Span& s) {
    stream_wrote(stream, reinterpret_cast<const void*>(s.lo), s.hi - s.lo);
}

}  // namespace emel
