// emel_kernels_cuda.hpp -- C++ host mirror of the emel-kernels operator
// contract over the device op table (include/emel_cuda.h).
//
// The reference API is Rust: `emel_kernels::Kernel::process_event(E)` with
// typed events holding borrowed `TensorView` / `TensorViewMut` over slices
// and family-specific `Result<(), FamilyError>` outputs
// (crates/emel-kernels/src/any/actor.rs:936-943, binary.rs:47-81,
// normalization.rs:58-96, reductions.rs:90-163).  This header keeps those
// names, argument orders and error variants for C++ callers; views bind
// device memory instead of slices.  Header-only: every call goes straight
// to the C ABI.  A rejected event returns its error without touching the
// output, exactly like the reference.
#pragma once

#include <array>
#include <cstdint>
#include <optional>
#include <stdexcept>
#include <string>

#include "emel_cuda.h"

namespace emel_kernels::cuda {

// DType wire codes (tensor_view.rs:160-209), the subset the device table serves.
enum class DType : uint32_t { F32 = 0, F16 = 1, I32 = 26, I64 = 27 };

inline uint64_t dtype_size(DType d) {
    switch (d) {
    case DType::F16: return 2;
    case DType::I64: return 8;
    default: return 4;
    }
}

// Layout { dtype, ne[4], nb[4] } (tensor_view.rs:215-342).
class Layout {
public:
    Layout(DType dtype, std::array<uint64_t, 4> ne, std::array<uint64_t, 4> nb) : dtype_(dtype), ne_(ne), nb_(nb) {}

    static std::optional<Layout> contiguous(DType dtype, std::array<uint64_t, 4> ne) {
        std::array<uint64_t, 4> nb{dtype_size(dtype), 0, 0, 0};
        for (int d = 1; d < 4; ++d)
            if (__builtin_mul_overflow(nb[d - 1], ne[d - 1], &nb[d])) return std::nullopt;
        return Layout(dtype, ne, nb);
    }

    std::optional<Layout> permuted(std::array<size_t, 4> axes) const {
        std::array<uint64_t, 4> ne{}, nb{};
        for (int d = 0; d < 4; ++d) {
            if (axes[d] >= 4) return std::nullopt;
            ne[d] = ne_[axes[d]];
            nb[d] = nb_[axes[d]];
        }
        return Layout(dtype_, ne, nb);
    }

    DType dtype() const { return dtype_; }
    const std::array<uint64_t, 4>& ne() const { return ne_; }
    const std::array<uint64_t, 4>& nb() const { return nb_; }

private:
    DType dtype_;
    std::array<uint64_t, 4> ne_;
    std::array<uint64_t, 4> nb_;
};

// A view of device storage: `data` is a device address, `storage_bytes` the
// length of the backing allocation the view may reach.
class TensorView {
public:
    TensorView(const void* data, uint64_t storage_bytes, Layout layout)
        : data_(const_cast<void*>(data)), bytes_(storage_bytes), layout_(layout) {}

    const Layout& layout() const { return layout_; }

    emel_tensor_view c() const {
        emel_tensor_view v{};
        v.data = data_;
        v.storage_bytes = bytes_;
        for (int d = 0; d < 4; ++d) {
            v.ne[d] = layout_.ne()[d];
            v.nb[d] = layout_.nb()[d];
        }
        v.dtype = static_cast<uint32_t>(layout_.dtype());
        return v;
    }

private:
    void* data_;
    uint64_t bytes_;
    Layout layout_;
};
using TensorViewMut = TensorView;

// Error variants shared by every family (binary.rs:20-29, broadcast.rs:29-38,
// unary.rs:22-31, normalization.rs:31-42, reductions.rs:21-30), plus the
// device outcomes.
enum class Error : int {
    InvalidView = EMEL_CUDA_INVALID_VIEW,
    ShapeMismatch = EMEL_CUDA_SHAPE_MISMATCH,
    InvalidParameters = EMEL_CUDA_INVALID_PARAMETERS,
    UnexpectedEvent = EMEL_CUDA_UNEXPECTED_EVENT,
    Internal = EMEL_CUDA_INTERNAL,
    DeviceError = EMEL_CUDA_DEVICE_ERROR,
    Timeout = EMEL_CUDA_TIMEOUT,
    InvalidArgument = EMEL_CUDA_INVALID_ARGUMENT,
    OutOfMemory = EMEL_CUDA_OUT_OF_MEMORY,
    InvalidRequest = EMEL_CUDA_INVALID_REQUEST,  // FlashAttnError::InvalidRequest (flash_attn.rs:35-44)
};
using BinaryError = Error;
using BroadcastError = Error;
using UnaryError = Error;
using NormalizationError = Error;
using ReductionError = Error;
using ActivationError = Error;
using FlashAttnError = Error;

// Result<(), Error>: empty when Ok.
class Result {
public:
    Result() = default;
    explicit Result(emel_cuda_status st) {
        if (st != EMEL_CUDA_OK) err_ = static_cast<Error>(st);
    }
    bool is_ok() const { return !err_.has_value(); }
    Error error() const { return *err_; }
    bool operator==(const Result& o) const { return err_ == o.err_; }
    static Result Ok() { return Result(); }
    static Result Err(Error e) { return Result(static_cast<emel_cuda_status>(e)); }

private:
    std::optional<Error> err_;
};

// ---- events ----------------------------------------------------------------
enum class UnarySubOp : int {
    Abs = 0, Sgn = 1, Neg = 2, Step = 3, Tanh = 4, Elu = 5, Relu = 6, Sigmoid = 7, Gelu = 8, GeluQuick = 9,
    Silu = 10, Hardswish = 11, Hardsigmoid = 12, Exp = 13, Expm1 = 14, Softplus = 15, GeluErf = 16, Xielu = 17,
    Floor = 18, Ceil = 19, Round = 20, Trunc = 21
};

#define EMEL_BINARY_EVENT(Name, code)                                          \
    struct Name {                                                              \
        static constexpr int kOp = code;                                       \
        Name(TensorView l, TensorView r, TensorViewMut o) : lhs(l), rhs(r), output(o) {} \
        TensorView lhs, rhs;                                                   \
        TensorViewMut output;                                                  \
    };
EMEL_BINARY_EVENT(OpAdd, EMEL_BINARY_ADD)
EMEL_BINARY_EVENT(OpSub, EMEL_BINARY_SUB)
EMEL_BINARY_EVENT(OpMul, EMEL_BINARY_MUL)
EMEL_BINARY_EVENT(OpDiv, EMEL_BINARY_DIV)
#undef EMEL_BINARY_EVENT

#define EMEL_ROW_EVENT(Name, code)                                                 \
    struct Name {                                                                  \
        static constexpr int kOp = code;                                           \
        Name(TensorView a, TensorView b, TensorViewMut d) : src0(a), src1(b), dst(d) {} \
        TensorView src0, src1;                                                     \
        TensorViewMut dst;                                                         \
    };
EMEL_ROW_EVENT(OpAddBroadcastRow, EMEL_BINARY_ADD)
EMEL_ROW_EVENT(OpSubBroadcastRow, EMEL_BINARY_SUB)
EMEL_ROW_EVENT(OpMulBroadcastRow, EMEL_BINARY_MUL)
EMEL_ROW_EVENT(OpDivBroadcastRow, EMEL_BINARY_DIV)
#undef EMEL_ROW_EVENT

struct OpUnary {
    OpUnary(UnarySubOp s, TensorView i, TensorViewMut o) : subop(s), input(i), output(o) {}
    UnarySubOp subop;
    TensorView input;
    TensorViewMut output;
};

// One typed unary event per formula (unary.rs:72-92; power.rs OpSqr/OpSqrt).
struct OpUnaryTyped {
    OpUnaryTyped(int o, TensorView i, TensorViewMut out) : op(o), input(i), output(out) {}
    int op;
    TensorView input;
    TensorViewMut output;
};
inline OpUnaryTyped OpSilu(TensorView i, TensorViewMut o) { return {EMEL_UNARY_SILU, i, o}; }
inline OpUnaryTyped OpGelu(TensorView i, TensorViewMut o) { return {EMEL_UNARY_GELU, i, o}; }
inline OpUnaryTyped OpRelu(TensorView i, TensorViewMut o) { return {EMEL_UNARY_RELU, i, o}; }
inline OpUnaryTyped OpExp(TensorView i, TensorViewMut o) { return {EMEL_UNARY_EXP, i, o}; }
inline OpUnaryTyped OpNeg(TensorView i, TensorViewMut o) { return {EMEL_UNARY_NEG, i, o}; }
inline OpUnaryTyped OpSqr(TensorView i, TensorViewMut o) { return {EMEL_UNARY_SQR, i, o}; }
inline OpUnaryTyped OpSqrt(TensorView i, TensorViewMut o) { return {EMEL_UNARY_SQRT, i, o}; }

struct OpScale {
    OpScale(TensorView i, TensorViewMut o, float s) : input(i), output(o), scale(s) {}
    TensorView input;
    TensorViewMut output;
    float scale;
};

#define EMEL_NORM_EVENT(Name)                                                              \
    struct Name {                                                                          \
        Name(TensorView i, TensorViewMut o, float e) : input(i), output(o), epsilon(e) {}  \
        TensorView input;                                                                  \
        TensorViewMut output;                                                              \
        float epsilon;                                                                     \
    };
EMEL_NORM_EVENT(OpNorm)
EMEL_NORM_EVENT(OpRmsNorm)
#undef EMEL_NORM_EVENT

#define EMEL_REDUCE_EVENT(Name)                                     \
    struct Name {                                                   \
        Name(TensorView s, TensorViewMut d) : src(s), dst(d) {}     \
        TensorView src;                                             \
        TensorViewMut dst;                                          \
    };
EMEL_REDUCE_EVENT(OpSoftMax)
EMEL_REDUCE_EVENT(OpSum)
EMEL_REDUCE_EVENT(OpMean)
EMEL_REDUCE_EVENT(OpSumRows)
EMEL_REDUCE_EVENT(OpArgmax)
#undef EMEL_REDUCE_EVENT

struct OpSoftMaxExt {
    OpSoftMaxExt(TensorView s, std::optional<TensorView> m, TensorViewMut d, float sc)
        : src(s), mask(m), dst(d), scale(sc) {}
    TensorView src;
    std::optional<TensorView> mask;
    TensorViewMut dst;
    float scale;
};

// flash_attn::FlashAttnOptions / OpFlashAttnExt (flash_attn.rs:24-31, 62-99):
// query / destination F32 [d, 1, heads, 1]; key / value F16 [d, tokens,
// kv_heads, 1].  Absent options resolve at dispatch (1 / sqrt(d), tokens).
struct FlashAttnOptions {
    std::optional<float> scale;
    std::optional<uint32_t> masked_total_tokens;
};
struct OpFlashAttnExt {
    OpFlashAttnExt(TensorView q, TensorView k, TensorView v, TensorViewMut d, FlashAttnOptions o = {})
        : query(q), key(k), value(v), destination(d), options(o) {}
    TensorView query, key, value;
    TensorViewMut destination;
    FlashAttnOptions options;
};

// ---- the actor -------------------------------------------------------------
// Single-writer like the reference's Kernel (not thread-safe): one context,
// one stream; process_event enqueues and, unless asynchronous, waits.
class Kernel {
public:
    explicit Kernel(int device = 0, bool synchronous = true) : sync_(synchronous) {
        if (emel_cuda_context_create(device, &ctx_) != EMEL_CUDA_OK) throw std::runtime_error("emel_cuda_context_create");
        if (emel_cuda_stream_create(ctx_, &stream_) != EMEL_CUDA_OK) throw std::runtime_error("emel_cuda_stream_create");
    }
    ~Kernel() {
        if (stream_) emel_cuda_stream_destroy(ctx_, stream_);
        if (ctx_) emel_cuda_context_destroy(ctx_);
    }
    Kernel(const Kernel&) = delete;
    Kernel& operator=(const Kernel&) = delete;

    emel_cuda_context* context() { return ctx_; }
    void* stream() { return stream_; }

    template <class E>
    Result process_event(const E& e) {
        return finish(dispatch(e));
    }

private:
    Result finish(emel_cuda_status st) {
        if (st == EMEL_CUDA_OK && sync_) st = emel_cuda_stream_synchronize(ctx_, stream_);
        return Result(st);
    }

    template <class E>
    auto dispatch(const E& e) -> decltype(e.lhs, emel_cuda_status()) {
        auto l = e.lhs.c(), r = e.rhs.c(), o = e.output.c();
        return emel_cuda_binary(ctx_, stream_, E::kOp, &l, &r, &o);
    }
    template <class E>
    auto dispatch(const E& e) -> decltype(e.src1, emel_cuda_status()) {
        auto a = e.src0.c(), b = e.src1.c(), d = e.dst.c();
        return emel_cuda_broadcast_row(ctx_, stream_, E::kOp, &a, &b, &d);
    }
    emel_cuda_status dispatch(const OpUnary& e) {
        auto i = e.input.c(), o = e.output.c();
        return emel_cuda_op_unary(ctx_, stream_, static_cast<int>(e.subop), &i, &o);
    }
    emel_cuda_status dispatch(const OpUnaryTyped& e) {
        auto i = e.input.c(), o = e.output.c();
        return emel_cuda_unary(ctx_, stream_, e.op, &i, &o);
    }
    emel_cuda_status dispatch(const OpScale& e) {
        auto i = e.input.c(), o = e.output.c();
        return emel_cuda_scale(ctx_, stream_, &i, &o, e.scale);
    }
    emel_cuda_status dispatch(const OpNorm& e) {
        auto i = e.input.c(), o = e.output.c();
        return emel_cuda_norm(ctx_, stream_, &i, &o, e.epsilon);
    }
    emel_cuda_status dispatch(const OpRmsNorm& e) {
        auto i = e.input.c(), o = e.output.c();
        return emel_cuda_rms_norm(ctx_, stream_, &i, &o, e.epsilon);
    }
    emel_cuda_status dispatch(const OpSoftMax& e) {
        auto s = e.src.c(), d = e.dst.c();
        return emel_cuda_soft_max(ctx_, stream_, &s, &d);
    }
    emel_cuda_status dispatch(const OpSoftMaxExt& e) {
        auto s = e.src.c(), d = e.dst.c();
        if (e.mask) {
            auto m = e.mask->c();
            return emel_cuda_soft_max_ext(ctx_, stream_, &s, &m, &d, e.scale);
        }
        return emel_cuda_soft_max_ext(ctx_, stream_, &s, nullptr, &d, e.scale);
    }
    emel_cuda_status dispatch(const OpSum& e) {
        auto s = e.src.c(), d = e.dst.c();
        return emel_cuda_sum(ctx_, stream_, &s, &d);
    }
    emel_cuda_status dispatch(const OpMean& e) {
        auto s = e.src.c(), d = e.dst.c();
        return emel_cuda_mean(ctx_, stream_, &s, &d);
    }
    emel_cuda_status dispatch(const OpSumRows& e) {
        auto s = e.src.c(), d = e.dst.c();
        return emel_cuda_sum_rows(ctx_, stream_, &s, &d);
    }
    emel_cuda_status dispatch(const OpArgmax& e) {
        auto s = e.src.c(), d = e.dst.c();
        return emel_cuda_argmax(ctx_, stream_, &s, &d);
    }

    emel_cuda_status dispatch(const OpFlashAttnExt& e) {
        auto q = e.query.c(), k = e.key.c(), v = e.value.c(), d = e.destination.c();
        emel_flash_attn_options o{};
        if (e.options.scale) {
            o.scale = *e.options.scale;
            o.has_scale = 1;
        }
        if (e.options.masked_total_tokens) {
            o.masked_total_tokens = *e.options.masked_total_tokens;
            o.has_masked_total_tokens = 1;
        }
        return emel_cuda_flash_attn_ext(ctx_, stream_, &q, &k, &v, &d, &o);
    }

    emel_cuda_context* ctx_ = nullptr;
    void* stream_ = nullptr;
    bool sync_;
};

// Device buffer helper for tests and callers without their own allocator.
class DeviceBuffer {
public:
    DeviceBuffer(Kernel& k, uint64_t bytes) : k_(k), bytes_(bytes) {
        if (emel_cuda_malloc(k.context(), bytes ? bytes : 1, &ptr_) != EMEL_CUDA_OK) throw std::runtime_error("malloc");
    }
    ~DeviceBuffer() { emel_cuda_free(k_.context(), ptr_); }
    DeviceBuffer(const DeviceBuffer&) = delete;
    DeviceBuffer& operator=(const DeviceBuffer&) = delete;

    void upload(const void* host, uint64_t bytes) {
        emel_cuda_memcpy_h2d(k_.context(), k_.stream(), ptr_, host, bytes);
        emel_cuda_stream_synchronize(k_.context(), k_.stream());
    }
    void download(void* host, uint64_t bytes) {
        emel_cuda_memcpy_d2h(k_.context(), k_.stream(), host, ptr_, bytes);
        emel_cuda_stream_synchronize(k_.context(), k_.stream());
    }
    TensorView view(Layout l) const { return TensorView(ptr_, bytes_, l); }
    void* data() const { return ptr_; }

private:
    Kernel& k_;
    uint64_t bytes_;
    void* ptr_ = nullptr;
};

}  // namespace emel_kernels::cuda
