// Host side of the device op table: context, memory and stream handles,
// view validation in the reference's guard order, dimension
// canonicalisation and launch planning, and the extern "C" entry points
// declared in include/emel_cuda.h.
//
// Validation mirrors crates/emel-kernels/src/any/tensor_view.rs:259-447 and
// the per-family guards it cites.  It touches no device memory and makes no
// CUDA call, so a rejected request returns before the context or stream is
// even looked at and never writes its destination.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>

#include <cuda_runtime.h>

#include "emel_cuda.h"
#include "launch.hpp"

struct emel_cuda_context {
    int device;
    int sm_count;
    void* workspace;
    uint64_t workspace_bytes;
    void* tables;  // binary16 domain tables, built at creation
    uint64_t launches;
    uint64_t fa_prepared_tokens;  // FlashAttnWorkspace::prepared_tokens (flash_attn.rs:117-118)
    uint64_t fa_reuse_count;      // FlashAttnWorkspace::reuse_count
    char last_error[256];
};

namespace {

using emel::DType;
using u128 = unsigned __int128;

uint64_t dtype_size(uint32_t dtype) {
    switch (dtype) {
    case EMEL_DTYPE_F32: return 4;
    case EMEL_DTYPE_F16: return 2;
    case EMEL_DTYPE_I32: return 4;
    case EMEL_DTYPE_I64: return 8;
    default: return 0;
    }
}

// A validated view: element count and effective byte strides.
struct Checked {
    uint64_t count = 0;
    uint64_t nb[4] = {0, 0, 0, 0};
    uint64_t elem = 0;
};

// Layout::element_count (tensor_view.rs:346-358).
bool count_of(const emel_tensor_view& v, uint64_t* out) {
    uint64_t n = 1;
    for (int d = 0; d < 4; ++d) {
        if (v.ne[d] == 0 || __builtin_mul_overflow(n, v.ne[d], &n)) return false;
    }
    *out = n;
    return true;
}

// Layout::effective_f32_strides (tensor_view.rs:262-277) for any element size.
bool strides_of(const emel_tensor_view& v, uint64_t elem, uint64_t out[4]) {
    if (v.nb[0] != 0) {
        for (int d = 0; d < 4; ++d) out[d] = v.nb[d];
        return true;
    }
    out[0] = elem;
    for (int d = 1; d < 4; ++d)
        if (__builtin_mul_overflow(out[d - 1], v.ne[d - 1], &out[d])) return false;
    return true;
}

// The device pointer must be able to stand in for the reference's slice:
// non-null and aligned to the element type.
bool addressable(const emel_tensor_view& v, uint64_t elem) {
    return v.data != nullptr && reinterpret_cast<uintptr_t>(v.data) % elem == 0;
}

// Layout::validate_element_storage (tensor_view.rs:392-447).
bool validate_as(const emel_tensor_view* v, uint32_t dtype, bool singleton_zero_ok, Checked* out) {
    if (v == nullptr || v->dtype != dtype) return false;
    const uint64_t elem = dtype_size(dtype);
    Checked c;
    c.elem = elem;
    if (!count_of(*v, &c.count) || !strides_of(*v, elem, c.nb)) return false;
    for (int d = 0; d < 4; ++d) {
        const bool zero_ok = singleton_zero_ok && v->ne[d] == 1 && c.nb[d] == 0;
        if (!zero_ok && (c.nb[d] < elem || c.nb[d] % elem != 0)) return false;
    }
    u128 span = 0;
    for (int d = 0; d < 4; ++d) span += (u128)(v->ne[d] - 1) * (u128)c.nb[d];
    if (span + elem > (u128)v->storage_bytes) return false;
    if (!addressable(*v, elem)) return false;
    if (out) *out = c;
    return true;
}

// F32 views always; F16 views as this device table's extension.
bool validate_float(const emel_tensor_view* v, bool singleton_zero_ok, Checked* out) {
    if (v == nullptr || (v->dtype != EMEL_DTYPE_F32 && v->dtype != EMEL_DTYPE_F16)) return false;
    return validate_as(v, v->dtype, singleton_zero_ok, out);
}

// normalization_view_valid (normalization.rs:237-287).
bool normalization_valid(const emel_tensor_view* v, Checked* out) {
    if (v == nullptr || v->dtype != EMEL_DTYPE_F32 || v->ne[0] == 0) return false;
    if (v->nb[0] != 0) {
        if (v->nb[0] < 4 || v->nb[0] % 4 != 0) return false;
        for (int d = 0; d < 4; ++d)
            if (v->ne[d] > 1 && v->nb[d] == 0) return false;
    }
    return validate_as(v, EMEL_DTYPE_F32, false, out);
}

bool same_ne(const emel_tensor_view* a, const emel_tensor_view* b) {
    return std::memcmp(a->ne, b->ne, sizeof(a->ne)) == 0;
}

// Layout::is_dense_contiguous_for (tensor_view.rs:297-314) on effective strides.
bool dense(const emel_tensor_view& v, const Checked& c) {
    uint64_t expect = c.elem;
    for (int d = 0; d < 4; ++d) {
        if (c.nb[d] != expect) return false;
        expect *= v.ne[d];
    }
    return true;
}

bool aligned16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

emel::Operand operand(const emel_tensor_view* v, const Checked& c) {
    emel::Operand o{};
    o.ptr = static_cast<char*>(v->data);
    for (int d = 0; d < 4; ++d) {
        o.st[d] = (int64_t)(c.nb[d] / c.elem);
        o.ne[d] = v->ne[d];
    }
    return o;
}

// ---------------------------------------------------------------------------
// Elementwise planning.
// ---------------------------------------------------------------------------

// Shared-extent plan: drop singleton dimensions, merge neighbours that every
// operand stores contiguously, then pick the kernel shape.
emel::EwPlan plan_shared(DType dt, const uint64_t ne_in[4], emel::Operand* ops[3], int nops, bool src1_bcast) {
    emel::EwPlan p{};
    p.dtype = dt;
    uint64_t ne[4];
    int64_t st[3][4];
    uint64_t bne[4];  // src1 extents along the kept dims (broadcast plans)
    int k = 0;
    for (int d = 0; d < 4; ++d) {
        if (ne_in[d] == 1) continue;
        ne[k] = ne_in[d];
        bne[k] = src1_bcast ? ops[2]->ne[d] : ne_in[d];
        for (int o = 0; o < nops; ++o) st[o][k] = ops[o]->st[d];
        ++k;
    }
    if (k == 0) {
        ne[0] = 1;
        bne[0] = 1;
        for (int o = 0; o < nops; ++o) st[o][0] = 1;
        k = 1;
    }
    // merge d+1 into d when every operand (and the broadcast pattern) allows it
    int m = 0;
    for (int d = 1; d < k; ++d) {
        bool ok = true;
        for (int o = 0; o < nops; ++o)
            if (st[o][d] != st[o][m] * (int64_t)ne[m]) ok = false;
        if (src1_bcast && !(bne[m] == ne[m] && bne[d] == ne[d])) ok = false;
        if (ok) {
            ne[m] *= ne[d];
            bne[m] *= bne[d];
        } else {
            ++m;
            ne[m] = ne[d];
            bne[m] = bne[d];
            for (int o = 0; o < nops; ++o) st[o][m] = st[o][d];
        }
    }
    k = m + 1;
    for (int d = k; d < 4; ++d) {
        ne[d] = 1;
        bne[d] = 1;
        for (int o = 0; o < nops; ++o) st[o][d] = 0;
    }
    p.ndim = k;
    p.count = 1;
    for (int d = 0; d < 4; ++d) {
        p.ne[d] = ne[d];
        p.count *= ne[d];
    }
    emel::Operand* outs[3] = {&p.dst, &p.src0, &p.src1};
    for (int o = 0; o < nops; ++o) {
        outs[o]->ptr = ops[o]->ptr;
        for (int d = 0; d < 4; ++d) {
            outs[o]->st[d] = st[o][d];
            outs[o]->ne[d] = (o == 2) ? bne[d] : ne[d];
        }
    }
    p.src1_bcast = false;
    if (nops == 3 && src1_bcast)
        for (int d = 0; d < 4; ++d)
            if (bne[d] != ne[d]) p.src1_bcast = true;
    const int N = dt == DType::F16 ? 8 : 4;
    // dim0 unit stride for dst and src0, and for src1 unless it repeats one
    // column across the row
    bool unit0 = st[0][0] == 1 && st[1][0] == 1;
    if (nops == 3 && !(p.src1_bcast && bne[0] == 1) && st[2][0] != 1) unit0 = false;
    bool all_aligned = true;
    for (int o = 0; o < nops; ++o)
        if (!aligned16(ops[o]->ptr)) all_aligned = false;
    if (k == 1 && unit0 && !p.src1_bcast) {
        p.kind = emel::EwKind::Flat;
        p.vec = all_aligned;
        if (!all_aligned) p.kind = emel::EwKind::Generic;
    } else if (unit0) {
        p.kind = emel::EwKind::Rows;
        bool v = all_aligned && ne[0] % N == 0 && (!p.src1_bcast || bne[0] == ne[0]);
        for (int o = 0; o < nops; ++o)
            for (int d = 1; d < 4; ++d)
                if (st[o][d] % N != 0) v = false;
        p.vec = v;
    } else {
        p.kind = emel::EwKind::Generic;
    }
    if (p.kind == emel::EwKind::Generic) {
        bool small = p.count < (1ull << 32);
        for (int d = 0; d < 4; ++d)
            if (ne[d] > (1ull << 31)) small = false;
        if (!small) {
            // 64-bit ordinal decode: give every operand the iteration extents
            p.kind = emel::EwKind::Ordinal;
        }
    }
    return p;
}

// Equal-count plan where operands may have different extents.
emel::EwPlan plan_equal_count(DType dt, const emel_tensor_view* views[3], const Checked* cs[3], int nops) {
    emel::Operand ops[3];
    emel::Operand* pops[3];
    for (int o = 0; o < nops; ++o) {
        ops[o] = operand(views[o], *cs[o]);
        pops[o] = &ops[o];
    }
    bool shared = true;
    for (int o = 1; o < nops; ++o)
        if (!same_ne(views[0], views[o])) shared = false;
    if (shared) return plan_shared(dt, views[0]->ne, pops, nops, false);
    bool all_dense = true;
    for (int o = 0; o < nops; ++o)
        if (!dense(*views[o], *cs[o])) all_dense = false;
    if (all_dense) {
        // identical ordinal -> offset maps: stream them as one run
        uint64_t flat_ne[4] = {cs[0]->count, 1, 1, 1};
        for (int o = 0; o < nops; ++o) {
            ops[o].st[0] = 1;
            ops[o].st[1] = ops[o].st[2] = ops[o].st[3] = 0;
            ops[o].ne[0] = cs[0]->count;
            ops[o].ne[1] = ops[o].ne[2] = ops[o].ne[3] = 1;
        }
        return plan_shared(dt, flat_ne, pops, nops, false);
    }
    emel::EwPlan p{};
    p.dtype = dt;
    p.kind = emel::EwKind::Ordinal;
    p.count = cs[0]->count;
    p.ndim = 4;
    for (int d = 0; d < 4; ++d) p.ne[d] = views[0]->ne[d];
    emel::Operand* outs[3] = {&p.dst, &p.src0, &p.src1};
    for (int o = 0; o < nops; ++o) *outs[o] = ops[o];
    return p;
}

// ---------------------------------------------------------------------------
// Row planning.
// ---------------------------------------------------------------------------
emel::RowOperand row_operand(const emel_tensor_view* v, const Checked& c) {
    emel::RowOperand o{};
    o.ptr = static_cast<char*>(v->data);
    for (int d = 0; d < 4; ++d) {
        o.st[d] = (int64_t)(c.nb[d] / c.elem);
        o.ne[d] = v->ne[d];
    }
    return o;
}

bool row_vec_ok(const emel::RowOperand& o) {
    return o.st[0] == 1 && aligned16(o.ptr) && o.st[1] % 4 == 0 && o.st[2] % 4 == 0 && o.st[3] % 4 == 0;
}

emel::RowPlan plan_rows(const emel_tensor_view* src, const Checked& cs, const emel_tensor_view* dst,
                        const Checked* cd) {
    emel::RowPlan p{};
    for (int d = 0; d < 4; ++d) p.ne[d] = src->ne[d];
    p.rows = cs.count / src->ne[0];
    p.src = row_operand(src, cs);
    if (dst) p.dst = row_operand(dst, *cd);
    p.contiguous_rows = p.src.st[0] == 1 && (!dst || p.dst.st[0] == 1);
    p.vec = p.ne[0] % 4 == 0 && row_vec_ok(p.src) && (!dst || row_vec_ok(p.dst));
    p.flat = dense(*src, cs) && aligned16(src->data);
    p.dense = false;
    p.dst_ordinal = false;
    return p;
}

// ---------------------------------------------------------------------------
// Status helpers.
// ---------------------------------------------------------------------------
emel_cuda_status device_status(emel_cuda_context* ctx, cudaError_t err) {
    if (err == cudaSuccess) return EMEL_CUDA_OK;
    std::snprintf(ctx->last_error, sizeof(ctx->last_error), "%s: %s", cudaGetErrorName(err), cudaGetErrorString(err));
    return err == cudaErrorMemoryAllocation ? EMEL_CUDA_OUT_OF_MEMORY : EMEL_CUDA_DEVICE_ERROR;
}

}  // namespace

// Per-stream record of the device bytes written by the library's last
// launch, process-wide (two contexts may share a stream).  A stream not in
// the table, or whose record was taken, is unknown: the next kernel reads
// nothing before its predecessor has finished.
namespace emel {
namespace {
struct StreamRecord {
    cudaStream_t stream;
    uintptr_t lo, hi;
    bool used, known;
};
constexpr int kStreamRecords = 64;
std::mutex g_stream_mu;
StreamRecord g_streams[kStreamRecords];
int g_stream_next = 0;

StreamRecord* stream_slot(cudaStream_t stream) {
    for (auto& r : g_streams)
        if (r.used && r.stream == stream) return &r;
    StreamRecord* r = &g_streams[g_stream_next];
    g_stream_next = (g_stream_next + 1) % kStreamRecords;
    *r = StreamRecord{stream, 0, 0, true, false};
    return r;
}
}  // namespace

void stream_take(cudaStream_t stream, uintptr_t* lo, uintptr_t* hi, bool* known) {
    std::lock_guard<std::mutex> lock(g_stream_mu);
    StreamRecord* r = stream_slot(stream);
    *lo = r->lo;
    *hi = r->hi;
    *known = r->known;
    r->known = false;
}

void stream_wrote(cudaStream_t stream, const void* p, uint64_t bytes) {
    std::lock_guard<std::mutex> lock(g_stream_mu);
    StreamRecord* r = stream_slot(stream);
    r->lo = reinterpret_cast<uintptr_t>(p);
    r->hi = r->lo + bytes;
    r->known = true;
}
}  // namespace emel

namespace {

// Clears the stream's write record (a launch that reports no output range).
void forget_stream(void* stream) {
    uintptr_t lo, hi;
    bool known;
    emel::stream_take(static_cast<cudaStream_t>(stream), &lo, &hi, &known);
}

emel::LaunchEnv env_of(emel_cuda_context* ctx, void* stream) {
    emel::LaunchEnv e{};
    emel::stream_take(static_cast<cudaStream_t>(stream), &e.prev_lo, &e.prev_hi, &e.prev_known);
    e.stream = static_cast<cudaStream_t>(stream);
    e.sm_count = ctx->sm_count;
    e.device = ctx->device;
    e.launches = &ctx->launches;
    e.workspace = ctx->workspace;
    e.workspace_bytes = ctx->workspace_bytes;
    e.tables = ctx->tables;
    return e;
}

// Every launch targets the context's device.
cudaError_t select_device(emel_cuda_context* ctx) {
    int cur = -1;
    cudaError_t err = cudaGetDevice(&cur);
    if (err != cudaSuccess) return err;
    return cur == ctx->device ? cudaSuccess : cudaSetDevice(ctx->device);
}

emel_cuda_status run_unary_plan(emel_cuda_context* ctx, void* stream, const emel::EwPlan& plan, int op, float a,
                                float b) {
    if (ctx == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    cudaError_t err = select_device(ctx);
    if (err == cudaSuccess) err = emel::launch_unary(env_of(ctx, stream), plan, op, a, b);
    return device_status(ctx, err);
}

bool unary_op_known(int op) {
    return (op >= EMEL_UNARY_ABS && op <= EMEL_UNARY_TRUNC && op != EMEL_UNARY_XIELU) ||
           (op >= EMEL_UNARY_SQR && op <= EMEL_UNARY_COS);
}

DType dt_of(uint32_t code) { return code == EMEL_DTYPE_F16 ? DType::F16 : DType::F32; }

// Single-input, same-extent ops over F32 views (activation.rs:327-333,
// elementwise.rs:219-225, tensor_view.rs:1096-1110).
emel_cuda_status same_shape_unary(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                  const emel_tensor_view* dst, int op, float a, float b) {
    Checked cs, cd;
    if (!validate_as(src, EMEL_DTYPE_F32, false, &cs) || !validate_as(dst, EMEL_DTYPE_F32, false, &cd))
        return EMEL_CUDA_INVALID_VIEW;
    if (!same_ne(src, dst)) return EMEL_CUDA_SHAPE_MISMATCH;
    const emel_tensor_view* views[3] = {dst, src, nullptr};
    const Checked* cks[3] = {&cd, &cs, nullptr};
    return run_unary_plan(ctx, stream, plan_equal_count(DType::F32, views, cks, 2), op, a, b);
}

}  // namespace

// ===========================================================================
// extern "C" entry points
// ===========================================================================
extern "C" {

emel_cuda_status emel_cuda_context_create(int device, emel_cuda_context** out) {
    if (out == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    *out = nullptr;
    auto* ctx = new (std::nothrow) emel_cuda_context();
    if (ctx == nullptr) return EMEL_CUDA_OUT_OF_MEMORY;
    ctx->device = device;
    ctx->last_error[0] = '\0';
    cudaError_t err = cudaSetDevice(device);
    if (err == cudaSuccess) err = cudaDeviceGetAttribute(&ctx->sm_count, cudaDevAttrMultiProcessorCount, device);
    if (err == cudaSuccess) {
        ctx->workspace_bytes = emel::reduction_workspace_bytes(ctx->sm_count);
        err = cudaMalloc(&ctx->workspace, ctx->workspace_bytes);
    }
    if (err == cudaSuccess) err = cudaMemset(ctx->workspace, 0, ctx->workspace_bytes);
    // the binary16 domain tables: every table op evaluated once per binary16 input
    if (err == cudaSuccess) err = cudaMalloc(&ctx->tables, emel::kDomainTableBytes);
    if (err == cudaSuccess) err = emel::build_domain_tables(ctx->tables, nullptr);
    if (err == cudaSuccess) err = cudaDeviceSynchronize();
    if (err != cudaSuccess) {
        emel_cuda_status st = device_status(ctx, err);
        if (ctx->workspace) cudaFree(ctx->workspace);
        if (ctx->tables) cudaFree(ctx->tables);
        delete ctx;
        return st;
    }
    *out = ctx;
    return EMEL_CUDA_OK;
}

emel_cuda_status emel_cuda_context_destroy(emel_cuda_context* ctx) {
    if (ctx == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    cudaError_t err = select_device(ctx);
    if (err == cudaSuccess && ctx->workspace) err = cudaFree(ctx->workspace);
    if (err == cudaSuccess && ctx->tables) err = cudaFree(ctx->tables);
    delete ctx;
    return err == cudaSuccess ? EMEL_CUDA_OK : EMEL_CUDA_DEVICE_ERROR;
}

const char* emel_cuda_context_last_error(const emel_cuda_context* ctx) {
    return ctx ? ctx->last_error : "null context";
}

uint64_t emel_cuda_launch_count(const emel_cuda_context* ctx) { return ctx ? ctx->launches : 0; }

emel_cuda_status emel_cuda_malloc(emel_cuda_context* ctx, uint64_t bytes, void** out) {
    if (ctx == nullptr || out == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    cudaError_t err = select_device(ctx);
    if (err == cudaSuccess) err = cudaMalloc(out, bytes);
    return device_status(ctx, err);
}

emel_cuda_status emel_cuda_free(emel_cuda_context* ctx, void* ptr) {
    if (ctx == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    cudaError_t err = select_device(ctx);
    if (err == cudaSuccess) err = cudaFree(ptr);
    return device_status(ctx, err);
}

emel_cuda_status emel_cuda_memcpy_h2d(emel_cuda_context* ctx, void* stream, void* dst, const void* src,
                                      uint64_t bytes) {
    if (ctx == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    cudaError_t err = select_device(ctx);
    forget_stream(stream);  // the stream's last work is now a copy
    if (err == cudaSuccess) err = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, (cudaStream_t)stream);
    return device_status(ctx, err);
}

emel_cuda_status emel_cuda_memcpy_d2h(emel_cuda_context* ctx, void* stream, void* dst, const void* src,
                                      uint64_t bytes) {
    if (ctx == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    cudaError_t err = select_device(ctx);
    forget_stream(stream);
    if (err == cudaSuccess) err = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, (cudaStream_t)stream);
    return device_status(ctx, err);
}

emel_cuda_status emel_cuda_memset(emel_cuda_context* ctx, void* stream, void* dst, int value, uint64_t bytes) {
    if (ctx == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    cudaError_t err = select_device(ctx);
    forget_stream(stream);
    if (err == cudaSuccess) err = cudaMemsetAsync(dst, value, bytes, (cudaStream_t)stream);
    return device_status(ctx, err);
}

emel_cuda_status emel_cuda_stream_create(emel_cuda_context* ctx, void** out) {
    if (ctx == nullptr || out == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    cudaError_t err = select_device(ctx);
    cudaStream_t s = nullptr;
    if (err == cudaSuccess) err = cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking);
    *out = s;
    return device_status(ctx, err);
}

emel_cuda_status emel_cuda_stream_destroy(emel_cuda_context* ctx, void* stream) {
    if (ctx == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    return device_status(ctx, cudaStreamDestroy((cudaStream_t)stream));
}

emel_cuda_status emel_cuda_stream_synchronize(emel_cuda_context* ctx, void* stream) {
    if (ctx == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    const cudaStream_t s = (cudaStream_t)stream;
    cudaError_t err = cudaStreamSynchronize(s);
    // A kernel whose bounded wait expired left the fault word set: report it
    // once and re-arm it.
    // [0] the fault word (offset 64), [2] the rejected-request word (offset 72)
    uint32_t words[3] = {0, 0, 0};
    char* base = static_cast<char*>(ctx->workspace) + emel::kFaultWordOffset;
    static_assert(emel::kRejectWordOffset == emel::kFaultWordOffset + 8, "header words");
    if (err == cudaSuccess) err = cudaMemcpyAsync(words, base, sizeof(words), cudaMemcpyDeviceToHost, s);
    if (err == cudaSuccess) err = cudaStreamSynchronize(s);
    if (err == cudaSuccess && (words[0] != 0 || words[2] != 0)) {
        err = cudaMemsetAsync(base, 0, sizeof(words), s);
        if (err == cudaSuccess) err = cudaStreamSynchronize(s);
        if (err == cudaSuccess) {
            if (words[0] != 0) {
                std::snprintf(ctx->last_error, sizeof(ctx->last_error), "a bounded device wait expired");
                return EMEL_CUDA_TIMEOUT;
            }
            std::snprintf(ctx->last_error, sizeof(ctx->last_error), "a request was rejected on the device (status %u)",
                          words[2]);
            return (emel_cuda_status)words[2];
        }
    }
    return device_status(ctx, err);
}

// ---- events and launch capture ---------------------------------------------

emel_cuda_status emel_cuda_event_create(emel_cuda_context* ctx, void** out) {
    if (ctx == nullptr || out == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    cudaEvent_t e = nullptr;
    cudaError_t err = select_device(ctx);
    if (err == cudaSuccess) err = cudaEventCreate(&e);
    *out = e;
    return device_status(ctx, err);
}

emel_cuda_status emel_cuda_event_record(emel_cuda_context* ctx, void* event, void* stream) {
    if (ctx == nullptr || event == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    forget_stream(stream);
    return device_status(ctx, cudaEventRecord((cudaEvent_t)event, (cudaStream_t)stream));
}

emel_cuda_status emel_cuda_event_record_timed(emel_cuda_context* ctx, void* event, void* stream) {
    if (ctx == nullptr || event == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    forget_stream(stream);
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    cudaError_t err = cudaStreamIsCapturing((cudaStream_t)stream, &cap);
    if (err == cudaSuccess) {
        // inside a capture only an external record becomes a graph node
        err = cap == cudaStreamCaptureStatusActive
                  ? cudaEventRecordWithFlags((cudaEvent_t)event, (cudaStream_t)stream, cudaEventRecordExternal)
                  : cudaEventRecord((cudaEvent_t)event, (cudaStream_t)stream);
    }
    return device_status(ctx, err);
}

emel_cuda_status emel_cuda_event_elapsed_ms(emel_cuda_context* ctx, void* start, void* end, float* ms) {
    if (ctx == nullptr || start == nullptr || end == nullptr || ms == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    return device_status(ctx, cudaEventElapsedTime(ms, (cudaEvent_t)start, (cudaEvent_t)end));
}

emel_cuda_status emel_cuda_event_destroy(emel_cuda_context* ctx, void* event) {
    if (ctx == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    return device_status(ctx, cudaEventDestroy((cudaEvent_t)event));
}

emel_cuda_status emel_cuda_stream_wait_event(emel_cuda_context* ctx, void* stream, void* event) {
    if (ctx == nullptr || event == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    forget_stream(stream);  // what the event covers is not in this stream's record
    return device_status(ctx, cudaStreamWaitEvent((cudaStream_t)stream, (cudaEvent_t)event, 0));
}

}  // extern "C"

struct emel_cuda_graph {
    cudaGraph_t graph;
    cudaGraphExec_t exec;
    uint64_t kernels;  // kernels captured: a replay launches this many
};

namespace {
thread_local uint64_t capture_launch_base = 0;
}

extern "C" {

emel_cuda_status emel_cuda_graph_begin(emel_cuda_context* ctx, void* stream) {
    if (ctx == nullptr || stream == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    cudaError_t err = select_device(ctx);
    if (err == cudaSuccess) err = cudaStreamBeginCapture((cudaStream_t)stream, cudaStreamCaptureModeThreadLocal);
    capture_launch_base = ctx->launches;
    uintptr_t lo, hi;
    bool known;
    emel::stream_take((cudaStream_t)stream, &lo, &hi, &known);  // a captured graph starts with nothing known
    return device_status(ctx, err);
}

emel_cuda_status emel_cuda_graph_end(emel_cuda_context* ctx, void* stream, emel_cuda_graph** out) {
    if (ctx == nullptr || stream == nullptr || out == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    *out = nullptr;
    cudaGraph_t g = nullptr;
    cudaError_t err = cudaStreamEndCapture((cudaStream_t)stream, &g);
    // the captured launches did not run: the stream's real last kernel is
    // whatever ran before the capture, which the record no longer knows
    forget_stream(stream);
    // captured kernels did not run: the replay accounts for them
    const uint64_t captured = ctx->launches - capture_launch_base;
    ctx->launches = capture_launch_base;
    if (err != cudaSuccess) return device_status(ctx, err);
    cudaGraphExec_t exec = nullptr;
    err = cudaGraphInstantiate(&exec, g, 0);
    if (err != cudaSuccess) {
        cudaGraphDestroy(g);
        return device_status(ctx, err);
    }
    auto* h = new (std::nothrow) emel_cuda_graph{g, exec, captured};
    if (h == nullptr) {
        cudaGraphExecDestroy(exec);
        cudaGraphDestroy(g);
        return EMEL_CUDA_OUT_OF_MEMORY;
    }
    *out = h;
    return EMEL_CUDA_OK;
}

emel_cuda_status emel_cuda_graph_launch(emel_cuda_context* ctx, emel_cuda_graph* graph, void* stream) {
    if (ctx == nullptr || graph == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    cudaError_t err = select_device(ctx);
    forget_stream(stream);  // the graph's writes are not in the record
    if (err == cudaSuccess) err = cudaGraphLaunch(graph->exec, (cudaStream_t)stream);
    if (err == cudaSuccess) ctx->launches += graph->kernels;
    return device_status(ctx, err);
}

// ---- peer exchange over NVLink ----------------------------------------------

}  // extern "C"

struct emel_cuda_exchange {
    int device;
    int world;
    int rank;
    uint32_t bytes;
    uint64_t timeout_ns;
    char* buffer;      // this rank's buffer (cudaMalloc, shared by IPC)
    uint32_t* epoch;   // this rank's step counter (device)
    char* peers[emel::kExchangeMaxRanks];
    bool opened[emel::kExchangeMaxRanks];  // peers[r] came from cudaIpcOpenMemHandle
    bool connected;
};

namespace {

static_assert(sizeof(cudaIpcMemHandle_t) == EMEL_CUDA_EXCHANGE_HANDLE_BYTES, "IPC handle size");

void exchange_close_peers(emel_cuda_exchange* ex) {
    for (int r = 0; r < emel::kExchangeMaxRanks; ++r) {
        if (ex->opened[r]) cudaIpcCloseMemHandle(ex->peers[r]);
        ex->opened[r] = false;
        ex->peers[r] = nullptr;
    }
    ex->connected = false;
}

bool aligned16_ptr(const void* p) { return p != nullptr && (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

emel::ExchangeArgs exchange_args(emel_cuda_context* ctx, const emel_cuda_exchange* ex, const void* payload) {
    emel::ExchangeArgs a{};
    for (int r = 0; r < ex->world; ++r) a.peers[r] = ex->peers[r];
    a.payload = payload;
    a.epoch = ex->epoch;
    a.fault = reinterpret_cast<uint32_t*>(static_cast<char*>(ctx->workspace) + emel::kFaultWordOffset);
    a.world = ex->world;
    a.rank = ex->rank;
    a.bytes = ex->bytes;
    a.slot_bytes = ex->bytes;
    a.timeout_ns = ex->timeout_ns;
    return a;
}

}  // namespace

extern "C" {

emel_cuda_status emel_cuda_exchange_create(emel_cuda_context* ctx, int world, int rank, uint32_t bytes_per_rank,
                                           uint32_t timeout_ms, emel_cuda_exchange** out) {
    if (ctx == nullptr || out == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    *out = nullptr;
    if (world < 1 || world > emel::kExchangeMaxRanks || rank < 0 || rank >= world || bytes_per_rank == 0 ||
        bytes_per_rank % 16 != 0 || bytes_per_rank > emel::kExchangeMaxBytes || timeout_ms == 0)
        return EMEL_CUDA_INVALID_ARGUMENT;
    cudaError_t err = select_device(ctx);
    if (err != cudaSuccess) return device_status(ctx, err);
    auto* ex = new (std::nothrow) emel_cuda_exchange();
    if (ex == nullptr) return EMEL_CUDA_OUT_OF_MEMORY;
    ex->device = ctx->device;
    ex->world = world;
    ex->rank = rank;
    ex->bytes = bytes_per_rank;
    ex->timeout_ns = (uint64_t)timeout_ms * 1000000ull;
    const uint64_t bytes = emel::exchange_buffer_bytes(bytes_per_rank);
    err = cudaMalloc(&ex->buffer, bytes);
    if (err == cudaSuccess) err = cudaMalloc(&ex->epoch, 16);
    if (err == cudaSuccess) err = cudaMemset(ex->buffer, 0, bytes);
    if (err == cudaSuccess) err = cudaMemset(ex->epoch, 0, 16);
    if (err == cudaSuccess) err = cudaDeviceSynchronize();
    if (err != cudaSuccess) {
        emel_cuda_status st = device_status(ctx, err);
        if (ex->buffer) cudaFree(ex->buffer);
        if (ex->epoch) cudaFree(ex->epoch);
        delete ex;
        return st;
    }
    *out = ex;
    return EMEL_CUDA_OK;
}

emel_cuda_status emel_cuda_exchange_handle(const emel_cuda_exchange* ex, void* handle_out) {
    if (ex == nullptr || handle_out == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    if (cudaSetDevice(ex->device) != cudaSuccess) return EMEL_CUDA_DEVICE_ERROR;
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, ex->buffer) != cudaSuccess) return EMEL_CUDA_DEVICE_ERROR;
    std::memcpy(handle_out, &h, sizeof(h));
    return EMEL_CUDA_OK;
}

emel_cuda_status emel_cuda_exchange_connect(emel_cuda_context* ctx, emel_cuda_exchange* ex, const void* handles) {
    if (ctx == nullptr || ex == nullptr || handles == nullptr || ex->connected) return EMEL_CUDA_INVALID_ARGUMENT;
    cudaError_t err = select_device(ctx);
    if (err != cudaSuccess) return device_status(ctx, err);
    const auto* h = static_cast<const unsigned char*>(handles);
    for (int r = 0; r < ex->world; ++r) {
        if (r == ex->rank) {
            ex->peers[r] = ex->buffer;
            continue;
        }
        cudaIpcMemHandle_t hr;
        std::memcpy(&hr, h + (size_t)r * sizeof(hr), sizeof(hr));
        void* p = nullptr;
        err = cudaIpcOpenMemHandle(&p, hr, cudaIpcMemLazyEnablePeerAccess);
        if (err != cudaSuccess) {
            exchange_close_peers(ex);
            return device_status(ctx, err);
        }
        ex->peers[r] = static_cast<char*>(p);
        ex->opened[r] = true;
    }
    ex->connected = true;
    return EMEL_CUDA_OK;
}

emel_cuda_status emel_cuda_exchange_publish(emel_cuda_context* ctx, void* stream, emel_cuda_exchange* ex,
                                            const void* payload) {
    if (ctx == nullptr || ex == nullptr || !ex->connected || !aligned16_ptr(payload)) return EMEL_CUDA_INVALID_ARGUMENT;
    cudaError_t err = select_device(ctx);
    forget_stream(stream);
    if (err == cudaSuccess) err = emel::launch_exchange_publish((cudaStream_t)stream, exchange_args(ctx, ex, payload));
    if (err == cudaSuccess) ++ctx->launches;
    return device_status(ctx, err);
}

emel_cuda_status emel_cuda_exchange_wait(emel_cuda_context* ctx, void* stream, emel_cuda_exchange* ex,
                                         void* gathered) {
    if (ctx == nullptr || ex == nullptr || !ex->connected || !aligned16_ptr(gathered)) return EMEL_CUDA_INVALID_ARGUMENT;
    cudaError_t err = select_device(ctx);
    forget_stream(stream);
    if (err == cudaSuccess)
        err = emel::launch_exchange_wait((cudaStream_t)stream, exchange_args(ctx, ex, nullptr), gathered);
    if (err == cudaSuccess) ++ctx->launches;
    return device_status(ctx, err);
}

static bool scalar_shape(const emel_tensor_view* v);
static bool index_view(const emel_tensor_view* v, Checked* c);

emel_cuda_status emel_cuda_exchange_wait_sum_argmax(emel_cuda_context* ctx, void* stream, emel_cuda_exchange* ex,
                                                    void* gathered, const emel_tensor_view* sum_dst,
                                                    const emel_tensor_view* argmax_dst) {
    if (sum_dst == nullptr || argmax_dst == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    Checked cs, ci;
    // the destinations of OpSum and OpArgmax (reductions.rs:452-458, 520-530)
    if (!validate_as(sum_dst, EMEL_DTYPE_F32, false, &cs) || !index_view(argmax_dst, &ci)) return EMEL_CUDA_INVALID_VIEW;
    if (!scalar_shape(sum_dst) || !scalar_shape(argmax_dst)) return EMEL_CUDA_SHAPE_MISMATCH;
    if (ctx == nullptr || ex == nullptr || !ex->connected || !aligned16_ptr(gathered) ||
        ex->bytes != 8 + sizeof(emel_cuda_argmax_partial))
        return EMEL_CUDA_INVALID_ARGUMENT;
    cudaError_t err = select_device(ctx);
    forget_stream(stream);
    if (err == cudaSuccess) {
        const emel::CombineOut out{sum_dst->data, argmax_dst->data, (int)argmax_dst->dtype};
        err = emel::launch_exchange_wait_combine((cudaStream_t)stream, exchange_args(ctx, ex, nullptr), gathered, out);
    }
    if (err == cudaSuccess) ++ctx->launches;
    return device_status(ctx, err);
}

emel_cuda_status emel_cuda_exchange_destroy(emel_cuda_context* ctx, emel_cuda_exchange* ex) {
    if (ctx == nullptr || ex == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    cudaError_t err = select_device(ctx);
    exchange_close_peers(ex);
    if (err == cudaSuccess) err = cudaFree(ex->buffer);
    const cudaError_t err2 = cudaFree(ex->epoch);
    delete ex;
    return device_status(ctx, err != cudaSuccess ? err : err2);
}

emel_cuda_status emel_cuda_graph_destroy(emel_cuda_context* ctx, emel_cuda_graph* graph) {
    if (ctx == nullptr || graph == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    cudaError_t err = cudaGraphExecDestroy(graph->exec);
    cudaError_t err2 = cudaGraphDestroy(graph->graph);
    delete graph;
    return device_status(ctx, err != cudaSuccess ? err : err2);
}

// ---- binary family ---------------------------------------------------------

emel_cuda_status emel_cuda_binary(emel_cuda_context* ctx, void* stream, int op, const emel_tensor_view* lhs,
                                  const emel_tensor_view* rhs, const emel_tensor_view* dst) {
    if (op < EMEL_BINARY_ADD || op > EMEL_BINARY_DIV) return EMEL_CUDA_UNEXPECTED_EVENT;
    Checked cl, cr, cd;
    // binary.rs:336-345: all three views under the singleton-zero-stride contract
    if (!validate_float(lhs, true, &cl) || !validate_float(rhs, true, &cr) || !validate_float(dst, true, &cd) ||
        lhs->dtype != rhs->dtype || lhs->dtype != dst->dtype)
        return EMEL_CUDA_INVALID_VIEW;
    // binary.rs:347-354: equal logical element counts
    if (cl.count != cr.count || cl.count != cd.count) return EMEL_CUDA_SHAPE_MISMATCH;
    if (ctx == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    const emel_tensor_view* views[3] = {dst, lhs, rhs};
    const Checked* cks[3] = {&cd, &cl, &cr};
    const emel::EwPlan plan = plan_equal_count(dt_of(dst->dtype), views, cks, 3);
    cudaError_t err = select_device(ctx);
    if (err == cudaSuccess) err = emel::launch_binary(env_of(ctx, stream), plan, op);
    return device_status(ctx, err);
}

static emel_cuda_status broadcast_common(emel_cuda_context* ctx, void* stream, int op, const emel_tensor_view* src0,
                                         const emel_tensor_view* src1, const emel_tensor_view* dst, bool row_contract) {
    if (op < EMEL_BINARY_ADD || op > EMEL_BINARY_DIV) return EMEL_CUDA_UNEXPECTED_EVENT;
    Checked c0, c1, cd;
    if (!validate_float(src0, true, &c0) || !validate_float(src1, true, &c1) || !validate_float(dst, true, &cd) ||
        src0->dtype != src1->dtype || src0->dtype != dst->dtype)
        return EMEL_CUDA_INVALID_VIEW;
    if (row_contract) {
        // broadcast.rs:334-350
        const bool ok = same_ne(src0, dst) && dst->ne[0] > 0 && src1->ne[0] == dst->ne[0] && src1->ne[1] == 1 &&
                        src1->ne[2] == 1 && src1->ne[3] == 1 && dst->ne[1] > 0 && cd.count > c1.count;
        if (!ok) return EMEL_CUDA_SHAPE_MISMATCH;
    } else {
        // ggml repeat contract: src0 and dst share extents; src1 extents divide them
        if (!same_ne(src0, dst)) return EMEL_CUDA_SHAPE_MISMATCH;
        for (int d = 0; d < 4; ++d)
            if (dst->ne[d] % src1->ne[d] != 0) return EMEL_CUDA_SHAPE_MISMATCH;
    }
    if (ctx == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    emel::Operand ops[3] = {operand(dst, cd), operand(src0, c0), operand(src1, c1)};
    emel::Operand* pops[3] = {&ops[0], &ops[1], &ops[2]};
    const bool bcast = !same_ne(src1, dst);
    const emel::EwPlan plan = plan_shared(dt_of(dst->dtype), dst->ne, pops, 3, bcast);
    cudaError_t err = select_device(ctx);
    if (err == cudaSuccess) err = emel::launch_binary(env_of(ctx, stream), plan, op);
    return device_status(ctx, err);
}

emel_cuda_status emel_cuda_broadcast_row(emel_cuda_context* ctx, void* stream, int op, const emel_tensor_view* src0,
                                         const emel_tensor_view* src1, const emel_tensor_view* dst) {
    return broadcast_common(ctx, stream, op, src0, src1, dst, true);
}

emel_cuda_status emel_cuda_binary_repeat(emel_cuda_context* ctx, void* stream, int op, const emel_tensor_view* src0,
                                         const emel_tensor_view* src1, const emel_tensor_view* dst) {
    return broadcast_common(ctx, stream, op, src0, src1, dst, false);
}

// ---- unary family ------------------------------------------------------------

emel_cuda_status emel_cuda_unary(emel_cuda_context* ctx, void* stream, int op, const emel_tensor_view* src,
                                 const emel_tensor_view* dst) {
    if (!unary_op_known(op)) return EMEL_CUDA_UNEXPECTED_EVENT;
    Checked cs, cd;
    // unary.rs:455-461
    if (!validate_float(src, false, &cs) || !validate_float(dst, false, &cd) || src->dtype != dst->dtype)
        return EMEL_CUDA_INVALID_VIEW;
    if (cs.count != cd.count) return EMEL_CUDA_SHAPE_MISMATCH;
    const emel_tensor_view* views[3] = {dst, src, nullptr};
    const Checked* cks[3] = {&cd, &cs, nullptr};
    if (ctx == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    return run_unary_plan(ctx, stream, plan_equal_count(dt_of(dst->dtype), views, cks, 2), op, 0.0f, 0.0f);
}

emel_cuda_status emel_cuda_op_unary(emel_cuda_context* ctx, void* stream, int subop, const emel_tensor_view* src,
                                    const emel_tensor_view* dst) {
    // unary.rs:942-1027: eight accepted subops; any failure is UnexpectedEvent
    const bool accepted = subop == EMEL_UNARY_ABS || subop == EMEL_UNARY_NEG || subop == EMEL_UNARY_TANH ||
                          subop == EMEL_UNARY_ELU || subop == EMEL_UNARY_RELU || subop == EMEL_UNARY_GELU ||
                          subop == EMEL_UNARY_SILU || subop == EMEL_UNARY_EXP;
    Checked cs, cd;
    if (!accepted || !validate_as(src, EMEL_DTYPE_F32, false, &cs) || !validate_as(dst, EMEL_DTYPE_F32, false, &cd) ||
        cs.count != cd.count)
        return EMEL_CUDA_UNEXPECTED_EVENT;
    if (ctx == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    const emel_tensor_view* views[3] = {dst, src, nullptr};
    const Checked* cks[3] = {&cd, &cs, nullptr};
    return run_unary_plan(ctx, stream, plan_equal_count(DType::F32, views, cks, 2), subop, 0.0f, 0.0f);
}

emel_cuda_status emel_cuda_scale(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                 const emel_tensor_view* dst, float scale) {
    return same_shape_unary(ctx, stream, src, dst, emel::kScale, scale, 0.0f);
}

emel_cuda_status emel_cuda_clamp(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                 const emel_tensor_view* dst, float min, float max) {
    return same_shape_unary(ctx, stream, src, dst, emel::kClamp, min, max);
}

emel_cuda_status emel_cuda_leaky_relu(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                      const emel_tensor_view* dst, float negative_slope) {
    return same_shape_unary(ctx, stream, src, dst, emel::kLeakyRelu, negative_slope, 0.0f);
}

emel_cuda_status emel_cuda_add1(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                const emel_tensor_view* dst, float scalar) {
    return same_shape_unary(ctx, stream, src, dst, emel::kAdd1, scalar, 0.0f);
}

emel_cuda_status emel_cuda_copy(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                const emel_tensor_view* dst) {
    return same_shape_unary(ctx, stream, src, dst, emel::kCopy, 0.0f, 0.0f);
}

// shape.rs OpCpy / OpCont: count-equal ordinal copy (unary plan with the
// identity formula: a load and a store per element, bits unchanged).
static bool dense_contiguous_f32(const emel_tensor_view* v) {
    if (v->dtype != EMEL_DTYPE_F32) return false;
    uint64_t expected = 4;
    for (int d = 0; d < 4; ++d) {
        if (v->nb[d] != expected) return false;
        if (__builtin_mul_overflow(expected, v->ne[d], &expected)) return false;
    }
    return true;
}

static emel_cuda_status shape_copy(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                   const emel_tensor_view* dst, bool cont) {
    Checked cs, cd;
    if (!validate_as(src, EMEL_DTYPE_F32, false, &cs) || !validate_as(dst, EMEL_DTYPE_F32, false, &cd))
        return EMEL_CUDA_INVALID_VIEW;
    if (cs.count != cd.count) return EMEL_CUDA_SHAPE_MISMATCH;
    if (cont && !dense_contiguous_f32(dst)) return EMEL_CUDA_INVALID_LAYOUT;
    if (ctx == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    const emel_tensor_view* views[3] = {dst, src, nullptr};
    const Checked* cks[3] = {&cd, &cs, nullptr};
    return run_unary_plan(ctx, stream, plan_equal_count(DType::F32, views, cks, 2), emel::kCopy, 0.0f, 0.0f);
}

emel_cuda_status emel_cuda_cpy(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                               const emel_tensor_view* dst) {
    return shape_copy(ctx, stream, src, dst, false);
}

emel_cuda_status emel_cuda_cont(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                const emel_tensor_view* dst) {
    return shape_copy(ctx, stream, src, dst, true);
}

emel_cuda_status emel_cuda_silu_back(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                     const emel_tensor_view* grad, const emel_tensor_view* dst) {
    Checked cs, cg, cd;
    // activation.rs:335-349
    if (!validate_as(src, EMEL_DTYPE_F32, false, &cs) || !validate_as(grad, EMEL_DTYPE_F32, false, &cg) ||
        !validate_as(dst, EMEL_DTYPE_F32, false, &cd))
        return EMEL_CUDA_INVALID_VIEW;
    if (!same_ne(src, grad) || !same_ne(src, dst)) return EMEL_CUDA_SHAPE_MISMATCH;
    if (ctx == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    const emel_tensor_view* views[3] = {dst, src, grad};
    const Checked* cks[3] = {&cd, &cs, &cg};
    const emel::EwPlan plan = plan_equal_count(DType::F32, views, cks, 3);
    cudaError_t err = select_device(ctx);
    if (err == cudaSuccess) err = emel::launch_binary(env_of(ctx, stream), plan, emel::kSiluBack);
    return device_status(ctx, err);
}

// ---- row gather (get_rows.rs) -------------------------------------------------

namespace {

struct GrIndex {
    uint64_t ne[3] = {0, 0, 0};
    uint64_t st[3] = {0, 0, 0};  // elements
    uint64_t count = 0;
    bool valid = false;
};

// IndexView::with_strides (get_rows.rs:44-139, 180-215) over an I32 view
// with ne[3] == 1; nb[0] == 0 selects the implicit contiguous strides.
GrIndex gr_index_view(const emel_tensor_view* v) {
    GrIndex x;
    if (v == nullptr || v->dtype != EMEL_DTYPE_I32 || v->ne[3] != 1 || v->reserved != 0) return x;
    uint64_t bs[3];
    bool strides_valid = true, shape_valid = true, zero = false;
    const bool implicit = v->nb[0] == 0;
    if (implicit) {
        bs[0] = 4;
        for (int d = 1; d < 3; ++d)
            if (__builtin_mul_overflow(bs[d - 1], v->ne[d - 1], &bs[d])) {
                strides_valid = false;
                bs[d] = 0;
            }
    } else {
        for (int d = 0; d < 3; ++d) bs[d] = v->nb[d];
    }
    uint64_t count = 1;
    for (int d = 0; d < 3; ++d) {
        x.ne[d] = v->ne[d];
        if (v->ne[d] > 1 && bs[d] == 0 && !implicit) strides_valid = false;
        if (bs[d] != 0 && (bs[d] < 4 || bs[d] % 4 != 0)) strides_valid = false;
        x.st[d] = bs[d] / 4;
        if (v->ne[d] == 0) zero = true;
        else if (!zero && __builtin_mul_overflow(count, v->ne[d], &count)) {
            shape_valid = false;
            count = 0;
        }
    }
    if (zero) count = 0;
    bool span = true;
    if (!zero) {
        u128 max_offset = 0;
        for (int d = 0; d < 3; ++d) max_offset += (u128)(v->ne[d] - 1) * (u128)bs[d];
        span = max_offset + 4 <= (u128)(v->storage_bytes / 4) * 4;
    }
    x.count = count;
    x.valid = strides_valid && shape_valid && span && (zero || v->data != nullptr);
    return x;
}

bool gr_empty_f32_source_valid(const emel_tensor_view* v) {
    if (v->dtype != EMEL_DTYPE_F32 || v->ne[0] == 0 || v->ne[1] == 0 || (v->nb[0] != 0 && v->nb[0] != 4)) return false;
    if (v->nb[0] != 0)
        for (int d = 0; d < 4; ++d)
            if (v->ne[d] > 1 && v->nb[d] == 0) return false;
    return true;
}

bool gr_destination_valid(const emel_tensor_view* dst, uint64_t count) {
    Checked cd;
    if (count == 0) return dst->dtype == EMEL_DTYPE_F32 && dense_contiguous_f32(dst);
    return validate_as(dst, EMEL_DTYPE_F32, false, &cd) && dense_contiguous_f32(dst);
}

// F16View::validate (f16_matmul.rs:45-85) / Bf16View::validate (get_rows.rs:300-340)
bool gr_half_view_valid(const emel_tensor_view* v, uint32_t dtype, uint64_t s[4]) {
    if (v->dtype != dtype || v->data == nullptr) return false;
    uint64_t count = 1;
    for (int d = 0; d < 4; ++d)
        if (v->ne[d] == 0 || __builtin_mul_overflow(count, v->ne[d], &count)) return false;
    if (v->nb[0] != 0) {
        for (int d = 0; d < 4; ++d) s[d] = v->nb[d];
    } else {
        s[0] = 2;
        for (int d = 1; d < 4; ++d)
            if (__builtin_mul_overflow(s[d - 1], v->ne[d - 1], &s[d])) return false;
    }
    for (int d = 0; d < 4; ++d) {
        if (dtype == EMEL_DTYPE_F16) {
            if (v->ne[d] > 1 && (s[d] < 2 || s[d] % 2 != 0)) return false;
        } else if (v->nb[0] != 0) {
            if ((v->ne[d] > 1 && v->nb[d] == 0) || (v->nb[d] != 0 && (v->nb[d] < 2 || v->nb[d] % 2 != 0)))
                return false;
        }
    }
    u128 max_offset = 0;
    for (int d = 0; d < 4; ++d) max_offset += (u128)(v->ne[d] - 1) * (u128)s[d];
    return max_offset + 2 <= (u128)(v->storage_bytes / 2) * 2;
}

// PackedRowView::validate (tensor_view.rs:483-526)
bool gr_packed_view_valid(const emel_tensor_view* v, uint32_t code, uint64_t bv, uint64_t bb, uint64_t* row_bytes) {
    if (v->dtype != code || v->data == nullptr) return false;
    for (int d = 0; d < 4; ++d)
        if (v->ne[d] == 0) return false;
    if (v->ne[0] % bv != 0 || v->nb[0] != 1) return false;
    uint64_t rb, s2, s3;
    if (__builtin_mul_overflow(v->ne[0] / bv, bb, &rb)) return false;
    if (__builtin_mul_overflow(rb, v->ne[1], &s2)) return false;
    if (__builtin_mul_overflow(s2, v->ne[2], &s3)) return false;
    if (rb == 0 || v->nb[1] != rb || v->nb[2] != s2 || v->nb[3] != s3) return false;
    u128 max_offset = 0;
    for (int d = 1; d < 4; ++d) max_offset += (u128)(v->ne[d] - 1) * (u128)v->nb[d];
    *row_bytes = rb;
    return max_offset + rb <= (u128)v->storage_bytes;
}

bool gr_shape_valid(const emel_tensor_view* src, const GrIndex& x, const emel_tensor_view* dst) {
    return src->ne[0] > 0 && src->ne[1] > 0 && dst->ne[0] == src->ne[0] && dst->ne[1] == x.ne[0] &&
           dst->ne[2] == x.ne[1] && dst->ne[3] == x.ne[2] && src->ne[2] == x.ne[1] && src->ne[3] == x.ne[2];
}

}  // namespace

emel_cuda_status emel_cuda_get_rows(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                    const emel_tensor_view* indices, const emel_tensor_view* dst) {
    if (src == nullptr || indices == nullptr || dst == nullptr) return EMEL_CUDA_INVALID_VIEW;
    const GrIndex ix = gr_index_view(indices);
    const uint32_t t = src->dtype;
    emel::GatherPlan p{};
    uint64_t hs[4] = {0, 0, 0, 0}, row_bytes = 0, fs[4] = {0, 0, 0, 0};
    bool views = false;
    Checked cs;
    switch (t) {
    case EMEL_DTYPE_F32:
        p.kind = emel::kGatherF32;
        views = ix.valid && (ix.count == 0 ? gr_empty_f32_source_valid(src) : validate_as(src, EMEL_DTYPE_F32, true, &cs)) &&
                gr_destination_valid(dst, ix.count);
        break;
    case EMEL_DTYPE_F16:
    case EMEL_DTYPE_BF16: {
        p.kind = t == EMEL_DTYPE_F16 ? emel::kGatherF16 : emel::kGatherBF16;
        Checked cd;
        views = ix.valid && gr_half_view_valid(src, t, hs) && validate_as(dst, EMEL_DTYPE_F32, false, &cd) &&
                dense_contiguous_f32(dst);
        break;
    }
    case EMEL_DTYPE_Q4_0:
    case EMEL_DTYPE_Q8_0:
    case EMEL_DTYPE_Q4_K: {
        p.kind = t == EMEL_DTYPE_Q4_0 ? emel::kGatherQ4_0 : (t == EMEL_DTYPE_Q8_0 ? emel::kGatherQ8_0 : emel::kGatherQ4_K);
        const uint64_t bv = t == EMEL_DTYPE_Q4_K ? 256 : 32;
        const uint64_t bb = t == EMEL_DTYPE_Q4_0 ? 18 : (t == EMEL_DTYPE_Q8_0 ? 34 : 144);
        Checked cd;
        views = ix.valid && gr_packed_view_valid(src, t, bv, bb, &row_bytes) &&
                (ix.count == 0 ? dense_contiguous_f32(dst)
                               : (validate_as(dst, EMEL_DTYPE_F32, false, &cd) && dense_contiguous_f32(dst))) &&
                dst->dtype == EMEL_DTYPE_F32;
        break;
    }
    default:
        return EMEL_CUDA_INVALID_VIEW;
    }
    // get_rows.rs guard order: view, shape, source stride (F32), indices (on the device)
    if (!views) return EMEL_CUDA_INVALID_VIEW;
    if (!gr_shape_valid(src, ix, dst)) return EMEL_CUDA_SHAPE_MISMATCH;
    if (t == EMEL_DTYPE_F32 && !(src->nb[0] == 0 || (src->nb[0] >= 4 && src->nb[0] % 4 == 0)))
        return EMEL_CUDA_UNSUPPORTED_SOURCE_STRIDE;
    if (ctx == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    if (ix.count == 0) return EMEL_CUDA_OK;  // the reference's metadata-only no-op
    // device additions: element-aligned pointers
    const uintptr_t sa = reinterpret_cast<uintptr_t>(src->data), ia = reinterpret_cast<uintptr_t>(indices->data);
    const uintptr_t da = reinterpret_cast<uintptr_t>(dst->data);
    if ((ia & 3u) || (da & 3u) || (t == EMEL_DTYPE_F32 ? (sa & 3u) : (sa & 1u)) ||
        (t == EMEL_DTYPE_F32 && (src->nb[1] % 4 || src->nb[2] % 4 || src->nb[3] % 4)))
        return EMEL_CUDA_INVALID_ARGUMENT;
    p.src = static_cast<const char*>(src->data);
    p.dst = static_cast<float*>(dst->data);
    p.idx = static_cast<const int32_t*>(indices->data);
    for (int d = 0; d < 3; ++d) {
        p.idx_ne[d] = ix.ne[d];
        p.idx_st[d] = (int64_t)ix.st[d];
    }
    p.cols = src->ne[0];
    p.rows = src->ne[1];
    p.batches = src->ne[2];
    p.row_bytes = row_bytes;
    p.dst_rows = ix.count;
    if (t == EMEL_DTYPE_F32) {
        for (int d = 0; d < 4; ++d) fs[d] = cs.nb[d];
        for (int d = 0; d < 4; ++d) p.src_st[d] = (int64_t)fs[d];
        p.vec = p.cols % 4 == 0 && (da & 15u) == 0;
    } else if (t == EMEL_DTYPE_F16 || t == EMEL_DTYPE_BF16) {
        for (int d = 0; d < 4; ++d) p.src_st[d] = (int64_t)hs[d];
        p.vec = hs[0] == 2 && p.cols % 8 == 0 && (da & 15u) == 0;
    }
    char* ws = static_cast<char*>(ctx->workspace);
    p.flag = reinterpret_cast<uint32_t*>(ws + emel::kCallFlagOffset);
    p.reject = reinterpret_cast<uint32_t*>(ws + emel::kRejectWordOffset);
    p.reject_code = EMEL_CUDA_INDEX_OUT_OF_BOUNDS;
    cudaError_t err = select_device(ctx);
    if (err == cudaSuccess) err = emel::launch_get_rows(env_of(ctx, stream), p);
    return device_status(ctx, err);
}

namespace {

// ByteTensorView::validate (tensor_view.rs:588-643) with a non-null buffer;
// `s` receives Layout::effective_f32_strides (tensor_view.rs:262-277).
bool gr_byte_view_valid(const emel_tensor_view* v, uint64_t s[4]) {
    if (v->dtype != EMEL_DTYPE_F32 || v->data == nullptr) return false;
    uint64_t count = 1;
    for (int d = 0; d < 4; ++d)
        if (v->ne[d] == 0 || __builtin_mul_overflow(count, v->ne[d], &count)) return false;
    if (v->nb[0] != 0 && (v->nb[0] < 4 || v->nb[0] % 4 != 0)) return false;
    if (v->nb[0] != 0) {
        for (int d = 0; d < 4; ++d)
            if (v->ne[d] > 1 && v->nb[d] == 0) return false;
        for (int d = 0; d < 4; ++d) s[d] = v->nb[d];
    } else {
        s[0] = 4;
        for (int d = 1; d < 4; ++d)
            if (__builtin_mul_overflow(s[d - 1], v->ne[d - 1], &s[d])) return false;
    }
    u128 max_offset = 0;
    for (int d = 1; d < 4; ++d) max_offset += (u128)(v->ne[d] - 1) * (u128)s[d];
    return max_offset + (u128)v->ne[0] * 4 <= (u128)v->storage_bytes;
}

// empty_f32_bytes_source_valid (get_rows.rs:951-971)
bool gr_byte_empty_valid(const emel_tensor_view* v) {
    if (v->dtype != EMEL_DTYPE_F32 || v->ne[0] == 0 || v->ne[1] == 0) return false;
    if (v->nb[0] != 0 && (v->nb[0] < 4 || v->nb[0] % 4 != 0)) return false;
    if (v->nb[0] != 0)
        for (int d = 0; d < 4; ++d)
            if (v->ne[d] > 1 && v->nb[d] == 0) return false;
    return true;
}

}  // namespace

emel_cuda_status emel_cuda_get_rows_f32_bytes(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                              const emel_tensor_view* indices, const emel_tensor_view* dst) {
    if (src == nullptr || indices == nullptr || dst == nullptr) return EMEL_CUDA_INVALID_VIEW;
    const GrIndex ix = gr_index_view(indices);
    uint64_t s[4] = {0, 0, 0, 0};
    const bool views = ix.valid && (ix.count == 0 ? gr_byte_empty_valid(src) : gr_byte_view_valid(src, s)) &&
                       gr_destination_valid(dst, ix.count);
    // get_rows.rs guard order: view, shape, indices (on the device)
    if (!views) return EMEL_CUDA_INVALID_VIEW;
    if (!gr_shape_valid(src, ix, dst)) return EMEL_CUDA_SHAPE_MISMATCH;
    if (ctx == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    if (ix.count == 0) return EMEL_CUDA_OK;
    const uintptr_t ia = reinterpret_cast<uintptr_t>(indices->data), da = reinterpret_cast<uintptr_t>(dst->data);
    if ((ia & 3u) || (da & 3u)) return EMEL_CUDA_INVALID_ARGUMENT;
    emel::GatherPlan p{};
    p.kind = emel::kGatherF32Bytes;
    p.src = static_cast<const char*>(src->data);
    p.dst = static_cast<float*>(dst->data);
    p.idx = static_cast<const int32_t*>(indices->data);
    for (int d = 0; d < 3; ++d) {
        p.idx_ne[d] = ix.ne[d];
        p.idx_st[d] = (int64_t)ix.st[d];
    }
    p.cols = src->ne[0];
    p.rows = src->ne[1];
    p.batches = src->ne[2];
    p.dst_rows = ix.count;
    for (int d = 0; d < 4; ++d) p.src_st[d] = (int64_t)s[d];
    p.vec = p.cols % 4 == 0 && (da & 15u) == 0;
    char* ws = static_cast<char*>(ctx->workspace);
    p.flag = reinterpret_cast<uint32_t*>(ws + emel::kCallFlagOffset);
    p.reject = reinterpret_cast<uint32_t*>(ws + emel::kRejectWordOffset);
    p.reject_code = EMEL_CUDA_INDEX_OUT_OF_BOUNDS;
    cudaError_t err = select_device(ctx);
    if (err == cudaSuccess) err = emel::launch_get_rows(env_of(ctx, stream), p);
    return device_status(ctx, err);
}

// ---- rotary position embedding (rope.rs) -----------------------------------

static bool rope_positions_valid(const emel_tensor_view* v) {
    // Layout::validate_i32 (tensor_view.rs:388-447): raw strides, each >= 4 and a multiple of 4
    if (v == nullptr || v->dtype != EMEL_DTYPE_I32 || v->data == nullptr || v->reserved != 0) return false;
    uint64_t count = 1;
    for (int d = 0; d < 4; ++d) {
        if (v->ne[d] == 0 || __builtin_mul_overflow(count, v->ne[d], &count)) return false;
        if (v->nb[d] < 4 || v->nb[d] % 4 != 0) return false;
    }
    u128 max_offset = 0;
    for (int d = 0; d < 4; ++d) max_offset += (u128)(v->ne[d] - 1) * (u128)v->nb[d];
    return max_offset + 4 <= (u128)(v->storage_bytes / 4) * 4;
}

static bool dense_contiguous_i32(const emel_tensor_view* v) {
    if (v->dtype != EMEL_DTYPE_I32) return false;
    uint64_t expected = 4;
    for (int d = 0; d < 4; ++d) {
        if (v->nb[d] != expected) return false;
        if (__builtin_mul_overflow(expected, v->ne[d], &expected)) return false;
    }
    return true;
}

emel_cuda_status emel_cuda_rope(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                const emel_tensor_view* positions, const emel_tensor_view* dst,
                                const emel_rope_params* params) {
    if (params == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    Checked cs, cd;
    // rope.rs:338-440, transitions in order: view, parameters, mode / shape
    if (src == nullptr || dst == nullptr || !validate_as(src, EMEL_DTYPE_F32, false, &cs) ||
        !rope_positions_valid(positions) || !validate_as(dst, EMEL_DTYPE_F32, false, &cd))
        return EMEL_CUDA_INVALID_VIEW;
    const emel_rope_params pr = *params;
    const uint64_t cols = src->ne[0];
    const bool params_ok = pr.n_dims > 0 && pr.n_dims % 2 == 0 && (uint64_t)pr.n_dims <= cols &&
                           pr.ext_factor == 0.0f && std::isfinite(pr.freq_base) && pr.freq_base > 0.0f &&
                           std::isfinite(pr.freq_scale) && pr.freq_scale > 0.0f && std::isfinite(pr.attn_factor);
    if (!params_ok) return EMEL_CUDA_INVALID_PARAMETERS;
    const bool shape_ok = same_ne(src, dst) && cols > 0 && positions->ne[0] == src->ne[2] && positions->ne[1] == 1 &&
                          positions->ne[2] == 1 && positions->ne[3] == 1 && src->ne[2] > 0;
    const bool known = pr.mode == emel::kRopeNorm || pr.mode == emel::kRopeNeox || pr.mode == emel::kRopeTimestep;
    const bool layout_ok = pr.mode != emel::kRopeTimestep ||
                           ((uint64_t)pr.n_dims == cols && dense_contiguous_f32(src) &&
                            dense_contiguous_i32(positions) && dense_contiguous_f32(dst));
    if (shape_ok && !known) return EMEL_CUDA_INVALID_MODE;
    if (!shape_ok || !layout_ok) return EMEL_CUDA_SHAPE_MISMATCH;
    if (ctx == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    if ((reinterpret_cast<uintptr_t>(src->data) | reinterpret_cast<uintptr_t>(dst->data) |
         reinterpret_cast<uintptr_t>(positions->data)) & 3u)
        return EMEL_CUDA_INVALID_ARGUMENT;
    // the kernel counts a position's (row, pair) items in 32 bits
    if ((u128)src->ne[1] * (u128)(cols > 2 * 2048 ? 2048 : cols) * 256u >= ((u128)1 << 32)) return EMEL_CUDA_INVALID_ARGUMENT;
    emel::RopePlan p{};
    p.mode = pr.mode;
    p.src = static_cast<const char*>(src->data);
    p.dst = static_cast<char*>(dst->data);
    p.positions = static_cast<const char*>(positions->data);
    p.pos_stride = (int64_t)positions->nb[0];
    for (int d = 0; d < 4; ++d) {
        p.src_st[d] = (int64_t)cs.nb[d];
        p.dst_st[d] = (int64_t)cd.nb[d];
    }
    p.cols = cols;
    p.rows = src->ne[1];
    p.npos = src->ne[2];
    p.batches = src->ne[3];
    p.n_dims = (uint64_t)pr.n_dims;
    // the two per-operation scalars, with the same libm calls as the reference (rope.rs:536-540, 592)
    p.theta_scale = powf(pr.freq_base, -2.0f / (float)pr.n_dims);
    p.neg_log_period = -logf(pr.freq_base);
    p.freq_scale = pr.freq_scale;
    p.attn_factor = pr.attn_factor;
    // 16-byte vectors: unit dim-0 stride, 16-byte aligned row starts, and whole
    // vectors of pairs (norm: n_dims % 4, neox: (n_dims / 2) % 4; a table
    // chunk of 2048 pairs keeps both)
    bool vec = pr.mode != emel::kRopeTimestep && cs.nb[0] == 4 && cd.nb[0] == 4 &&
               (pr.mode == emel::kRopeNorm ? pr.n_dims % 4 == 0 : (pr.n_dims / 2) % 4 == 0) &&
               ((reinterpret_cast<uintptr_t>(src->data) | reinterpret_cast<uintptr_t>(dst->data)) & 15u) == 0;
    for (int d = 1; d < 4; ++d) vec = vec && cs.nb[d] % 16 == 0 && cd.nb[d] % 16 == 0;
    p.vec = vec;
    cudaError_t err = select_device(ctx);
    if (err == cudaSuccess) err = emel::launch_rope(env_of(ctx, stream), p);
    return device_status(ctx, err);
}

// ---- vocabulary matvec + argmax (matmul.rs OpMulMatArgmax, F32) -----------------

emel_cuda_status emel_cuda_mul_mat_argmax(emel_cuda_context* ctx, void* stream, const emel_tensor_view* lhs,
                                          const emel_tensor_view* rhs, const emel_tensor_view* dst,
                                          int32_t* index_out) {
    Checked cl, cr, cd;
    // argmax_views_valid (matmul.rs:1416-1423)
    if (lhs == nullptr || rhs == nullptr || dst == nullptr || !validate_as(lhs, EMEL_DTYPE_F32, false, &cl) ||
        !validate_as(rhs, EMEL_DTYPE_F32, false, &cr) || !validate_as(dst, EMEL_DTYPE_F32, false, &cd) ||
        !dense_contiguous_f32(lhs) || !dense_contiguous_f32(rhs) || !dense_contiguous_f32(dst))
        return EMEL_CUDA_INVALID_VIEW;
    // argmax_shape_valid (matmul.rs:1504-1520): lhs [k, m], rhs [1, k], dst [1]
    const uint64_t* l = lhs->ne;
    const uint64_t* r = rhs->ne;
    const uint64_t* d = dst->ne;
    if (!(l[0] > 0 && l[1] > 0 && l[2] == 1 && l[3] == 1 && r[0] == 1 && r[1] == l[0] && r[2] == 1 && r[3] == 1 &&
          d[0] == 1 && d[1] == 1 && d[2] == 1 && d[3] == 1))
        return EMEL_CUDA_SHAPE_MISMATCH;
    if (ctx == nullptr || index_out == nullptr || (reinterpret_cast<uintptr_t>(index_out) & 3u) ||
        ((reinterpret_cast<uintptr_t>(lhs->data) | reinterpret_cast<uintptr_t>(rhs->data) |
          reinterpret_cast<uintptr_t>(dst->data)) & 3u) ||
        l[1] > 0x7fffffffull)
        return EMEL_CUDA_INVALID_ARGUMENT;
    emel::MvArgmaxPlan p{};
    p.lhs = static_cast<const float*>(lhs->data);
    p.rhs = static_cast<const float*>(rhs->data);
    p.k = l[0];
    p.rows = l[1];
    p.vec = p.k % 4 == 0 && ((reinterpret_cast<uintptr_t>(lhs->data) | reinterpret_cast<uintptr_t>(rhs->data)) & 15u) == 0;
    p.dst_value = static_cast<float*>(dst->data);
    p.dst_index = index_out;
    char* ws = static_cast<char*>(ctx->workspace);
    p.ticket = reinterpret_cast<unsigned*>(ws);
    p.partials = ws + 256;
    p.fault = reinterpret_cast<uint32_t*>(ws + emel::kFaultWordOffset);
    cudaError_t err = select_device(ctx);
    if (err == cudaSuccess) err = emel::launch_mul_mat_argmax(env_of(ctx, stream), p);
    return device_status(ctx, err);
}

static emel_cuda_status mul_mat_argmax_packed(emel_cuda_context* ctx, void* stream, const emel_tensor_view* lhs,
                                              const emel_tensor_view* rhs, const emel_tensor_view* dst,
                                              int32_t* index_out, uint32_t code, uint64_t block_bytes) {
    Checked cr, cd;
    uint64_t row_bytes = 0;
    // quantized_views_valid (matmul.rs:1522-1542): packed rows of at most
    // 1024 blocks, dense F32 rhs and destination
    if (lhs == nullptr || rhs == nullptr || dst == nullptr ||
        !gr_packed_view_valid(lhs, code, 32, block_bytes, &row_bytes) || lhs->ne[0] / 32 > 1024 ||
        !validate_as(rhs, EMEL_DTYPE_F32, false, &cr) || !validate_as(dst, EMEL_DTYPE_F32, false, &cd) ||
        !dense_contiguous_f32(rhs) || !dense_contiguous_f32(dst))
        return EMEL_CUDA_INVALID_VIEW;
    // quantized_shape_valid (matmul.rs:1544-1564)
    const uint64_t* l = lhs->ne;
    const uint64_t* r = rhs->ne;
    const uint64_t* d = dst->ne;
    if (!(l[0] > 0 && l[1] > 0 && l[2] == 1 && l[3] == 1 && r[0] == 1 && r[1] == l[0] && r[2] == 1 && r[3] == 1 &&
          d[0] == 1 && d[1] == 1 && d[2] == 1 && d[3] == 1))
        return EMEL_CUDA_SHAPE_MISMATCH;
    if (ctx == nullptr || index_out == nullptr || (reinterpret_cast<uintptr_t>(index_out) & 3u) ||
        ((reinterpret_cast<uintptr_t>(lhs->data) | reinterpret_cast<uintptr_t>(rhs->data) |
          reinterpret_cast<uintptr_t>(dst->data)) & 3u) ||
        l[1] > 0x7fffffffull)
        return EMEL_CUDA_INVALID_ARGUMENT;
    emel::MvArgmaxPlan p{};
    p.rhs = static_cast<const float*>(rhs->data);
    p.k = l[0];
    p.rows = l[1];
    p.dst_value = static_cast<float*>(dst->data);
    p.dst_index = index_out;
    char* ws = static_cast<char*>(ctx->workspace);
    p.ticket = reinterpret_cast<unsigned*>(ws);
    p.partials = ws + 256;
    p.fault = reinterpret_cast<uint32_t*>(ws + emel::kFaultWordOffset);
    cudaError_t err = select_device(ctx);
    if (err == cudaSuccess)
        err = emel::launch_mul_mat_argmax_packed(env_of(ctx, stream), p, static_cast<const uint8_t*>(lhs->data),
                                                 (int)code);
    return device_status(ctx, err);
}

emel_cuda_status emel_cuda_mul_mat_argmax_q8_0(emel_cuda_context* ctx, void* stream, const emel_tensor_view* lhs,
                                               const emel_tensor_view* rhs, const emel_tensor_view* dst,
                                               int32_t* index_out) {
    return mul_mat_argmax_packed(ctx, stream, lhs, rhs, dst, index_out, EMEL_DTYPE_Q8_0, 34);
}

emel_cuda_status emel_cuda_mul_mat_argmax_q4_0(emel_cuda_context* ctx, void* stream, const emel_tensor_view* lhs,
                                               const emel_tensor_view* rhs, const emel_tensor_view* dst,
                                               int32_t* index_out) {
    return mul_mat_argmax_packed(ctx, stream, lhs, rhs, dst, index_out, EMEL_DTYPE_Q4_0, 18);
}

emel_cuda_status emel_cuda_mul_mat_argmax_q4_1(emel_cuda_context* ctx, void* stream, const emel_tensor_view* lhs,
                                               const emel_tensor_view* rhs, const emel_tensor_view* dst,
                                               int32_t* index_out) {
    return mul_mat_argmax_packed(ctx, stream, lhs, rhs, dst, index_out, EMEL_DTYPE_Q4_1, 20);
}

emel_cuda_status emel_cuda_mul_mat_argmax_q5_0(emel_cuda_context* ctx, void* stream, const emel_tensor_view* lhs,
                                               const emel_tensor_view* rhs, const emel_tensor_view* dst,
                                               int32_t* index_out) {
    return mul_mat_argmax_packed(ctx, stream, lhs, rhs, dst, index_out, EMEL_DTYPE_Q5_0, 22);
}

static emel_cuda_status mul_mat_argmax_k(emel_cuda_context* ctx, void* stream, const emel_tensor_view* lhs,
                                         const emel_tensor_view* rhs, const emel_tensor_view* dst, int32_t* index_out,
                                         uint32_t code, uint64_t block_bytes) {
    Checked cr, cd;
    uint64_t row_bytes = 0;
    // quantized_views_valid (matmul.rs:1522-1542): K-quant rows of at most
    // 128 blocks of 256 values, dense F32 rhs and destination
    if (lhs == nullptr || rhs == nullptr || dst == nullptr ||
        !gr_packed_view_valid(lhs, code, 256, block_bytes, &row_bytes) || lhs->ne[0] / 256 > 128 ||
        !validate_as(rhs, EMEL_DTYPE_F32, false, &cr) || !validate_as(dst, EMEL_DTYPE_F32, false, &cd) ||
        !dense_contiguous_f32(rhs) || !dense_contiguous_f32(dst))
        return EMEL_CUDA_INVALID_VIEW;
    const uint64_t* l = lhs->ne;
    const uint64_t* r = rhs->ne;
    const uint64_t* d = dst->ne;
    if (!(l[0] > 0 && l[1] > 0 && l[2] == 1 && l[3] == 1 && r[0] == 1 && r[1] == l[0] && r[2] == 1 && r[3] == 1 &&
          d[0] == 1 && d[1] == 1 && d[2] == 1 && d[3] == 1))
        return EMEL_CUDA_SHAPE_MISMATCH;
    if (ctx == nullptr || index_out == nullptr || (reinterpret_cast<uintptr_t>(index_out) & 3u) ||
        ((reinterpret_cast<uintptr_t>(lhs->data) | reinterpret_cast<uintptr_t>(rhs->data) |
          reinterpret_cast<uintptr_t>(dst->data)) & 3u) ||
        l[1] > 0x7fffffffull)
        return EMEL_CUDA_INVALID_ARGUMENT;
    emel::MvArgmaxPlan p{};
    p.rhs = static_cast<const float*>(rhs->data);
    p.k = l[0];
    p.rows = l[1];
    p.dst_value = static_cast<float*>(dst->data);
    p.dst_index = index_out;
    char* ws = static_cast<char*>(ctx->workspace);
    p.ticket = reinterpret_cast<unsigned*>(ws);
    p.partials = ws + 256;
    p.fault = reinterpret_cast<uint32_t*>(ws + emel::kFaultWordOffset);
    cudaError_t err = select_device(ctx);
    if (err == cudaSuccess)
        err = emel::launch_mul_mat_argmax_k(env_of(ctx, stream), p, static_cast<const uint8_t*>(lhs->data), (int)code);
    return device_status(ctx, err);
}

emel_cuda_status emel_cuda_mul_mat_argmax_q4_k(emel_cuda_context* ctx, void* stream, const emel_tensor_view* lhs,
                                               const emel_tensor_view* rhs, const emel_tensor_view* dst,
                                               int32_t* index_out) {
    return mul_mat_argmax_k(ctx, stream, lhs, rhs, dst, index_out, EMEL_DTYPE_Q4_K, 144);
}

emel_cuda_status emel_cuda_mul_mat_argmax_q6_k(emel_cuda_context* ctx, void* stream, const emel_tensor_view* lhs,
                                               const emel_tensor_view* rhs, const emel_tensor_view* dst,
                                               int32_t* index_out) {
    return mul_mat_argmax_k(ctx, stream, lhs, rhs, dst, index_out, EMEL_DTYPE_Q6_K, 210);
}

emel_cuda_status emel_cuda_mul_mat_argmax_q2_k(emel_cuda_context* ctx, void* stream, const emel_tensor_view* lhs,
                                               const emel_tensor_view* rhs, const emel_tensor_view* dst,
                                               int32_t* index_out) {
    return mul_mat_argmax_k(ctx, stream, lhs, rhs, dst, index_out, EMEL_DTYPE_Q2_K, 84);
}

emel_cuda_status emel_cuda_mul_mat_argmax_q3_k(emel_cuda_context* ctx, void* stream, const emel_tensor_view* lhs,
                                               const emel_tensor_view* rhs, const emel_tensor_view* dst,
                                               int32_t* index_out) {
    return mul_mat_argmax_k(ctx, stream, lhs, rhs, dst, index_out, EMEL_DTYPE_Q3_K, 110);
}

// ---- single-query attention -------------------------------------------------

// dense_f32_layout (flash_attn.rs:305-325): effective strides exactly row-major.
static bool fa_dense_f32(const emel_tensor_view* v) {
    uint64_t s[4];
    if (v->dtype != EMEL_DTYPE_F32 || !strides_of(*v, 4, s)) return false;
    uint64_t expected = 4;
    for (int d = 0; d < 4; ++d) {
        if (s[d] != expected) return false;
        if (__builtin_mul_overflow(expected, v->ne[d], &expected)) return false;
    }
    return true;
}

emel_cuda_status emel_cuda_flash_attn_ext(emel_cuda_context* ctx, void* stream, const emel_tensor_view* query,
                                          const emel_tensor_view* key, const emel_tensor_view* value,
                                          const emel_tensor_view* dst, const emel_flash_attn_options* options) {
    if (query == nullptr || key == nullptr || value == nullptr || dst == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    // OpFlashAttnExt::new (flash_attn.rs:78-99): resolve the optional parameters
    const uint64_t head_dim = query->ne[0], heads = query->ne[2], tokens = key->ne[1], kv_heads = key->ne[2];
    float scale = 1.0f / std::sqrt((float)head_dim);
    uint64_t masked_total = tokens;
    if (options != nullptr && options->has_scale) scale = options->scale;
    if (options != nullptr && options->has_masked_total_tokens) masked_total = options->masked_total_tokens;
    // valid_request (flash_attn.rs:262-303): every rule maps to InvalidRequest
    Checked cq, cd;
    uint64_t ks[4], vs[4];
    const bool valid =
        validate_as(query, EMEL_DTYPE_F32, false, &cq) && validate_as(dst, EMEL_DTYPE_F32, false, &cd) &&
        gr_half_view_valid(key, EMEL_DTYPE_F16, ks) && gr_half_view_valid(value, EMEL_DTYPE_F16, vs) &&
        fa_dense_f32(query) && fa_dense_f32(dst) && head_dim != 0 && query->ne[1] == 1 && heads != 0 && tokens != 0 &&
        kv_heads != 0 && key->ne[0] == head_dim && value->ne[0] == head_dim && value->ne[1] == tokens &&
        value->ne[2] == kv_heads && dst->ne[0] == head_dim && dst->ne[1] == 1 && dst->ne[2] == heads &&
        query->ne[3] == 1 && key->ne[3] == 1 && value->ne[3] == 1 && dst->ne[3] == 1 && heads % kv_heads == 0 &&
        head_dim <= 4096 && masked_total >= tokens && std::isfinite(scale) && scale > 0.0f;
    if (!valid) return EMEL_CUDA_INVALID_REQUEST;
    // device additions: element-aligned pointers, a grid of one CTA per head
    const uintptr_t a32 = reinterpret_cast<uintptr_t>(query->data) | reinterpret_cast<uintptr_t>(dst->data);
    const uintptr_t a16 = reinterpret_cast<uintptr_t>(key->data) | reinterpret_cast<uintptr_t>(value->data);
    if (ctx == nullptr || (a32 & 3u) != 0 || (a16 & 1u) != 0 || heads > 0x7fffffffull)
        return EMEL_CUDA_INVALID_ARGUMENT;
    emel::FlashAttnPlan p{};
    p.q = static_cast<const float*>(query->data);
    p.k = static_cast<const char*>(key->data);
    p.v = static_cast<const char*>(value->data);
    p.dst = static_cast<float*>(dst->data);
    for (int d = 0; d < 3; ++d) {
        // a singleton dimension's stride is never multiplied by a nonzero coordinate
        p.ks[d] = key->ne[d] > 1 ? ks[d] : 0;
        p.vs[d] = value->ne[d] > 1 ? vs[d] : 0;
    }
    p.d = head_dim;
    p.tokens = tokens;
    p.heads = heads;
    p.rep = heads / kv_heads;
    p.scale = scale;
    p.k_rows = head_dim % 8 == 0 && (head_dim == 1 || p.ks[0] == 2) && ((reinterpret_cast<uintptr_t>(key->data) |
                                                                        p.ks[1] | p.ks[2]) & 15u) == 0;
    p.v_bulk = head_dim % 8 == 0 && p.vs[0] == 2 &&
               ((reinterpret_cast<uintptr_t>(value->data) | p.vs[1] | p.vs[2]) & 15u) == 0;
    p.v_dense = p.v_bulk && (tokens == 1 || p.vs[1] == head_dim * 2);
    p.fault = reinterpret_cast<uint32_t*>(static_cast<char*>(ctx->workspace) + emel::kFaultWordOffset);
    cudaError_t err = select_device(ctx);
    if (err == cudaSuccess) err = emel::launch_flash_attn(env_of(ctx, stream), p);
    if (err == cudaSuccess) {
        // FlashAttnWorkspace bookkeeping (flash_attn.rs:337-341)
        if (ctx->fa_prepared_tokens == tokens) ++ctx->fa_reuse_count;
        ctx->fa_prepared_tokens = tokens;
    }
    return device_status(ctx, err);
}

emel_cuda_status emel_cuda_flash_attn_workspace(const emel_cuda_context* ctx, uint64_t* prepared_tokens,
                                                uint64_t* reuse_count) {
    if (ctx == nullptr || prepared_tokens == nullptr || reuse_count == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    *prepared_tokens = ctx->fa_prepared_tokens;
    *reuse_count = ctx->fa_reuse_count;
    return EMEL_CUDA_OK;
}

// ---- diagonal family ---------------------------------------------------------

// square_side (diag.rs:107-120): the side of a non-empty perfect square.
static bool diag_square_side(uint64_t len, uint64_t* side) {
    if (len == 0) return false;
    uint64_t s = (uint64_t)std::sqrt((double)len);
    while (s > 0 && (u128)s * s > len) --s;
    while ((u128)(s + 1) * (s + 1) <= len) ++s;
    if ((u128)s * s != len) return false;
    *side = s;
    return true;
}

static bool ranges_overlap(const void* a, uint64_t abytes, const void* b, uint64_t bbytes) {
    const uintptr_t x = reinterpret_cast<uintptr_t>(a), y = reinterpret_cast<uintptr_t>(b);
    return x < y + bbytes && y < x + abytes;
}

static emel_cuda_status diag_launch(emel_cuda_context* ctx, void* stream, const float* input, float* output,
                                    uint64_t side, uint64_t n_past, int mode) {
    emel::DiagPlan p{};
    p.in = input;
    p.out = output;
    p.side = side;
    p.n_past = n_past;
    p.vec = side % 4 == 0 && ((reinterpret_cast<uintptr_t>(input) | reinterpret_cast<uintptr_t>(output)) & 15u) == 0;
    cudaError_t err = select_device(ctx);
    if (err == cudaSuccess) err = emel::launch_diag(env_of(ctx, stream), p, mode);
    return device_status(ctx, err);
}

emel_cuda_status emel_cuda_diag(emel_cuda_context* ctx, void* stream, const float* input, uint64_t input_len,
                                float* output, uint64_t output_len) {
    // OpDiag::side (diag.rs:56-65) behind guard_diag_valid
    const uint64_t n = input_len;
    if (n == 0 || (u128)n * n != (u128)output_len) return EMEL_CUDA_INVALID_SHAPE;
    if (ctx == nullptr || input == nullptr || output == nullptr ||
        ((reinterpret_cast<uintptr_t>(input) | reinterpret_cast<uintptr_t>(output)) & 3u) != 0 ||
        output_len > UINT64_MAX / 8 || ranges_overlap(input, n * 4, output, output_len * 4))
        return EMEL_CUDA_INVALID_ARGUMENT;
    return diag_launch(ctx, stream, input, output, n, 0, emel::kDiag);
}

emel_cuda_status emel_cuda_diag_mask(emel_cuda_context* ctx, void* stream, int mode, const float* input,
                                     uint64_t input_len, float* output, uint64_t output_len, int32_t n_past) {
    if (mode != EMEL_DIAG_MASK_INF && mode != EMEL_DIAG_MASK_ZERO) return EMEL_CUDA_INVALID_ARGUMENT;
    // mask_valid (diag.rs:122-124)
    uint64_t side = 0;
    if (n_past < 0 || input_len != output_len || !diag_square_side(input_len, &side)) return EMEL_CUDA_INVALID_SHAPE;
    if (ctx == nullptr || input == nullptr || output == nullptr ||
        ((reinterpret_cast<uintptr_t>(input) | reinterpret_cast<uintptr_t>(output)) & 3u) != 0 ||
        input_len > UINT64_MAX / 8 || (input != output && ranges_overlap(input, input_len * 4, output, output_len * 4)))
        return EMEL_CUDA_INVALID_ARGUMENT;
    return diag_launch(ctx, stream, input, output, side, (uint64_t)n_past,
                       mode == EMEL_DIAG_MASK_INF ? emel::kDiagMaskInf : emel::kDiagMaskZero);
}

emel_cuda_status emel_cuda_soft_max_diag_mask_inf(emel_cuda_context* ctx, void* stream, const float* input,
                                                  uint64_t input_len, float* output, uint64_t output_len,
                                                  int32_t n_past) {
    // the mask's guards (mask_valid, diag.rs:122-124); the soft_max of its
    // dense [side, side] result has none left to fail
    uint64_t side = 0;
    if (n_past < 0 || input_len != output_len || !diag_square_side(input_len, &side)) return EMEL_CUDA_INVALID_SHAPE;
    if (ctx == nullptr || input == nullptr || output == nullptr ||
        ((reinterpret_cast<uintptr_t>(input) | reinterpret_cast<uintptr_t>(output)) & 3u) != 0 ||
        input_len > UINT64_MAX / 8 || (input != output && ranges_overlap(input, input_len * 4, output, output_len * 4)))
        return EMEL_CUDA_INVALID_ARGUMENT;
    return diag_launch(ctx, stream, input, output, side, (uint64_t)n_past, emel::kDiagSoftMaxCausal);
}

// ---- gated linear units ------------------------------------------------------

emel_cuda_status emel_cuda_glu(emel_cuda_context* ctx, void* stream, int subop, const float* input,
                               uint64_t input_len, float* output, uint64_t output_len) {
    if (ctx == nullptr || subop < emel::kReGlu || subop > emel::kGeGluQuick) return EMEL_CUDA_INVALID_ARGUMENT;
    // glu.rs:84-91 (split_len) behind guard_invalid (glu.rs:258-260)
    if (input_len == 0 || input_len % 2 != 0 || output_len != input_len / 2) return EMEL_CUDA_INVALID_SHAPE;
    if (input == nullptr || output == nullptr || (reinterpret_cast<uintptr_t>(input) & 3u) != 0 ||
        (reinterpret_cast<uintptr_t>(output) & 3u) != 0 || input_len > (UINT64_MAX / 8))
        return EMEL_CUDA_INVALID_ARGUMENT;
    const uint64_t n = output_len;
    // values = input[0, n), gates = input[n, 2n), output[0, n): three 1-D F32 views
    emel_tensor_view vv{}, gv{}, ov{};
    const void* ptrs[3] = {input, input + n, output};
    emel_tensor_view* vs[3] = {&vv, &gv, &ov};
    for (int k = 0; k < 3; ++k) {
        vs[k]->data = const_cast<void*>(ptrs[k]);
        vs[k]->storage_bytes = n * 4;
        vs[k]->ne[0] = n;
        vs[k]->ne[1] = vs[k]->ne[2] = vs[k]->ne[3] = 1;
        vs[k]->nb[0] = 4;
        vs[k]->nb[1] = vs[k]->nb[2] = vs[k]->nb[3] = n * 4;
        vs[k]->dtype = EMEL_DTYPE_F32;
    }
    Checked cv, cg, co;
    if (!validate_as(&vv, EMEL_DTYPE_F32, false, &cv) || !validate_as(&gv, EMEL_DTYPE_F32, false, &cg) ||
        !validate_as(&ov, EMEL_DTYPE_F32, false, &co))
        return EMEL_CUDA_INVALID_ARGUMENT;
    const emel_tensor_view* views[3] = {&ov, &vv, &gv};
    const Checked* cks[3] = {&co, &cv, &cg};
    const emel::EwPlan plan = plan_equal_count(DType::F32, views, cks, 3);
    cudaError_t err = select_device(ctx);
    if (err == cudaSuccess) err = emel::launch_binary(env_of(ctx, stream), plan, emel::kGluBase + subop);
    return device_status(ctx, err);
}

// ---- row normalisation --------------------------------------------------------

static emel_cuda_status norm_common(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                    const emel_tensor_view* weight, const emel_tensor_view* dst, float eps, int op) {
    Checked cs, cd, cw;
    // normalization.rs:364-382: view -> shape -> parameters
    if (!normalization_valid(src, &cs) || !normalization_valid(dst, &cd)) return EMEL_CUDA_INVALID_VIEW;
    if (op == 2 && !validate_as(weight, EMEL_DTYPE_F32, true, &cw)) return EMEL_CUDA_INVALID_VIEW;
    if (!same_ne(src, dst)) return EMEL_CUDA_SHAPE_MISMATCH;
    if (op == 2 && !(weight->ne[0] == src->ne[0] && weight->ne[1] == 1 && weight->ne[2] == 1 && weight->ne[3] == 1))
        return EMEL_CUDA_SHAPE_MISMATCH;
    if (!(std::isfinite(eps) && eps >= 0.0f)) return EMEL_CUDA_INVALID_PARAMETERS;
    if (ctx == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    emel::RowPlan p = plan_rows(src, cs, dst, &cd);
    if (op == 2) {
        p.aux = row_operand(weight, cw);
        p.has_aux = true;
        p.aux_dtype = (int)DType::F32;
    }
    cudaError_t err = select_device(ctx);
    if (err == cudaSuccess) err = emel::launch_norm(env_of(ctx, stream), p, op, eps);
    return device_status(ctx, err);
}

emel_cuda_status emel_cuda_norm(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                const emel_tensor_view* dst, float eps) {
    return norm_common(ctx, stream, src, nullptr, dst, eps, 0);
}

emel_cuda_status emel_cuda_rms_norm(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                    const emel_tensor_view* dst, float eps) {
    return norm_common(ctx, stream, src, nullptr, dst, eps, 1);
}

emel_cuda_status emel_cuda_rms_norm_mul(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                        const emel_tensor_view* weight, const emel_tensor_view* dst, float eps) {
    return norm_common(ctx, stream, src, weight, dst, eps, 2);
}

// ---- softmax -------------------------------------------------------------------

static emel_cuda_status soft_max_common(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                        const emel_tensor_view* mask, const emel_tensor_view* dst, float scale,
                                        bool apply_scale) {
    Checked cs, cd, cm;
    if (!validate_as(src, EMEL_DTYPE_F32, false, &cs) || !validate_as(dst, EMEL_DTYPE_F32, false, &cd))
        return EMEL_CUDA_INVALID_VIEW;
    if (mask && !validate_float(mask, false, &cm)) return EMEL_CUDA_INVALID_VIEW;
    // reductions.rs:473-483
    const uint64_t width = src->ne[0];
    if (!(width > 0 && cs.count % width == 0 && cs.count == cd.count)) return EMEL_CUDA_SHAPE_MISMATCH;
    if (mask && !(mask->ne[0] == width && mask->ne[1] >= src->ne[1] && src->ne[2] % mask->ne[2] == 0 &&
                  src->ne[3] % mask->ne[3] == 0))
        return EMEL_CUDA_SHAPE_MISMATCH;
    if (ctx == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    emel::RowPlan p = plan_rows(src, cs, dst, &cd);
    // reductions.rs:485-495: dense (f64 sum) when both layouts are dense
    p.dense = dense(*src, cs) && dense(*dst, cd);
    if (!same_ne(src, dst)) {
        if (dense(*dst, cd)) {
            // same ordinal -> address map as a dense view with src's extents
            p.dst.st[0] = 1;
            p.dst.st[1] = (int64_t)src->ne[0];
            p.dst.st[2] = (int64_t)(src->ne[0] * src->ne[1]);
            p.dst.st[3] = (int64_t)(src->ne[0] * src->ne[1] * src->ne[2]);
            p.vec = p.ne[0] % 4 == 0 && row_vec_ok(p.src) && row_vec_ok(p.dst);
        } else {
            p.dst_ordinal = true;
        }
    }
    if (mask) {
        p.aux = row_operand(mask, cm);
        p.has_aux = true;
        p.aux_dtype = (int)dt_of(mask->dtype);
    }
    cudaError_t err = select_device(ctx);
    if (err == cudaSuccess) err = emel::launch_soft_max(env_of(ctx, stream), p, apply_scale, scale);
    return device_status(ctx, err);
}

emel_cuda_status emel_cuda_soft_max(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                    const emel_tensor_view* dst) {
    return soft_max_common(ctx, stream, src, nullptr, dst, 1.0f, false);
}

emel_cuda_status emel_cuda_soft_max_ext(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                        const emel_tensor_view* mask, const emel_tensor_view* dst, float scale) {
    return soft_max_common(ctx, stream, src, mask, dst, scale, true);
}

// ---- reductions ------------------------------------------------------------------

static bool scalar_shape(const emel_tensor_view* v) {
    return v->ne[0] == 1 && v->ne[1] == 1 && v->ne[2] == 1 && v->ne[3] == 1;
}

static bool rows_shape(const emel_tensor_view* src, const emel_tensor_view* dst) {
    return dst->ne[0] == 1 && dst->ne[1] == src->ne[1] && dst->ne[2] == src->ne[2] && dst->ne[3] == src->ne[3];
}

static bool index_view(const emel_tensor_view* v, Checked* c) {
    return validate_as(v, EMEL_DTYPE_F32, false, c) || validate_as(v, EMEL_DTYPE_I64, false, c) ||
           validate_as(v, EMEL_DTYPE_I32, false, c);
}

static emel_cuda_status sum_common(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                   const emel_tensor_view* dst, int mode) {
    Checked cs, cd;
    // reductions.rs:452-458, 520-530
    if (!validate_as(src, EMEL_DTYPE_F32, false, &cs) || !validate_as(dst, EMEL_DTYPE_F32, false, &cd))
        return EMEL_CUDA_INVALID_VIEW;
    if (!scalar_shape(dst)) return EMEL_CUDA_SHAPE_MISMATCH;
    if (ctx == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    const emel::RowPlan p = plan_rows(src, cs, nullptr, nullptr);
    cudaError_t err = select_device(ctx);
    if (err == cudaSuccess) err = emel::launch_sum(env_of(ctx, stream), p, mode, dst->data);
    return device_status(ctx, err);
}

emel_cuda_status emel_cuda_sum(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                               const emel_tensor_view* dst) {
    return sum_common(ctx, stream, src, dst, 0);
}

emel_cuda_status emel_cuda_mean(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                const emel_tensor_view* dst) {
    return sum_common(ctx, stream, src, dst, 1);
}

emel_cuda_status emel_cuda_sum_f64(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src, double* out) {
    Checked cs;
    if (!validate_as(src, EMEL_DTYPE_F32, false, &cs)) return EMEL_CUDA_INVALID_VIEW;
    if (ctx == nullptr || out == nullptr || reinterpret_cast<uintptr_t>(out) % 8 != 0) return EMEL_CUDA_INVALID_ARGUMENT;
    const emel::RowPlan p = plan_rows(src, cs, nullptr, nullptr);
    cudaError_t err = select_device(ctx);
    if (err == cudaSuccess) err = emel::launch_sum(env_of(ctx, stream), p, 2, out);
    return device_status(ctx, err);
}

emel_cuda_status emel_cuda_sum_rows(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                    const emel_tensor_view* dst) {
    Checked cs, cd;
    // reductions.rs:460-463, 532-542
    if (!validate_as(src, EMEL_DTYPE_F32, false, &cs) || !validate_as(dst, EMEL_DTYPE_F32, false, &cd))
        return EMEL_CUDA_INVALID_VIEW;
    if (!rows_shape(src, dst)) return EMEL_CUDA_SHAPE_MISMATCH;
    if (ctx == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    emel::RowPlan p = plan_rows(src, cs, dst, &cd);
    p.vec = p.ne[0] % 4 == 0 && row_vec_ok(p.src);  // dst is written one value per row
    cudaError_t err = select_device(ctx);
    if (err == cudaSuccess) err = emel::launch_sum_rows(env_of(ctx, stream), p);
    return device_status(ctx, err);
}

emel_cuda_status emel_cuda_argmax(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                  const emel_tensor_view* dst) {
    Checked cs, cd;
    if (!validate_as(src, EMEL_DTYPE_F32, false, &cs) || !index_view(dst, &cd)) return EMEL_CUDA_INVALID_VIEW;
    if (!scalar_shape(dst)) return EMEL_CUDA_SHAPE_MISMATCH;
    if (ctx == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    const emel::RowPlan p = plan_rows(src, cs, nullptr, nullptr);
    cudaError_t err = select_device(ctx);
    if (err == cudaSuccess) err = emel::launch_argmax(env_of(ctx, stream), p, 0, (int)dst->dtype, 0, dst->data);
    return device_status(ctx, err);
}

emel_cuda_status emel_cuda_argmax_partial_compute(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                                  int64_t index_base, emel_cuda_argmax_partial* out) {
    Checked cs;
    if (!validate_as(src, EMEL_DTYPE_F32, false, &cs)) return EMEL_CUDA_INVALID_VIEW;
    if (ctx == nullptr || out == nullptr || reinterpret_cast<uintptr_t>(out) % 8 != 0) return EMEL_CUDA_INVALID_ARGUMENT;
    const emel::RowPlan p = plan_rows(src, cs, nullptr, nullptr);
    cudaError_t err = select_device(ctx);
    if (err == cudaSuccess) err = emel::launch_argmax(env_of(ctx, stream), p, 1, 0, index_base, out);
    return device_status(ctx, err);
}

emel_cuda_status emel_cuda_argmax_combine(const emel_cuda_argmax_partial* partials, int count, int64_t* index_out,
                                          float* value_out) {
    if (partials == nullptr || count <= 0 || index_out == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    // shards are in ordinal order; a later shard wins only with a strictly
    // greater value (reductions.rs:721), so ties keep the earliest index
    bool has = false;
    float best = 0.0f;
    int64_t idx = 0;
    for (int k = 0; k < count; ++k) {
        const emel_cuda_argmax_partial& q = partials[k];
        if (!q.has_value) continue;
        if (!has || q.value > best || (q.value == best && q.index < idx)) {
            has = true;
            best = q.value;
            idx = q.index;
        }
    }
    if (partials[0].first_is_nan || !has) {
        idx = 0;
    }
    *index_out = idx;
    if (value_out) *value_out = best;
    return EMEL_CUDA_OK;
}

emel_cuda_status emel_cuda_argmax_rows(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                       const emel_tensor_view* dst) {
    Checked cs, cd;
    if (!validate_as(src, EMEL_DTYPE_F32, false, &cs) || !index_view(dst, &cd)) return EMEL_CUDA_INVALID_VIEW;
    if (!rows_shape(src, dst)) return EMEL_CUDA_SHAPE_MISMATCH;
    if (ctx == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    emel::RowPlan p = plan_rows(src, cs, dst, &cd);
    p.vec = p.ne[0] % 4 == 0 && row_vec_ok(p.src);  // dst is written one index per row
    cudaError_t err = select_device(ctx);
    if (err == cudaSuccess) err = emel::launch_argmax_rows(env_of(ctx, stream), p, (int)dst->dtype);
    return device_status(ctx, err);
}

}  // extern "C"

namespace emel {

// The OpSum request checks of emel_cuda_sum (reductions.rs:452-458,
// 520-530), for entry points that run without a context.
emel_cuda_status check_scalar_sum(const emel_tensor_view* src, const emel_tensor_view* dst, RowPlan* plan) {
    Checked cs, cd;
    if (!validate_as(src, EMEL_DTYPE_F32, false, &cs) || !validate_as(dst, EMEL_DTYPE_F32, false, &cd))
        return EMEL_CUDA_INVALID_VIEW;
    if (!scalar_shape(dst)) return EMEL_CUDA_SHAPE_MISMATCH;
    *plan = plan_rows(src, cs, nullptr, nullptr);
    return EMEL_CUDA_OK;
}

}  // namespace emel

// ===========================================================================
// Generic operation envelope (emel_cuda_generic)
// ===========================================================================
namespace {

using u128g = unsigned __int128;

// validate_span (generic.rs:822-862): every extent nonzero, the element count
// representable, no zero stride on an extent > 1, and the highest byte inside
// the storage.  F32 views resolve the implicit nb[0] == 0 form.
bool generic_span_valid(const emel_tensor_view* v, uint64_t nb[4], uint64_t* count) {
    if (v->dtype == EMEL_DTYPE_F32) {
        if (!strides_of(*v, 4, nb)) return false;
    } else {
        for (int d = 0; d < 4; ++d) nb[d] = v->nb[d];
    }
    uint64_t c = 1;
    for (int d = 0; d < 4; ++d) {
        if (v->ne[d] == 0 || __builtin_mul_overflow(c, v->ne[d], &c)) return false;
        if (v->ne[d] > 1 && nb[d] == 0) return false;
    }
    u128g max_offset = 0;
    for (int d = 0; d < 4; ++d) {
        const u128g term = (u128g)(v->ne[d] - 1) * (u128g)nb[d];
        if (__builtin_add_overflow(max_offset, term, &max_offset)) return false;
    }
    u128g end;
    if (__builtin_add_overflow(max_offset, (u128g)1, &end)) return false;
    if (end > (u128g)v->storage_bytes) return false;
    *count = c;
    return true;
}

// RawTensorView::f32_valid (generic.rs:467-473): an F32 view whose span is
// valid and whose every byte stride is at least 4.
bool generic_f32_valid(const emel_tensor_view* v, Checked* out) {
    if (v == nullptr || v->dtype != EMEL_DTYPE_F32) return false;
    Checked c;
    c.elem = 4;
    if (!generic_span_valid(v, c.nb, &c.count)) return false;
    for (int d = 0; d < 4; ++d)
        if (c.nb[d] < 4) return false;
    *out = c;
    return true;
}

// The device reads binary32 with aligned loads.
bool generic_device_aligned(const emel_tensor_view* v, const Checked& c) {
    if (reinterpret_cast<uintptr_t>(v->data) % 4 != 0) return false;
    for (int d = 0; d < 4; ++d)
        if (c.nb[d] % 4 != 0) return false;
    return true;
}

// parameter_f32 (generic.rs:907-911): slot k is bytes [4k, 4k + 4) of the
// initialised prefix.
bool generic_param(const emel_cuda_generic_request* r, int slot, float* out) {
    const uint32_t end = (uint32_t)slot * 4u + 4u;
    if (end > r->params_len) return false;
    std::memcpy(out, r->params + slot * 4, 4);
    return true;
}

enum class GenericKind { Copy, Binary, Scalar, Clamp, SiluBack, Repeat, Unary, Sum, Mean, Argmax, SoftMax, Norm };

}  // namespace

extern "C" emel_cuda_status emel_cuda_generic(emel_cuda_context* ctx, void* stream,
                                              const emel_cuda_generic_request* r) {
    if (r == nullptr || r->op >= 95 || r->params_len > 64) return EMEL_CUDA_INVALID_ARGUMENT;
    // GenericRequest::validate (generic.rs:747-766): every present view
    const emel_tensor_view* all[4] = {r->src0, r->src1, r->src2, r->dst};
    for (const emel_tensor_view* v : all) {
        uint64_t nb[4], count;
        if (v != nullptr && !generic_span_valid(v, nb, &count)) return EMEL_CUDA_INVALID_SHAPE;
    }
    // maintained routes of the device table (sm.rs:324-419)
    GenericKind kind;
    int code = 0;
    switch (r->op) {
    case 0: kind = GenericKind::Copy; break;
    case 1: kind = GenericKind::Binary; code = EMEL_BINARY_ADD; break;
    case 5: kind = GenericKind::Binary; code = EMEL_BINARY_SUB; break;
    case 6: kind = GenericKind::Binary; code = EMEL_BINARY_MUL; break;
    case 7: kind = GenericKind::Binary; code = EMEL_BINARY_DIV; break;
    case 3: kind = GenericKind::Scalar; code = emel::kAdd1; break;
    case 32: kind = GenericKind::Scalar; code = emel::kScale; break;
    case 70: kind = GenericKind::Scalar; code = emel::kLeakyRelu; break;
    case 50: kind = GenericKind::Clamp; code = emel::kClamp; break;
    case 22: kind = GenericKind::SiluBack; break;
    case 19: kind = GenericKind::Repeat; break;
    case 8: kind = GenericKind::Unary; code = EMEL_UNARY_SQR; break;
    case 9: kind = GenericKind::Unary; code = EMEL_UNARY_SQRT; break;
    case 10: kind = GenericKind::Unary; code = EMEL_UNARY_LOG; break;
    case 11: kind = GenericKind::Unary; code = EMEL_UNARY_SIN; break;
    case 12: kind = GenericKind::Unary; code = EMEL_UNARY_COS; break;
    case 13: kind = GenericKind::Sum; break;
    case 16: kind = GenericKind::Mean; break;
    case 17: kind = GenericKind::Argmax; break;
    case 46: kind = GenericKind::SoftMax; break;
    case 23: kind = GenericKind::Norm; code = 3; break;
    case 24: kind = GenericKind::Norm; code = 4; break;
    case 85:
        // generic.rs:1307-1350 (execute_generic_unary); any other subop is a
        // known-invalid request (actor.rs guard_generic_known_invalid)
        kind = GenericKind::Unary;
        switch (r->unary_subop) {
        case 0: code = EMEL_UNARY_ABS; break;
        case 2: code = EMEL_UNARY_NEG; break;
        case 4: code = EMEL_UNARY_TANH; break;
        case 5: code = EMEL_UNARY_ELU; break;
        case 6: code = EMEL_UNARY_RELU; break;
        case 8: code = emel::kGeluGeneric; break;
        case 10: code = EMEL_UNARY_SILU; break;
        case 13: code = EMEL_UNARY_EXP; break;
        default: return EMEL_CUDA_INVALID_SHAPE;
        }
        break;
    default:
        return EMEL_CUDA_UNSUPPORTED_OPERATION;
    }
    // operand rules of the route (generic.rs:938-990, 1136-1190)
    Checked c0, c1, cd;
    const bool v0 = generic_f32_valid(r->src0, &c0);
    const bool v1 = generic_f32_valid(r->src1, &c1);
    const bool vd = generic_f32_valid(r->dst, &cd);
    float pa = 0.0f, pb = 0.0f;
    bool ok = false;
    switch (kind) {
    case GenericKind::Copy:
    case GenericKind::Unary:
    case GenericKind::SoftMax: ok = v0 && vd && c0.count == cd.count; break;
    case GenericKind::Binary: ok = v0 && v1 && vd && c0.count == c1.count && c0.count == cd.count; break;
    case GenericKind::Scalar:
        ok = v0 && vd && c0.count == cd.count && generic_param(r, 0, &pa) && std::isfinite(pa);
        break;
    case GenericKind::Clamp:
        ok = v0 && vd && c0.count == cd.count && generic_param(r, 0, &pa) && generic_param(r, 1, &pb) &&
             std::isfinite(pa) && std::isfinite(pb) && pa <= pb;
        break;
    case GenericKind::SiluBack: ok = v0 && v1 && vd && same_ne(r->src0, r->src1) && same_ne(r->src0, r->dst); break;
    case GenericKind::Repeat:
        ok = v0 && vd;
        for (int d = 0; ok && d < 4; ++d) ok = r->dst->ne[d] % r->src0->ne[d] == 0;
        break;
    case GenericKind::Sum:
    case GenericKind::Mean:
    case GenericKind::Argmax: ok = v0 && vd && cd.count == 1; break;
    case GenericKind::Norm:
        ok = v0 && vd && same_ne(r->src0, r->dst) && generic_param(r, 0, &pa) && std::isfinite(pa) && pa >= 0.0f;
        break;
    }
    if (!ok) return EMEL_CUDA_INVALID_SHAPE;
    const bool uses1 = kind == GenericKind::Binary || kind == GenericKind::SiluBack;
    if (!generic_device_aligned(r->src0, c0) || !generic_device_aligned(r->dst, cd) ||
        (uses1 && !generic_device_aligned(r->src1, c1))) {
        if (ctx != nullptr)
            std::snprintf(ctx->last_error, sizeof(ctx->last_error), "device views need 4-byte aligned data and strides");
        return EMEL_CUDA_INVALID_ARGUMENT;
    }
    if (ctx == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    cudaError_t err = select_device(ctx);
    if (err != cudaSuccess) return device_status(ctx, err);
    const emel::LaunchEnv env = env_of(ctx, stream);
    switch (kind) {
    case GenericKind::Copy:
    case GenericKind::Unary:
    case GenericKind::Scalar:
    case GenericKind::Clamp: {
        const emel_tensor_view* views[3] = {r->dst, r->src0, nullptr};
        const Checked* cks[3] = {&cd, &c0, nullptr};
        const int op = kind == GenericKind::Copy ? (int)emel::kCopy : code;
        err = emel::launch_unary(env, plan_equal_count(DType::F32, views, cks, 2), op, pa, pb);
        break;
    }
    case GenericKind::Binary:
    case GenericKind::SiluBack: {
        const emel_tensor_view* views[3] = {r->dst, r->src0, r->src1};
        const Checked* cks[3] = {&cd, &c0, &c1};
        err = emel::launch_binary(env, plan_equal_count(DType::F32, views, cks, 3),
                                  kind == GenericKind::Binary ? code : (int)emel::kSiluBack);
        break;
    }
    case GenericKind::Repeat: {
        emel::EwPlan p{};
        p.dtype = DType::F32;
        p.count = cd.count;
        for (int d = 0; d < 4; ++d) p.ne[d] = r->dst->ne[d];
        p.dst = operand(r->dst, cd);
        p.src0 = operand(r->src0, c0);
        err = emel::launch_repeat(env, p);
        break;
    }
    case GenericKind::Sum:
    case GenericKind::Mean:
        err = emel::launch_sum(env, plan_rows(r->src0, c0, nullptr, nullptr), kind == GenericKind::Sum ? 0 : 1,
                               r->dst->data);
        break;
    case GenericKind::Argmax:
        err = emel::launch_argmax(env, plan_rows(r->src0, c0, nullptr, nullptr), 0, (int)DType::F32, 0, r->dst->data);
        break;
    case GenericKind::SoftMax: {
        emel::RowPlan p = plan_rows(r->src0, c0, r->dst, &cd);
        if (!same_ne(r->src0, r->dst)) p.dst_ordinal = true;
        err = emel::launch_soft_max_generic(env, p);
        break;
    }
    case GenericKind::Norm:
        err = emel::launch_norm_generic(env, plan_rows(r->src0, c0, r->dst, &cd), code, pa);
        break;
    }
    return device_status(ctx, err);
}
