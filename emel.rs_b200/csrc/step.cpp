// The graph seam: emel-graph's processor runs a step through a kernel
// callback, RunKernelFn = fn(&ExecuteRequest, &mut i32) -> bool
// (crates/emel-graph/src/processor/kernel_step/sm.rs:125-126; the request
// is processor/sm.rs:170-199).  A device step is the step plan that request
// points at: a fixed list of op-coded generic requests (the envelope the
// kernels actor dispatches, generic.rs:580-766) with their views copied in,
// run in order on one stream -- or, when asked, captured into one CUDA graph
// on the first run and replayed afterwards -- then synchronised, so the
// callback returns the way the reference's synchronous kernel step does.
//
// Everything here goes through the public entry points (emel_cuda_generic,
// emel_cuda_graph_*, emel_cuda_stream_synchronize), so a step validates and
// fails exactly as the individual requests do.
#include <cstring>
#include <new>
#include <vector>

#include "emel_cuda.h"

struct emel_cuda_step {
    emel_cuda_context* ctx;
    void* stream;
    uint32_t flags;
    std::vector<emel_tensor_view> views;               // four slots per request
    std::vector<emel_cuda_generic_request> requests;   // view pointers into `views`
    emel_cuda_graph* graph;
    uint64_t runs;
};

namespace {

constexpr uint32_t kKnownStepFlags = EMEL_CUDA_STEP_CAPTURE | EMEL_CUDA_STEP_ASYNC;

emel_cuda_status run_requests(emel_cuda_step* s) {
    for (const emel_cuda_generic_request& r : s->requests) {
        const emel_cuda_status st = emel_cuda_generic(s->ctx, s->stream, &r);
        if (st != EMEL_CUDA_OK) return st;
    }
    return EMEL_CUDA_OK;
}

emel_cuda_status run_step(emel_cuda_step* s) {
    if (!(s->flags & EMEL_CUDA_STEP_CAPTURE)) return run_requests(s);
    if (s->graph == nullptr) {
        emel_cuda_status st = emel_cuda_graph_begin(s->ctx, s->stream);
        if (st != EMEL_CUDA_OK) return st;
        const emel_cuda_status ran = run_requests(s);
        emel_cuda_graph* g = nullptr;
        st = emel_cuda_graph_end(s->ctx, s->stream, &g);  // always ends the capture
        if (ran != EMEL_CUDA_OK) {
            if (g != nullptr) emel_cuda_graph_destroy(s->ctx, g);
            return ran;
        }
        if (st != EMEL_CUDA_OK) return st;
        s->graph = g;
    }
    return emel_cuda_graph_launch(s->ctx, s->graph, s->stream);
}

}  // namespace

extern "C" {

emel_cuda_status emel_cuda_step_create(emel_cuda_context* ctx, void* stream, const emel_cuda_generic_request* requests,
                                       uint32_t count, uint32_t flags, emel_cuda_step** out) {
    if (out != nullptr) *out = nullptr;
    if (ctx == nullptr || out == nullptr || requests == nullptr || count == 0 || count > EMEL_CUDA_STEP_MAX_REQUESTS ||
        (flags & ~kKnownStepFlags) != 0)
        return EMEL_CUDA_INVALID_ARGUMENT;
    if ((flags & EMEL_CUDA_STEP_CAPTURE) && stream == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;  // no capture on the legacy stream
    for (uint32_t i = 0; i < count; ++i)
        if (requests[i].params_len > sizeof(requests[i].params)) return EMEL_CUDA_INVALID_ARGUMENT;
    auto* s = new (std::nothrow) emel_cuda_step();
    if (s == nullptr) return EMEL_CUDA_OUT_OF_MEMORY;
    try {
        s->views.resize((size_t)count * 4);
        s->requests.assign(requests, requests + count);
    } catch (...) {
        delete s;
        return EMEL_CUDA_OUT_OF_MEMORY;
    }
    for (uint32_t i = 0; i < count; ++i) {
        emel_cuda_generic_request& r = s->requests[i];
        const emel_tensor_view** slots[4] = {&r.src0, &r.src1, &r.src2, &r.dst};
        for (int k = 0; k < 4; ++k) {
            if (*slots[k] == nullptr) continue;
            s->views[(size_t)i * 4 + k] = **slots[k];
            *slots[k] = &s->views[(size_t)i * 4 + k];
        }
    }
    s->ctx = ctx;
    s->stream = stream;
    s->flags = flags;
    s->graph = nullptr;
    s->runs = 0;
    *out = s;
    return EMEL_CUDA_OK;
}

emel_cuda_status emel_cuda_step_destroy(emel_cuda_context* ctx, emel_cuda_step* step) {
    if (ctx == nullptr || step == nullptr || step->ctx != ctx) return EMEL_CUDA_INVALID_ARGUMENT;
    emel_cuda_status st = EMEL_CUDA_OK;
    if (step->graph != nullptr) st = emel_cuda_graph_destroy(ctx, step->graph);
    delete step;
    return st;
}

uint64_t emel_cuda_step_runs(const emel_cuda_step* step) { return step ? step->runs : 0; }

int emel_cuda_run_kernel(const emel_cuda_execute_request* request, int32_t* error_out) {
    if (request == nullptr || error_out == nullptr) {
        if (error_out != nullptr) *error_out = EMEL_CUDA_INVALID_ARGUMENT;
        return 0;
    }
    auto* s = reinterpret_cast<emel_cuda_step*>((uintptr_t)request->step_plan);
    auto* ctx = reinterpret_cast<emel_cuda_context*>((uintptr_t)request->compute_ctx);
    if (s == nullptr || ctx == nullptr || s->ctx != ctx) {
        *error_out = EMEL_CUDA_INVALID_ARGUMENT;
        return 0;
    }
    emel_cuda_status st = run_step(s);
    if (!(s->flags & EMEL_CUDA_STEP_ASYNC)) {
        // synchronous like the reference callback; a device-side failure of
        // this step (a bounded wait that expired, a rejected index) shows here
        const emel_cuda_status sync = emel_cuda_stream_synchronize(ctx, s->stream);
        if (st == EMEL_CUDA_OK) st = sync;
    }
    if (st == EMEL_CUDA_OK) ++s->runs;
    *error_out = st;
    return st == EMEL_CUDA_OK ? 1 : 0;
}

emel_cuda_status emel_cuda_layout_view(const uint64_t* dimensions, uint32_t rank, uint32_t element_type, void* data,
                                       uint64_t storage_bytes, emel_tensor_view* out) {
    if (out == nullptr || (rank > 0 && dimensions == nullptr) || rank > 4) return EMEL_CUDA_INVALID_ARGUMENT;
    uint32_t dtype = 0;
    uint64_t size = 0;
    switch (element_type) {
    case EMEL_ELEMENT_F32: dtype = EMEL_DTYPE_F32; size = 4; break;
    case EMEL_ELEMENT_F16: dtype = EMEL_DTYPE_F16; size = 2; break;
    case EMEL_ELEMENT_BF16: dtype = EMEL_DTYPE_BF16; size = 2; break;
    default: return EMEL_CUDA_INVALID_ARGUMENT;  // Quantized: the model format names the block type
    }
    std::memset(out, 0, sizeof(*out));
    // row-major dimensions, outermost first -> ne[0] is the innermost
    for (int d = 0; d < 4; ++d) out->ne[d] = 1;
    for (uint32_t d = 0; d < rank; ++d) out->ne[d] = dimensions[rank - 1 - d];
    uint64_t stride = size;
    for (int d = 0; d < 4; ++d) {
        out->nb[d] = stride;
        if (out->ne[d] != 0 && stride > UINT64_MAX / out->ne[d]) return EMEL_CUDA_INVALID_ARGUMENT;
        stride *= out->ne[d];
    }
    if (stride > storage_bytes) return EMEL_CUDA_INVALID_ARGUMENT;
    out->data = data;
    out->storage_bytes = storage_bytes;
    out->dtype = dtype;
    return EMEL_CUDA_OK;
}

}  // extern "C"
