// Whole-tensor reductions: sum / mean (reductions.rs:671-681, 703-713) and
// argmax (reductions.rs:715-730).
//
// One launch per reduction.  Every CTA streams a fixed, grid-strided share
// of the tensor (16-byte loads when the tensor is one dense run), reduces it
// in f64 (sum) or as (value, index) (argmax), and stores its partial in the
// context workspace.  The CTA that finishes last (atomic ticket, no waiting)
// folds the partials in a fixed order and writes the result, then re-arms
// the ticket.  With the grid fixed per device, the result is deterministic.
#include "common.cuh"
#include "launch.hpp"
#include "pdl.cuh"

namespace emel {

namespace {

constexpr int kThreads = 256;
// Four resident CTAs per SM (guaranteed by the launch bounds' register cap)
// with eight 16-byte loads in flight per thread: 128 KB of reads in flight
// per SM from one full wave.  A grid larger than what is resident would run
// a partial second wave; fewer threads with more loads each also shorten
// the ramp and tail that dominate a shard of one dim-3 slice (134 MB).
constexpr int kCtasPerSm = 4;
constexpr int kVecsInFlight = 8;

struct ArgPart {
    float v;
    uint32_t has;
    int64_t i;
};

__device__ __forceinline__ ArgPart better(ArgPart a, ArgPart b) {
    if (!b.has) return a;
    if (!a.has) return b;
    if (b.v > a.v) return b;
    if (a.v > b.v) return a;
    return b.i < a.i ? b : a;
}

__device__ __forceinline__ void arg_take(ArgPart& b, float v, int64_t i) {
    if ((!b.has && !is_nan(v)) || v > b.v) {
        b.v = v;
        b.i = i;
        b.has = 1;
    }
}

__device__ __forceinline__ double block_sum(double v, double* sh) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int lane = threadIdx.x & 31, warp = threadIdx.x / 32;
    __syncthreads();
    if (lane == 0) sh[warp] = v;
    __syncthreads();
    double t = 0.0;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) t += sh[w];
    return t;
}

__device__ __forceinline__ ArgPart block_arg(ArgPart v, ArgPart* sh) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        ArgPart w;
        w.v = __shfl_xor_sync(0xffffffffu, v.v, o);
        w.has = __shfl_xor_sync(0xffffffffu, v.has, o);
        w.i = __shfl_xor_sync(0xffffffffu, v.i, o);
        v = better(v, w);
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x / 32;
    __syncthreads();
    if (lane == 0) sh[warp] = v;
    __syncthreads();
    ArgPart t = sh[0];
#pragma unroll
    for (int w = 1; w < kThreads / 32; ++w) t = better(t, sh[w]);
    return t;
}

// Logical ordinal of (row r, column c) is r * ne0 + c; its address follows
// the view's strides.
__device__ __forceinline__ const float* row_ptr(const RowPlan& p, uint64_t r) {
    const uint64_t i1 = r % p.ne[1], q = r / p.ne[1], i2 = q % p.ne[2], i3 = q / p.ne[2];
    return reinterpret_cast<const float*>(p.src.ptr) + (int64_t)i1 * p.src.st[1] + (int64_t)i2 * p.src.st[2] +
           (int64_t)i3 * p.src.st[3];
}

// Flat = the view is one dense run of p.rows * ne0 floats.
// Source walks.  MODE 1: the view is one dense, 16-byte aligned run.
// MODE 2: rows of ne0 % 4 == 0 floats with unit dim-0 stride and 16-byte
// aligned starts (e.g. a permuted view whose rows stay contiguous); vector
// v of the logical order is found with 32-bit magic-number divisions.
// MODE 0: anything else, one element at a time (warps walk rows).
struct VecWalk {
    const float* base;
    FastDiv dv, d1, d2;
    uint32_t vpr, ne1, ne2;
    int64_t s1, s2, s3;
    uint64_t nvec;
};

template <int MODE>
__device__ __forceinline__ VecWalk vec_walk(const RowPlan& p) {
    VecWalk w{};
    w.base = reinterpret_cast<const float*>(p.src.ptr);
    w.nvec = p.rows * p.ne[0] / 4;
    if constexpr (MODE == 2) {
        w.vpr = (uint32_t)(p.ne[0] / 4);
        w.ne1 = (uint32_t)p.ne[1];
        w.ne2 = (uint32_t)p.ne[2];
        w.dv = make_fastdiv(w.vpr);
        w.d1 = make_fastdiv(w.ne1);
        w.d2 = make_fastdiv(w.ne2);
        w.s1 = p.src.st[1];
        w.s2 = p.src.st[2];
        w.s3 = p.src.st[3];
    }
    return w;
}

// Vector v of the logical order (elements 4v .. 4v+3).
template <int MODE>
__device__ __forceinline__ float4 vec_load(const VecWalk& w, uint64_t v) {
    if constexpr (MODE == 1) {
        return __ldcs(reinterpret_cast<const float4*>(w.base) + v);
    } else {
        const uint32_t row = fdiv((uint32_t)v, w.dv);
        const uint32_t c4 = (uint32_t)v - row * w.vpr;
        const uint32_t q = fdiv(row, w.d1), i1 = row - q * w.ne1;
        const uint32_t i3 = fdiv(q, w.d2), i2 = q - i3 * w.ne2;
        const float* r = w.base + (int64_t)i1 * w.s1 + (int64_t)i2 * w.s2 + (int64_t)i3 * w.s3;
        return __ldcs(reinterpret_cast<const float4*>(r) + c4);
    }
}

// partial_sum / partial_arg wait for the previous kernel (pdl_enter) on
// every path; with `early` (the input is clear of that kernel's writes) a
// thread's first batch of loads goes out before the wait.
template <int MODE>
__device__ __forceinline__ double partial_sum(const RowPlan& p, bool early) {
    double acc = 0.0, acc2 = 0.0;  // two chains: x, y and z, w of every vector
    const uint64_t gthreads = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t gid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if constexpr (MODE != 0) {
        constexpr int U = kVecsInFlight;
        const VecWalk w = vec_walk<MODE>(p);
        const uint32_t G = (uint32_t)gthreads;
        uint32_t i = (uint32_t)gid;
        if (early && (uint64_t)i + (U - 1) * (uint64_t)G < w.nvec) {
            float4 q[U];
#pragma unroll
            for (int k = 0; k < U; ++k) q[k] = vec_load<MODE>(w, i + k * G);
            pdl_enter();
#pragma unroll
            for (int k = 0; k < U; ++k) {
                acc += (double)q[k].x;
                acc2 += (double)q[k].z;
                acc += (double)q[k].y;
                acc2 += (double)q[k].w;
            }
            i += U * G;
        } else {
            pdl_enter();
        }
        for (; (uint64_t)i + (U - 1) * (uint64_t)G < w.nvec; i += U * G) {
            float4 q[U];
#pragma unroll
            for (int k = 0; k < U; ++k) q[k] = vec_load<MODE>(w, i + k * G);
#pragma unroll
            for (int k = 0; k < U; ++k) {
                acc += (double)q[k].x;
                acc2 += (double)q[k].z;
                acc += (double)q[k].y;
                acc2 += (double)q[k].w;
            }
        }
        for (; (uint64_t)i < w.nvec; i += G) {
            const float4 a = vec_load<MODE>(w, i);
            acc += (double)a.x;
            acc2 += (double)a.z;
            acc += (double)a.y;
            acc2 += (double)a.w;
        }
        if constexpr (MODE == 1) {
            const uint64_t n = p.rows * p.ne[0];
            const uint64_t t = w.nvec * 4 + gid;
            if (t < n) acc += (double)w.base[t];
        }
    } else {
        // warps walk rows; lanes walk columns
        const uint64_t warp = gid / 32, nwarps = gthreads / 32;
        const uint32_t lane = threadIdx.x & 31;
        pdl_enter();
        for (uint64_t r = warp; r < p.rows; r += nwarps) {
            const float* row = row_ptr(p, r);
            for (uint64_t c = lane; c < p.ne[0]; c += 32) acc += (double)row[(int64_t)c * p.src.st[0]];
        }
    }
    return acc + acc2;
}

// One argmax chain of the vector walk: the running maximum of one lane of
// the vectors (component c of vector v is element 4v + c) and the vector
// index where it was taken.  best starts as NaN; fmaxf ignores a NaN
// operand, so nb = fmaxf(best, v) differs from best exactly when v is
// strictly greater (the strict > of reductions.rs:721) or v is the chain's
// first non-NaN value; a tie keeps the earlier index (vectors arrive in
// increasing order within a chain).  A chain whose best is still NaN saw
// no comparable value.  Three instructions per element.
__device__ __forceinline__ void chain_take(float& best, uint32_t& idx, float v, uint32_t vec) {
    const float nb = fmaxf(best, v);
    if (nb != best) idx = vec;  // unordered compare: true while best is NaN
    best = nb;
}

template <int MODE>
__device__ __forceinline__ ArgPart partial_arg(const RowPlan& p, bool early) {
    ArgPart b{0.0f, 0, 0};
    const uint64_t gthreads = (uint64_t)gridDim.x * blockDim.x;
    const uint64_t gid = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if constexpr (MODE != 0) {
        // vector v holds logical elements 4v .. 4v+3 in both walks; four
        // independent chains, one per vector lane, folded at the end with
        // the first-index rule
        constexpr int U = kVecsInFlight;
        const VecWalk w = vec_walk<MODE>(p);
        const uint32_t G = (uint32_t)gthreads;
        const float nan = __int_as_float(0x7fc00000);
        float bv[4] = {nan, nan, nan, nan};
        uint32_t bi[4] = {0, 0, 0, 0};
        uint32_t i = (uint32_t)gid;
        if (early && (uint64_t)i + (U - 1) * (uint64_t)G < w.nvec) {
            float4 q[U];
#pragma unroll
            for (int k = 0; k < U; ++k) q[k] = vec_load<MODE>(w, i + k * G);
            pdl_enter();
#pragma unroll
            for (int k = 0; k < U; ++k) {
                const uint32_t v = i + k * G;
                chain_take(bv[0], bi[0], q[k].x, v);
                chain_take(bv[1], bi[1], q[k].y, v);
                chain_take(bv[2], bi[2], q[k].z, v);
                chain_take(bv[3], bi[3], q[k].w, v);
            }
            i += U * G;
        } else {
            pdl_enter();
        }
        for (; (uint64_t)i + (U - 1) * (uint64_t)G < w.nvec; i += U * G) {
            float4 q[U];
#pragma unroll
            for (int k = 0; k < U; ++k) q[k] = vec_load<MODE>(w, i + k * G);
#pragma unroll
            for (int k = 0; k < U; ++k) {
                const uint32_t v = i + k * G;
                chain_take(bv[0], bi[0], q[k].x, v);
                chain_take(bv[1], bi[1], q[k].y, v);
                chain_take(bv[2], bi[2], q[k].z, v);
                chain_take(bv[3], bi[3], q[k].w, v);
            }
        }
        for (; (uint64_t)i < w.nvec; i += G) {
            const float4 a = vec_load<MODE>(w, i);
            chain_take(bv[0], bi[0], a.x, i);
            chain_take(bv[1], bi[1], a.y, i);
            chain_take(bv[2], bi[2], a.z, i);
            chain_take(bv[3], bi[3], a.w, i);
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            ArgPart q{bv[c], is_nan(bv[c]) ? 0u : 1u, 4 * (int64_t)bi[c] + c};
            b = better(b, q);
        }
        if constexpr (MODE == 1) {
            const uint64_t n = p.rows * p.ne[0];
            const uint64_t t = w.nvec * 4 + gid;
            if (t < n) arg_take(b, w.base[t], (int64_t)t);
        }
    } else {
        const uint64_t warp = gid / 32, nwarps = gthreads / 32;
        const uint32_t lane = threadIdx.x & 31;
        pdl_enter();
        for (uint64_t r = warp; r < p.rows; r += nwarps) {
            const float* row = row_ptr(p, r);
            for (uint64_t c = lane; c < p.ne[0]; c += 32)
                arg_take(b, row[(int64_t)c * p.src.st[0]], (int64_t)(r * p.ne[0] + c));
        }
    }
    return b;
}

// Returns true in exactly one CTA: the last to finish.  The workspace ticket
// is re-armed by that CTA.
__device__ __forceinline__ bool last_cta(unsigned* ticket) {
    __shared__ bool is_last;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) is_last = atomicAdd(ticket, 1u) == gridDim.x - 1;
    __syncthreads();
    return is_last;
}

template <int MODE>
__global__ void __launch_bounds__(kThreads, kCtasPerSm) sum_all(RowPlan p, double* partials, unsigned* ticket, int mode, void* out,
                                                    int early) {
    __shared__ double sh[kThreads / 32];
    double acc = block_sum(partial_sum<MODE>(p, early != 0), sh);
    if (threadIdx.x == 0) partials[blockIdx.x] = acc;
    if (!last_cta(ticket)) return;
    // fixed-order fold: thread t adds partials t, t+256, ... then a fixed tree
    double t = 0.0;
    for (unsigned k = threadIdx.x; k < gridDim.x; k += kThreads) t += __ldcg(partials + k);
    t = block_sum(t, sh);
    if (threadIdx.x == 0) {
        const uint64_t n = p.rows * p.ne[0];
        if (mode == 0) *reinterpret_cast<float*>(out) = __double2float_rn(t);
        else if (mode == 1) *reinterpret_cast<float*>(out) = __double2float_rn(t / (double)n);
        else *reinterpret_cast<double*>(out) = t;
        *ticket = 0u;
    }
}

template <int MODE>
__global__ void __launch_bounds__(kThreads, kCtasPerSm) argmax_all(RowPlan p, ArgPart* partials, unsigned* ticket, int out_kind,
                                                       int dst_dtype, int64_t index_base, void* out, int early) {
    __shared__ ArgPart sh[kThreads / 32];
    ArgPart b = block_arg(partial_arg<MODE>(p, early != 0), sh);
    if (threadIdx.x == 0) partials[blockIdx.x] = b;
    if (!last_cta(ticket)) return;
    ArgPart t{0.0f, 0, 0};
    for (unsigned k = threadIdx.x; k < gridDim.x; k += kThreads) {
        ArgPart q;
        q.v = __ldcg(&partials[k].v);
        q.has = __ldcg(&partials[k].has);
        q.i = __ldcg(&partials[k].i);
        t = better(t, q);
    }
    t = block_arg(t, sh);
    if (threadIdx.x == 0) {
        const float first = reinterpret_cast<const float*>(p.src.ptr)[0];
        if (out_kind == 0) {
            // reductions.rs:716-727: the scan starts from element 0, so a NaN
            // there (or no comparable value at all) leaves index 0.
            const int64_t idx = (is_nan(first) || !t.has) ? 0 : t.i;
            if (dst_dtype == (int)DType::I64) *reinterpret_cast<int64_t*>(out) = idx;
            else if (dst_dtype == (int)DType::I32) *reinterpret_cast<int32_t*>(out) = (int32_t)idx;
            else *reinterpret_cast<float*>(out) = (float)idx;
        } else {
            struct Partial {
                float value;
                uint32_t has_value;
                int64_t index;
                uint32_t first_is_nan;
                uint32_t reserved;
            };
            Partial* o = reinterpret_cast<Partial*>(out);
            o->value = t.v;
            o->has_value = t.has;
            o->index = t.i + index_base;
            o->first_is_nan = is_nan(first) ? 1u : 0u;
            o->reserved = 0u;
        }
        *ticket = 0u;
    }
}

}  // namespace

uint64_t split_rows_workspace_offset(int sm_count) {
    // after the header (tickets, fault words) and one 16-byte partial per CTA
    return (256 + (uint64_t)sm_count * kCtasPerSm * 16 + 255) / 256 * 256;
}

uint64_t reduction_workspace_bytes(int sm_count) {
    // + the few-long-rows kernels' per-row chunk partials and row tickets
    return split_rows_workspace_offset(sm_count) + (uint64_t)sm_count * (kSplitRowChunks * 16 + 4) + 256;
}

static uint32_t reduce_grid(const LaunchEnv& env, uint64_t n) {
    constexpr uint64_t per_cta = (uint64_t)kThreads * kVecsInFlight * 4;  // one full batch per thread
    const uint64_t want = (n + per_cta - 1) / per_cta;
    const uint64_t cap = (uint64_t)env.sm_count * kCtasPerSm;
    const uint64_t g = want < cap ? want : cap;
    return (uint32_t)(g == 0 ? 1 : g);
}

// 1: one dense run; 2: contiguous 16-byte aligned rows whose vector count
// fits 32-bit addressing; 0: element by element.
static int walk_mode(const RowPlan& p) {
    const uint64_t nvec = p.rows * p.ne[0] / 4;
    if (nvec >= (1ull << 32)) return 0;  // the vector walks index vectors in 32 bits
    if (p.flat) return 1;
    if (p.vec && p.ne[1] < (1ull << 32) && p.ne[2] < (1ull << 32)) return 2;
    return 0;
}

cudaError_t launch_sum(const LaunchEnv& env, const RowPlan& p, int mode, void* out) {
    unsigned* ticket = reinterpret_cast<unsigned*>(env.workspace);
    double* partials = reinterpret_cast<double*>(reinterpret_cast<char*>(env.workspace) + 256);
    const uint32_t grid = reduce_grid(env, p.rows * p.ne[0]);
    const int early = reads_clear(env, span_of(p.src, 4));
    cudaError_t err;
    switch (walk_mode(p)) {
    case 1: err = launch_dependent(sum_all<1>, dim3(grid), dim3(kThreads), 0, env.stream, p, partials, ticket, mode, out, early); break;
    case 2: err = launch_dependent(sum_all<2>, dim3(grid), dim3(kThreads), 0, env.stream, p, partials, ticket, mode, out, early); break;
    default: err = launch_dependent(sum_all<0>, dim3(grid), dim3(kThreads), 0, env.stream, p, partials, ticket, mode, out, early); break;
    }
    if (err == cudaSuccess) stream_wrote(env.stream, out, mode == 2 ? 8 : 4);  // the workspace is the library's own
    ++*env.launches;
    return err != cudaSuccess ? err : cudaGetLastError();
}

cudaError_t launch_argmax(const LaunchEnv& env, const RowPlan& p, int out_kind, int dst_dtype, int64_t index_base,
                          void* out) {
    unsigned* ticket = reinterpret_cast<unsigned*>(env.workspace);
    ArgPart* partials = reinterpret_cast<ArgPart*>(reinterpret_cast<char*>(env.workspace) + 256);
    const uint32_t grid = reduce_grid(env, p.rows * p.ne[0]);
    const int early = reads_clear(env, span_of(p.src, 4));
    cudaError_t err;
    switch (walk_mode(p)) {
    case 1: err = launch_dependent(argmax_all<1>, dim3(grid), dim3(kThreads), 0, env.stream, p, partials, ticket, out_kind, dst_dtype, index_base, out, early); break;
    case 2: err = launch_dependent(argmax_all<2>, dim3(grid), dim3(kThreads), 0, env.stream, p, partials, ticket, out_kind, dst_dtype, index_base, out, early); break;
    default: err = launch_dependent(argmax_all<0>, dim3(grid), dim3(kThreads), 0, env.stream, p, partials, ticket, out_kind, dst_dtype, index_base, out, early); break;
    }
    if (err == cudaSuccess) stream_wrote(env.stream, out, out_kind == 0 ? 8 : 24);  // the workspace is the library's own
    ++*env.launches;
    return err != cudaSuccess ? err : cudaGetLastError();
}

}  // namespace emel

// ---------------------------------------------------------------------------
// Whole-tensor sum without allocation (emel_cuda_sum_noalloc).
//
// Its scratch is a file-scope device array instead of a context workspace:
// a 256-byte header holding the last-CTA ticket, then room for
// kNoAllocMaxPartials per-CTA partial sums.  Host code cannot use the
// array's name as a device address, so the first call on each device asks
// the runtime for it (cudaGetSymbolAddress, with that device current) and
// keeps it.  The kernel is the one emel_cuda_sum launches, with the same grid
// for the same device and input, so both entry points return the same bits.
// ---------------------------------------------------------------------------
#include <mutex>

#include "emel_cuda.h"

namespace emel {

emel_cuda_status check_scalar_sum(const emel_tensor_view* src, const emel_tensor_view* dst, RowPlan* plan);

namespace {

constexpr int kNoAllocMaxPartials = 2048;  // one per CTA: 4 CTAs per SM up to 512 SMs
constexpr int kNoAllocMaxDevices = 64;
constexpr size_t kNoAllocHeader = 256;     // ticket, padded to the partials' alignment

__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocHeader + kNoAllocMaxPartials * sizeof(double)];

std::mutex g_noalloc_mutex;
void* g_noalloc_addr[kNoAllocMaxDevices];
int g_noalloc_sms[kNoAllocMaxDevices];

}  // namespace
}  // namespace emel

extern "C" emel_cuda_status emel_cuda_sum_noalloc(void* stream, const emel_tensor_view* src,
                                                   const emel_tensor_view* dst) {
    using namespace emel;
    RowPlan p;
    const emel_cuda_status checked = check_scalar_sum(src, dst, &p);
    if (checked != EMEL_CUDA_OK) return checked;
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return EMEL_CUDA_DEVICE_ERROR;
    if (dev >= kNoAllocMaxDevices) return EMEL_CUDA_INVALID_ARGUMENT;
    void* scratch = nullptr;
    int sms = 0;
    {
        std::lock_guard<std::mutex> lock(g_noalloc_mutex);
        if (g_noalloc_addr[dev] == nullptr) {
            void* addr = nullptr;
            if (cudaGetSymbolAddress(&addr, g_noalloc_scratch) != cudaSuccess || addr == nullptr)
                return EMEL_CUDA_DEVICE_ERROR;
            int n = 0;
            if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
                return EMEL_CUDA_DEVICE_ERROR;
            g_noalloc_sms[dev] = n;
            g_noalloc_addr[dev] = addr;
        }
        scratch = g_noalloc_addr[dev];
        sms = g_noalloc_sms[dev];
    }
    LaunchEnv env{};
    env.stream = static_cast<cudaStream_t>(stream);
    env.sm_count = sms;
    env.device = dev;
    const uint32_t grid = reduce_grid(env, p.rows * p.ne[0]);
    if (grid > (uint32_t)kNoAllocMaxPartials) return EMEL_CUDA_OUT_OF_MEMORY;  // the scratch is too small
    unsigned* ticket = static_cast<unsigned*>(scratch);
    double* partials = reinterpret_cast<double*>(static_cast<char*>(scratch) + kNoAllocHeader);
    // the array keeps the previous call's contents: the ticket must start at 0
    if (cudaMemsetAsync(ticket, 0, sizeof(unsigned), env.stream) != cudaSuccess) return EMEL_CUDA_DEVICE_ERROR;
    {  // the stream's write record: this launch's output is not reported
        uintptr_t lo, hi;
        bool known;
        stream_take(env.stream, &lo, &hi, &known);
    }
    switch (walk_mode(p)) {
    case 1: sum_all<1><<<grid, kThreads, 0, env.stream>>>(p, partials, ticket, 0, dst->data, 0); break;
    case 2: sum_all<2><<<grid, kThreads, 0, env.stream>>>(p, partials, ticket, 0, dst->data, 0); break;
    default: sum_all<0><<<grid, kThreads, 0, env.stream>>>(p, partials, ticket, 0, dst->data, 0); break;
    }
    return cudaGetLastError() == cudaSuccess ? EMEL_CUDA_OK : EMEL_CUDA_DEVICE_ERROR;
}
