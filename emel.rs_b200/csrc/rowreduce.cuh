// Block-level reductions shared by the row kernels (rows.cu, rowring.cu):
// sums in f64, NaN-skipping maxima and (value, index) argmax, over groups
// of G threads (G <= 32: shuffles only; larger G: shuffles, then one
// shared-memory slot per warp folded in warp order, so the result does not
// depend on timing).
#pragma once

#include "common.cuh"

namespace emel {

namespace {

template <int G>
struct GroupScratch {
    double d[G > 32 ? G / 32 : 1];
    float f[G > 32 ? G / 32 : 1];
    int64_t i[G > 32 ? G / 32 : 1];
    uint32_t h[G > 32 ? G / 32 : 1];
};

template <int G>
__device__ __forceinline__ double group_sum(double v, GroupScratch<G>* s) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if constexpr (G > 32) {
        const int lane = threadIdx.x & 31, warp = (threadIdx.x % G) / 32;
        __syncthreads();
        if (lane == 0) s->d[warp] = v;
        __syncthreads();
        v = 0.0;
#pragma unroll
        for (int w = 0; w < G / 32; ++w) v += s->d[w];
    }
    return v;
}

// max that ignores NaN (the reference never selects a NaN unless it is the
// first element, which callers handle separately)
__device__ __forceinline__ float max_nn(float a, float b) { return is_nan(a) ? b : (is_nan(b) ? a : (b > a ? b : a)); }

template <int G>
__device__ __forceinline__ float group_max(float v, GroupScratch<G>* s) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = max_nn(v, __shfl_xor_sync(0xffffffffu, v, o));
    if constexpr (G > 32) {
        const int lane = threadIdx.x & 31, warp = (threadIdx.x % G) / 32;
        __syncthreads();
        if (lane == 0) s->f[warp] = v;
        __syncthreads();
        v = s->f[0];
#pragma unroll
        for (int w = 1; w < G / 32; ++w) v = max_nn(v, s->f[w]);
    }
    return v;
}

// (has, value, index): prefer has, then larger value, then smaller index.
struct ArgBest {
    float v;
    int64_t i;
    uint32_t has;
};

__device__ __forceinline__ ArgBest arg_better(ArgBest a, ArgBest b) {
    if (!b.has) return a;
    if (!a.has) return b;
    if (b.v > a.v) return b;
    if (a.v > b.v) return a;
    return b.i < a.i ? b : a;
}

template <int G>
__device__ __forceinline__ ArgBest group_argmax(ArgBest v, GroupScratch<G>* s) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        ArgBest w;
        w.v = __shfl_xor_sync(0xffffffffu, v.v, o);
        w.i = __shfl_xor_sync(0xffffffffu, v.i, o);
        w.has = __shfl_xor_sync(0xffffffffu, v.has, o);
        v = arg_better(v, w);
    }
    if constexpr (G > 32) {
        const int lane = threadIdx.x & 31, warp = (threadIdx.x % G) / 32;
        __syncthreads();
        if (lane == 0) {
            s->f[warp] = v.v;
            s->i[warp] = v.i;
            s->h[warp] = v.has;
        }
        __syncthreads();
        v = ArgBest{s->f[0], s->i[0], s->h[0]};
#pragma unroll
        for (int w = 1; w < G / 32; ++w) v = arg_better(v, ArgBest{s->f[w], s->i[w], s->h[w]});
    }
    return v;
}

}  // namespace

}  // namespace emel
