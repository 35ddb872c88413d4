// Diagonal family (diag.rs OpDiag / OpDiagMaskInf / OpDiagMaskZero) on the
// device: flat F32 slices holding a side x side row-major matrix.
//
// The masks' fused form with soft_max (softmax_causal_rows) is at the end.
//
// Each is one streaming pass: diag writes side^2 floats (the diagonal from
// the input vector, +0 elsewhere); the masks copy the lower part of every
// row (col <= row + n_past) and write the masked value above it without
// reading the input there.  One CTA walks whole rows with 16-byte vectors
// when rows are 16-byte aligned (side % 4 == 0 and aligned pointers); a
// vector that straddles the mask boundary is loaded and merged per lane.
// Element bits are copied unchanged (NaN payloads included).
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"
#include "launch.hpp"
#include "pdl.cuh"
#include "rowreduce.cuh"

namespace emel {
namespace {

constexpr int kDiagThreads = 256;

template <int MODE>
__device__ __forceinline__ float diag_masked_value() {
    return MODE == kDiagMaskInf ? __int_as_float(0xff800000) : 0.0f;
}

template <int MODE, bool VEC>
__global__ void __launch_bounds__(kDiagThreads) diag_rows(DiagPlan p) {
    pdl_enter();
    const uint64_t side = p.side;
    for (uint64_t row = blockIdx.x; row < side; row += gridDim.x) {
        float* orow = p.out + row * side;
        if constexpr (MODE == kDiag) {
            const float dv = p.in[row];
            if constexpr (VEC) {
                float4* o4 = reinterpret_cast<float4*>(orow);
                for (uint64_t c4 = threadIdx.x; c4 < side / 4; c4 += kDiagThreads) {
                    float4 v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    const uint64_t c = c4 * 4;
                    if (row >= c && row < c + 4) {
                        if (row == c) v.x = dv;
                        if (row == c + 1) v.y = dv;
                        if (row == c + 2) v.z = dv;
                        if (row == c + 3) v.w = dv;
                    }
                    __stcs(o4 + c4, v);
                }
            } else {
                for (uint64_t c = threadIdx.x; c < side; c += kDiagThreads) orow[c] = c == row ? dv : 0.0f;
            }
        } else {
            const float* irow = p.in + row * side;
            const uint64_t keep = row + p.n_past;  // columns <= keep are copied
            const float mv = diag_masked_value<MODE>();
            if constexpr (VEC) {
                float4* o4 = reinterpret_cast<float4*>(orow);
                const float4* i4 = reinterpret_cast<const float4*>(irow);
                for (uint64_t c4 = threadIdx.x; c4 < side / 4; c4 += kDiagThreads) {
                    const uint64_t c = c4 * 4;
                    float4 v = make_float4(mv, mv, mv, mv);
                    if (c + 3 <= keep) {
                        v = __ldcs(i4 + c4);
                    } else if (c <= keep) {
                        const float4 x = __ldcs(i4 + c4);
                        v.x = x.x;  // c <= keep
                        if (c + 1 <= keep) v.y = x.y;
                        if (c + 2 <= keep) v.z = x.z;
                    }
                    __stcs(o4 + c4, v);
                }
            } else {
                for (uint64_t c = threadIdx.x; c < side; c += kDiagThreads) orow[c] = c > keep ? mv : irow[c];
            }
        }
    }
}

// diag_mask_inf followed by soft_max (diag.rs:144-161, then reductions.rs
// OpSoftMax on the dense [side, side] result, 565-638) in one pass per row.
// Row r keeps columns 0 .. r + n_past; the rest are -inf.  While the kept
// values hold no NaN and their maximum is finite, every masked column's
// exp(-inf - max) is +0 and its output 0 / sum = +0, so only the kept
// prefix is read: max, e = exp(v - max) stored in dst, binary64 sum, e / sum.
// Otherwise the row is redone with the reference's selection and NaN rules
// over all columns (the scan's maximum starts from column 0).
// The fast path's two block reductions, without group_max / group_sum's
// leading barrier: the maximum uses the scratch's f array and the sum its d
// array, and between one row's read of an array and the next row's write to
// it every thread passes the other reduction's barrier, so one barrier per
// reduction and none at the end of a row.  (The exact path's group_max /
// group_sum keep their leading barriers.)
__device__ __forceinline__ float diag_max_fast(float v, GroupScratch<kDiagThreads>* s) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if ((threadIdx.x & 31) == 0) s->f[threadIdx.x / 32] = v;
    __syncthreads();
    v = s->f[0];
#pragma unroll
    for (int w = 1; w < kDiagThreads / 32; ++w) v = fmaxf(v, s->f[w]);
    return v;
}

__device__ __forceinline__ double diag_sum_fast(double v, GroupScratch<kDiagThreads>* s) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((threadIdx.x & 31) == 0) s->d[threadIdx.x / 32] = v;
    __syncthreads();
    v = 0.0;
#pragma unroll
    for (int w = 0; w < kDiagThreads / 32; ++w) v += s->d[w];
    return v;
}

template <bool VEC>
__global__ void __launch_bounds__(kDiagThreads) softmax_causal_rows(DiagPlan p) {
    __shared__ GroupScratch<kDiagThreads> red;
    pdl_enter();
    const uint64_t side = p.side;
    for (uint64_t row = blockIdx.x; row < side; row += gridDim.x) {
        const float* x = p.in + row * side;
        float* y = p.out + row * side;
        const uint64_t kept = row + p.n_past + 1 < side ? row + p.n_past + 1 : side;
        float m = -INFINITY;
        bool odd = false;
        if constexpr (VEC) {
            // 16-byte vectors; lanes at or past `kept` take no part
            const uint64_t nk = (kept + 3) / 4;
            for (uint64_t v = threadIdx.x; v < nk; v += kDiagThreads) {
                const float4 q = reinterpret_cast<const float4*>(x)[v];  // read again below: keep it cached
                const float e4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int l = 0; l < 4; ++l)
                    if (4 * v + l < kept) {
                        odd = odd || is_nan(e4[l]);
                        m = fmaxf(m, e4[l]);
                    }
            }
        } else {
            for (uint64_t c = threadIdx.x; c < kept; c += kDiagThreads) {
                const float v = x[c];
                odd = odd || is_nan(v);
                m = fmaxf(m, v);
            }
        }
        m = diag_max_fast(odd ? INFINITY : m, &red);  // the kept values hold no NaN here, or odd is set
        if (isfinite(m)) {
            double acc = 0.0;
            if constexpr (VEC) {
                const uint64_t nk = (kept + 3) / 4;
                for (uint64_t v = threadIdx.x; v < nk; v += kDiagThreads) {
                    const float4 q = reinterpret_cast<const float4*>(x)[v];
                    float e4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                    for (int l = 0; l < 4; ++l) {
                        e4[l] = 4 * v + l < kept ? softmax_exp(__fsub_rn(e4[l], m)) : 0.0f;
                        acc += (double)e4[l];
                    }
                    reinterpret_cast<float4*>(y)[v] = make_float4(e4[0], e4[1], e4[2], e4[3]);
                }
            } else {
                for (uint64_t c = threadIdx.x; c < kept; c += kDiagThreads) {
                    const float e = softmax_exp(__fsub_rn(x[c], m));
                    y[c] = e;
                    acc += (double)e;
                }
            }
            acc = diag_sum_fast(acc, &red);
            const float denom = __double2float_rn(acc);  // >= 1: the maximum contributes exp(0)
            const float inv = __frcp_rn(denom);
            if constexpr (VEC) {
                for (uint64_t v = threadIdx.x; v < side / 4; v += kDiagThreads) {
                    float4 o = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                    if (4 * v < kept) {
                        const float4 e = reinterpret_cast<const float4*>(y)[v];
                        o = make_float4(softmax_div(e.x, denom, inv), 4 * v + 1 < kept ? softmax_div(e.y, denom, inv) : 0.0f,
                                        4 * v + 2 < kept ? softmax_div(e.z, denom, inv) : 0.0f,
                                        4 * v + 3 < kept ? softmax_div(e.w, denom, inv) : 0.0f);
                    }
                    __stcs(reinterpret_cast<float4*>(y) + v, o);
                }
            } else {
                for (uint64_t c = threadIdx.x; c < side; c += kDiagThreads)
                    y[c] = c < kept ? softmax_div(y[c], denom, inv) : 0.0f;
            }
        } else {
            const float ninf = __int_as_float(0xff800000);
            float mm = __uint_as_float(0x7fc00000u);  // NaN = "no value yet"
            for (uint64_t c = threadIdx.x; c < side; c += kDiagThreads) mm = max_nn(mm, c < kept ? x[c] : ninf);
            mm = group_max<kDiagThreads>(mm, &red);
            const float first = x[0];
            if (is_nan(first)) mm = first;  // reductions.rs:572: the scan starts from column 0
            double acc = 0.0;
            for (uint64_t c = threadIdx.x; c < side; c += kDiagThreads) {
                const float e = lm_exp(f_sub(c < kept ? x[c] : ninf, mm));
                y[c] = e;
                acc += (double)e;
            }
            acc = group_sum<kDiagThreads>(acc, &red);
            const float denom = __double2float_rn(acc);
            for (uint64_t c = threadIdx.x; c < side; c += kDiagThreads) y[c] = f_div(y[c], denom);
        }
        if (!isfinite(m)) __syncthreads();  // after the exact path, before the next row's fast maximum
    }
}

template <int MODE>
cudaError_t launch_diag_mode(const LaunchEnv& env, const DiagPlan& p) {
    const uint64_t cap = (uint64_t)env.sm_count * 8;
    const dim3 grid((unsigned)(p.side < cap ? p.side : cap));
    if (p.vec) return launch_dependent(diag_rows<MODE, true>, grid, dim3(kDiagThreads), 0, env.stream, p);
    return launch_dependent(diag_rows<MODE, false>, grid, dim3(kDiagThreads), 0, env.stream, p);
}

}  // namespace

cudaError_t launch_diag(const LaunchEnv& env, const DiagPlan& p, int mode) {
    cudaError_t err;
    switch (mode) {
    case kDiagSoftMaxCausal: {
        const uint64_t cap = (uint64_t)env.sm_count * 8;
        const dim3 grid((unsigned)(p.side < cap ? p.side : cap));
        err = p.vec ? launch_dependent(softmax_causal_rows<true>, grid, dim3(kDiagThreads), 0, env.stream, p)
                    : launch_dependent(softmax_causal_rows<false>, grid, dim3(kDiagThreads), 0, env.stream, p);
        break;
    }
    case kDiag: err = launch_diag_mode<kDiag>(env, p); break;
    case kDiagMaskInf: err = launch_diag_mode<kDiagMaskInf>(env, p); break;
    default: err = launch_diag_mode<kDiagMaskZero>(env, p); break;
    }
    ++*env.launches;
    return err != cudaSuccess ? err : cudaGetLastError();
}

}  // namespace emel
