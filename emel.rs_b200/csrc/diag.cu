// Diagonal family (diag.rs OpDiag / OpDiagMaskInf / OpDiagMaskZero) on the
// device: flat F32 slices holding a side x side row-major matrix.
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

#include "launch.hpp"
#include "pdl.cuh"

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
    case kDiag: err = launch_diag_mode<kDiag>(env, p); break;
    case kDiagMaskInf: err = launch_diag_mode<kDiagMaskInf>(env, p); break;
    default: err = launch_diag_mode<kDiagMaskZero>(env, p); break;
    }
    ++*env.launches;
    return err != cudaSuccess ? err : cudaGetLastError();
}

}  // namespace emel
