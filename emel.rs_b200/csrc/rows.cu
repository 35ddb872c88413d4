// Row kernels: norm, rms_norm (optionally fused with a row-broadcast weight),
// soft_max (optionally scaled and masked), sum_rows and per-row argmax.
//
// A "row" is ne0 consecutive logical ordinals (normalization.rs:307-311,
// reductions.rs:497-500).  norm, rms_norm and soft_max need every element of
// a row twice (statistic, then output), so the row is held in registers and
// read from HBM exactly once:
//   * G threads own one row, each holding up to kMaxE elements;
//     G = 32 (rows <= 1 Ki), 256 (<= 8 Ki) or 1024 (<= 32 Ki elements);
//   * rows longer than one CTA can hold (vocabulary logits, 151936 wide) are
//     split across a thread-block cluster of up to 8 CTAs that exchange
//     their partial maxima and sums through distributed shared memory;
//   * rows beyond a cluster's capacity fall back to a streaming kernel that
//     reads the row once per pass.
// sum_rows and argmax stream their rows (no residency needed).
// Reductions accumulate in f64 where the reference does (normalization.rs:
// 323-334, 350-355; reductions.rs:582-590, 690-695); only the summation
// order differs from the reference's sequential loop, which moves the f64
// accumulator by a few ulp of f64 and the f32 result almost never.
// soft_max over non-dense views keeps the reference's sequential f32 sum
// (reductions.rs:620-626) exactly: one thread adds the row in order.
#include <cooperative_groups.h>

#include "common.cuh"
#include "launch.hpp"
#include "rowreduce.cuh"

namespace cg = cooperative_groups;

namespace emel {

namespace {

constexpr int kMaxE = 32;  // elements per thread for register-resident rows

// ---------------------------------------------------------------------------
// Row addressing.
// ---------------------------------------------------------------------------
__device__ __forceinline__ int64_t row_base(const RowOperand& o, uint64_t r, uint64_t ne1, uint64_t ne2) {
    const uint64_t i1 = r % ne1, q = r / ne1, i2 = q % ne2, i3 = q / ne2;
    return (int64_t)i1 * o.st[1] + (int64_t)i2 * o.st[2] + (int64_t)i3 * o.st[3];
}

// Mask row (i1, i2 % m2, i3 % m3) of a soft_max_ext mask.
__device__ __forceinline__ int64_t mask_row_base(const RowOperand& m, uint64_t r, uint64_t ne1, uint64_t ne2) {
    const uint64_t i1 = r % ne1, q = r / ne1, i2 = q % ne2, i3 = q / ne2;
    return (int64_t)i1 * m.st[1] + (int64_t)(i2 % m.ne[2]) * m.st[2] + (int64_t)(i3 % m.ne[3]) * m.st[3];
}

__device__ __forceinline__ float load_aux(const RowOperand& a, int dtype, int64_t elem) {
    if (dtype == (int)DType::F16) return f16_bits_to_f32(reinterpret_cast<const uint16_t*>(a.ptr)[elem]);
    return reinterpret_cast<const float*>(a.ptr)[elem];
}

// Element c of the thread's slot j (VEC consecutive elements per slot).
template <int G, int VEC>
__device__ __forceinline__ uint64_t slot_col(int j, int lane, int k, uint64_t col0) {
    return col0 + ((uint64_t)j * G + lane) * VEC + k;
}

// Loads this thread's share of a row [col0, col1) into x[]; absent -> NaN-free 0.
template <int G, int VEC>
__device__ __forceinline__ void load_row(float (&x)[kMaxE], const float* base, int64_t st0, uint64_t col0,
                                         uint64_t col1, int lane) {
    constexpr int SLOTS = kMaxE / VEC;
#pragma unroll
    for (int j = 0; j < SLOTS; ++j) {
        const uint64_t c = slot_col<G, VEC>(j, lane, 0, col0);
        if constexpr (VEC == 4) {
            if (c + 3 < col1) {
                const float4 v = __ldcs(reinterpret_cast<const float4*>(base + c));
                x[j * 4 + 0] = v.x;
                x[j * 4 + 1] = v.y;
                x[j * 4 + 2] = v.z;
                x[j * 4 + 3] = v.w;
            } else {
#pragma unroll
                for (int k = 0; k < 4; ++k) x[j * 4 + k] = (c + k < col1) ? base[c + k] : 0.0f;
            }
        } else {
            x[j] = c < col1 ? base[(int64_t)c * st0] : 0.0f;
        }
    }
}

template <int G, int VEC>
__device__ __forceinline__ void store_row(const float (&y)[kMaxE], float* base, int64_t st0, uint64_t col0,
                                          uint64_t col1, int lane) {
    constexpr int SLOTS = kMaxE / VEC;
#pragma unroll
    for (int j = 0; j < SLOTS; ++j) {
        const uint64_t c = slot_col<G, VEC>(j, lane, 0, col0);
        if constexpr (VEC == 4) {
            if (c + 3 < col1) {
                __stcs(reinterpret_cast<float4*>(base + c), make_float4(y[j * 4], y[j * 4 + 1], y[j * 4 + 2], y[j * 4 + 3]));
            } else {
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    if (c + k < col1) base[c + k] = y[j * 4 + k];
            }
        } else {
            if (c < col1) base[(int64_t)c * st0] = y[j];
        }
    }
}

template <int G, int VEC>
__device__ __forceinline__ bool owns(int j, int k, int lane, uint64_t col0, uint64_t col1) {
    return slot_col<G, VEC>(j / VEC, lane, k, col0) < col1;
}

// ---------------------------------------------------------------------------
// norm / rms_norm / rms_norm * weight  (normalization.rs:316-362)
// ---------------------------------------------------------------------------
template <int G, int VEC, int OP>
__global__ void __launch_bounds__(G > 256 ? G : 256) norm_rows(RowPlan p, float eps) {
    constexpr int CTA = G > 256 ? G : 256;
    constexpr int ROWS_PER_CTA = CTA / G;
    __shared__ GroupScratch<G> scratch[ROWS_PER_CTA];
    const int lane = threadIdx.x % G, sub = threadIdx.x / G;
    GroupScratch<G>* s = &scratch[sub];
    const uint64_t ne0 = p.ne[0];
    for (uint64_t r = (uint64_t)blockIdx.x * ROWS_PER_CTA + sub; r < p.rows; r += (uint64_t)gridDim.x * ROWS_PER_CTA) {
        const float* xrow = reinterpret_cast<const float*>(p.src.ptr) + row_base(p.src, r, p.ne[1], p.ne[2]);
        float* yrow = reinterpret_cast<float*>(p.dst.ptr) + row_base(p.dst, r, p.ne[1], p.ne[2]);
        float x[kMaxE];
        load_row<G, VEC>(x, xrow, p.src.st[0], 0, ne0, lane);
        double acc = 0.0;
#pragma unroll
        for (int e = 0; e < kMaxE; ++e) {
            if (!owns<G, VEC>(e, e % VEC, lane, 0, ne0)) continue;
            acc += OP == 0 ? (double)x[e] : (double)__fmul_rn(x[e], x[e]);
        }
        acc = group_sum<G>(acc, s);
        const float mean = __double2float_rn(acc / (double)ne0);
        float scale;
        if constexpr (OP == 0) {
            double vs = 0.0;
#pragma unroll
            for (int e = 0; e < kMaxE; ++e) {
                if (!owns<G, VEC>(e, e % VEC, lane, 0, ne0)) continue;
                const double c = (double)__fsub_rn(x[e], mean);
                vs += c * c;
            }
            vs = group_sum<G>(vs, s);
            const float variance = __double2float_rn(vs / (double)ne0);
            scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(variance, eps)));
#pragma unroll
            for (int e = 0; e < kMaxE; ++e) x[e] = f_mul(f_sub(x[e], mean), scale);
        } else {
            scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
#pragma unroll
            for (int e = 0; e < kMaxE; ++e) x[e] = f_mul(x[e], scale);
            if constexpr (OP == 2) {
                const float* w = reinterpret_cast<const float*>(p.aux.ptr);
#pragma unroll
                for (int e = 0; e < kMaxE; ++e) {
                    const uint64_t c = slot_col<G, VEC>(e / VEC, lane, e % VEC, 0);
                    if (c < ne0) x[e] = f_mul(x[e], __ldg(w + (int64_t)c * p.aux.st[0]));
                }
            }
        }
        store_row<G, VEC>(x, yrow, p.dst.st[0], 0, ne0, lane);
    }
}

// ---------------------------------------------------------------------------
// soft_max (reductions.rs:565-638) with optional scale and mask.
// ---------------------------------------------------------------------------
template <int G, int VEC>
__device__ __forceinline__ void scale_mask(float (&x)[kMaxE], const RowPlan& p, uint64_t r, uint64_t col0,
                                           uint64_t col1, int lane, bool apply_scale, float scale) {
    if (!apply_scale) return;
    int64_t mbase = 0;
    if (p.has_aux) mbase = mask_row_base(p.aux, r, p.ne[1], p.ne[2]);
#pragma unroll
    for (int e = 0; e < kMaxE; ++e) {
        const uint64_t c = slot_col<G, VEC>(e / VEC, lane, e % VEC, col0);
        if (c >= col1) continue;
        float v = f_mul(x[e], scale);
        if (p.has_aux) v = f_add(v, load_aux(p.aux, p.aux_dtype, mbase + (int64_t)c * p.aux.st[0]));
        x[e] = v;
    }
}

template <int G, int VEC>
__global__ void __launch_bounds__(G > 256 ? G : 256) softmax_rows(RowPlan p, bool apply_scale, float scale) {
    constexpr int CTA = G > 256 ? G : 256;
    constexpr int ROWS_PER_CTA = CTA / G;
    __shared__ GroupScratch<G> scratch[ROWS_PER_CTA];
    __shared__ float first_val[ROWS_PER_CTA];
    const int lane = threadIdx.x % G, sub = threadIdx.x / G;
    GroupScratch<G>* s = &scratch[sub];
    const uint64_t ne0 = p.ne[0];
    for (uint64_t r = (uint64_t)blockIdx.x * ROWS_PER_CTA + sub; r < p.rows; r += (uint64_t)gridDim.x * ROWS_PER_CTA) {
        const float* xrow = reinterpret_cast<const float*>(p.src.ptr) + row_base(p.src, r, p.ne[1], p.ne[2]);
        float* yrow = reinterpret_cast<float*>(p.dst.ptr) + row_base(p.dst, r, p.ne[1], p.ne[2]);
        float x[kMaxE];
        load_row<G, VEC>(x, xrow, p.src.st[0], 0, ne0, lane);
        scale_mask<G, VEC>(x, p, r, 0, ne0, lane, apply_scale, scale);
        float m = bitsf(0x7fc00000u);  // NaN = "no value yet"
#pragma unroll
        for (int e = 0; e < kMaxE; ++e)
            if (owns<G, VEC>(e, e % VEC, lane, 0, ne0)) m = max_nn(m, x[e]);
        if (lane == 0) first_val[sub] = x[0];
        m = group_max<G>(m, s);
        if constexpr (G <= 32) __syncwarp();
        else __syncthreads();
        if (is_nan(first_val[sub])) m = first_val[sub];  // reductions.rs:572: the scan starts from element 0
        double acc = 0.0;
#pragma unroll
        for (int e = 0; e < kMaxE; ++e) {
            x[e] = lm_exp(f_sub(x[e], m));
            if (owns<G, VEC>(e, e % VEC, lane, 0, ne0)) acc += (double)x[e];
        }
        acc = group_sum<G>(acc, s);
        const float denom = __double2float_rn(acc);
#pragma unroll
        for (int e = 0; e < kMaxE; ++e) x[e] = f_div(x[e], denom);
        store_row<G, VEC>(x, yrow, p.dst.st[0], 0, ne0, lane);
    }
}

// Non-dense views: the reference sums exp values sequentially in f32
// (reductions.rs:620-626).  One CTA per row stages exp values in shared
// memory and thread 0 adds them in row order.
// FIRST_PIN: the typed loop's scan starts from element 0, so a NaN there is
// the maximum (reductions.rs:572); the generic envelope's loop starts from
// -inf and skips NaNs (generic.rs:1966-1971).
template <bool FIRST_PIN>
__global__ void __launch_bounds__(256) softmax_rows_seq(RowPlan p, bool apply_scale, float scale) {
    extern __shared__ float ebuf[];
    __shared__ GroupScratch<256> s;
    __shared__ float total;
    const int lane = threadIdx.x;
    const uint64_t ne0 = p.ne[0];
    for (uint64_t r = blockIdx.x; r < p.rows; r += gridDim.x) {
        const float* xrow = reinterpret_cast<const float*>(p.src.ptr) + row_base(p.src, r, p.ne[1], p.ne[2]);
        float* yrow = reinterpret_cast<float*>(p.dst.ptr) + row_base(p.dst, r, p.ne[1], p.ne[2]);
        int64_t mbase = p.has_aux ? mask_row_base(p.aux, r, p.ne[1], p.ne[2]) : 0;
        float m = bitsf(0x7fc00000u);
        for (uint64_t c = lane; c < ne0; c += 256) {
            float v = xrow[(int64_t)c * p.src.st[0]];
            if (apply_scale) {
                v = f_mul(v, scale);
                if (p.has_aux) v = f_add(v, load_aux(p.aux, p.aux_dtype, mbase + (int64_t)c * p.aux.st[0]));
            }
            ebuf[c] = v;
            m = max_nn(m, v);
        }
        m = group_max<256>(m, &s);
        __syncthreads();
        if (FIRST_PIN && is_nan(ebuf[0])) m = ebuf[0];
        if (!FIRST_PIN && is_nan(m)) m = -INFINITY;  // no comparable value: the -inf start stays
        for (uint64_t c = lane; c < ne0; c += 256) ebuf[c] = lm_exp(f_sub(ebuf[c], m));
        __syncthreads();
        if (lane == 0) {
            float acc = 0.0f;
            for (uint64_t c = 0; c < ne0; ++c) acc = f_add(acc, ebuf[c]);
            total = acc;
        }
        __syncthreads();
        const float denom = total;
        for (uint64_t c = lane; c < ne0; c += 256) yrow[(int64_t)c * p.dst.st[0]] = f_div(ebuf[c], denom);
        __syncthreads();
    }
}

// Vocabulary-width rows: one cluster of CLUSTER CTAs (1024 threads each) per
// row; CTA k owns the k-th contiguous chunk.  Partial maxima and f64 sums
// are exchanged through distributed shared memory; the cluster barrier is a
// hardware barrier (no polling).
template <int CLUSTER>
__global__ void __launch_bounds__(1024) softmax_rows_cluster(RowPlan p, bool apply_scale, float scale, uint64_t chunk) {
    constexpr int G = 1024;
    __shared__ GroupScratch<G> s;
    __shared__ float part_max;
    __shared__ double part_sum;
    __shared__ float first_val;
    cg::cluster_group cluster = cg::this_cluster();
    const unsigned rank = cluster.block_rank();
    const int lane = threadIdx.x;
    const uint64_t ne0 = p.ne[0];
    const uint64_t r = blockIdx.x / CLUSTER;
    const uint64_t col0 = (uint64_t)rank * chunk;
    const uint64_t col1 = col0 + chunk < ne0 ? col0 + chunk : ne0;
    const float* xrow = reinterpret_cast<const float*>(p.src.ptr) + row_base(p.src, r, p.ne[1], p.ne[2]);
    float* yrow = reinterpret_cast<float*>(p.dst.ptr) + row_base(p.dst, r, p.ne[1], p.ne[2]);
    float x[kMaxE];
    load_row<G, 4>(x, xrow, 1, col0, col1, lane);
    scale_mask<G, 4>(x, p, r, col0, col1, lane, apply_scale, scale);
    float m = bitsf(0x7fc00000u);
#pragma unroll
    for (int e = 0; e < kMaxE; ++e)
        if (owns<G, 4>(e, e % 4, lane, col0, col1)) m = max_nn(m, x[e]);
    m = group_max<G>(m, &s);
    if (lane == 0) {
        part_max = m;
        first_val = x[0];
    }
    cluster.sync();
    float gm = bitsf(0x7fc00000u);
#pragma unroll
    for (int k = 0; k < CLUSTER; ++k) gm = max_nn(gm, *cluster.map_shared_rank(&part_max, k));
    const float f0 = *cluster.map_shared_rank(&first_val, 0);
    if (is_nan(f0)) gm = f0;
    double acc = 0.0;
#pragma unroll
    for (int e = 0; e < kMaxE; ++e) {
        x[e] = lm_exp(f_sub(x[e], gm));
        if (owns<G, 4>(e, e % 4, lane, col0, col1)) acc += (double)x[e];
    }
    acc = group_sum<G>(acc, &s);
    if (lane == 0) part_sum = acc;
    cluster.sync();
    double total = 0.0;
#pragma unroll
    for (int k = 0; k < CLUSTER; ++k) total += *cluster.map_shared_rank(&part_sum, k);
    const float denom = __double2float_rn(total);
#pragma unroll
    for (int e = 0; e < kMaxE; ++e) x[e] = f_div(x[e], denom);
    store_row<G, 4>(x, yrow, 1, col0, col1, lane);
    cluster.sync();  // keep this CTA's shared memory alive until every peer has read it
}

// ---------------------------------------------------------------------------
// sum_rows (reductions.rs:684-700) and per-row argmax (the 715-730 scan).
// ---------------------------------------------------------------------------
template <int G>
__global__ void __launch_bounds__(G > 256 ? G : 256) sum_rows_kernel(RowPlan p) {
    constexpr int CTA = G > 256 ? G : 256;
    constexpr int ROWS_PER_CTA = CTA / G;
    __shared__ GroupScratch<G> scratch[ROWS_PER_CTA];
    const int lane = threadIdx.x % G, sub = threadIdx.x / G;
    const uint64_t ne0 = p.ne[0];
    for (uint64_t r = (uint64_t)blockIdx.x * ROWS_PER_CTA + sub; r < p.rows; r += (uint64_t)gridDim.x * ROWS_PER_CTA) {
        const float* xrow = reinterpret_cast<const float*>(p.src.ptr) + row_base(p.src, r, p.ne[1], p.ne[2]);
        double acc = 0.0;
        if (p.vec) {
            for (uint64_t c = (uint64_t)lane * 4; c < ne0; c += (uint64_t)G * 4) {
                const float4 v = __ldcs(reinterpret_cast<const float4*>(xrow + c));
                acc += (double)v.x;
                acc += (double)v.y;
                acc += (double)v.z;
                acc += (double)v.w;
            }
        } else {
            for (uint64_t c = lane; c < ne0; c += G) acc += (double)xrow[(int64_t)c * p.src.st[0]];
        }
        acc = group_sum<G>(acc, &scratch[sub]);
        if (lane == 0) {
            float* yrow = reinterpret_cast<float*>(p.dst.ptr) + row_base(p.dst, r, p.ne[1], p.ne[2]);
            *yrow = __double2float_rn(acc);
        }
    }
}

__device__ __forceinline__ void arg_step(ArgBest& b, float v, int64_t i) {
    if ((!b.has && !is_nan(v)) || v > b.v) {
        b.v = v;
        b.i = i;
        b.has = 1;
    }
}

template <int G>
__global__ void __launch_bounds__(G > 256 ? G : 256) argmax_rows_kernel(RowPlan p, int dst_dtype) {
    constexpr int CTA = G > 256 ? G : 256;
    constexpr int ROWS_PER_CTA = CTA / G;
    __shared__ GroupScratch<G> scratch[ROWS_PER_CTA];
    const int lane = threadIdx.x % G, sub = threadIdx.x / G;
    const uint64_t ne0 = p.ne[0];
    for (uint64_t r = (uint64_t)blockIdx.x * ROWS_PER_CTA + sub; r < p.rows; r += (uint64_t)gridDim.x * ROWS_PER_CTA) {
        const float* xrow = reinterpret_cast<const float*>(p.src.ptr) + row_base(p.src, r, p.ne[1], p.ne[2]);
        ArgBest b{0.0f, 0, 0};
        if (p.vec) {
            for (uint64_t c = (uint64_t)lane * 4; c < ne0; c += (uint64_t)G * 4) {
                const float4 v = __ldcs(reinterpret_cast<const float4*>(xrow + c));
                arg_step(b, v.x, (int64_t)c);
                arg_step(b, v.y, (int64_t)c + 1);
                arg_step(b, v.z, (int64_t)c + 2);
                arg_step(b, v.w, (int64_t)c + 3);
            }
        } else {
            for (uint64_t c = lane; c < ne0; c += G) arg_step(b, xrow[(int64_t)c * p.src.st[0]], (int64_t)c);
        }
        b = group_argmax<G>(b, &scratch[sub]);
        if (lane == 0) {
            const int64_t idx = (is_nan(xrow[0]) || !b.has) ? 0 : b.i;
            const int64_t off = row_base(p.dst, r, p.ne[1], p.ne[2]);
            if (dst_dtype == (int)DType::I64) reinterpret_cast<int64_t*>(p.dst.ptr)[off] = idx;
            else if (dst_dtype == (int)DType::I32) reinterpret_cast<int32_t*>(p.dst.ptr)[off] = (int32_t)idx;
            else reinterpret_cast<float*>(p.dst.ptr)[off] = (float)idx;
        }
    }
}

uint32_t row_grid(const LaunchEnv& env, uint64_t rows, int rows_per_cta, int ctas_per_sm) {
    const uint64_t want = (rows + rows_per_cta - 1) / rows_per_cta;
    const uint64_t cap = (uint64_t)env.sm_count * ctas_per_sm * 16;
    const uint64_t g = want < cap ? want : cap;
    return (uint32_t)(g == 0 ? 1 : g);
}

template <int G>
constexpr int cta_of() {
    return G > 256 ? G : 256;
}

// ---------------------------------------------------------------------------
// Streaming fallbacks for rows no register tier holds (or non-dense softmax
// rows beyond shared memory): one 1024-thread CTA per row re-reads the row
// for each pass; identical arithmetic to the resident kernels.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float* dst_elem(const RowPlan& p, uint64_t r, uint64_t c) {
    if (!p.dst_ordinal) {
        return reinterpret_cast<float*>(p.dst.ptr) + row_base(p.dst, r, p.ne[1], p.ne[2]) + (int64_t)c * p.dst.st[0];
    }
    uint64_t ordinal = r * p.ne[0] + c;
    int64_t off = 0;
#pragma unroll
    for (int d = 0; d < 4; ++d) {
        off += (int64_t)(ordinal % p.dst.ne[d]) * p.dst.st[d];
        ordinal /= p.dst.ne[d];
    }
    return reinterpret_cast<float*>(p.dst.ptr) + off;
}

// OP 0 norm, 1 rms_norm, 2 rms_norm * weight (normalization.rs:316-362);
// OP 3 / 4: the generic envelope's norm / rms_norm (generic.rs:1992-2050),
// whose variance squares in binary32 and whose scale is 1 / sqrt(. + eps)
// evaluated in binary64 and rounded once.
template <int OP>
__global__ void __launch_bounds__(1024) norm_rows_stream(RowPlan p, float eps) {
    __shared__ GroupScratch<1024> s;
    constexpr bool kNorm = OP == 0 || OP == 3;
    constexpr bool kGeneric = OP >= 3;
    const uint64_t ne0 = p.ne[0];
    for (uint64_t r = blockIdx.x; r < p.rows; r += gridDim.x) {
        const float* xrow = reinterpret_cast<const float*>(p.src.ptr) + row_base(p.src, r, p.ne[1], p.ne[2]);
        const int64_t st0 = p.src.st[0];
        double acc = 0.0;
        for (uint64_t c = threadIdx.x; c < ne0; c += 1024) {
            const float x = xrow[(int64_t)c * st0];
            acc += kNorm ? (double)x : (double)__fmul_rn(x, x);
        }
        acc = group_sum<1024>(acc, &s);
        const float mean = __double2float_rn(acc / (double)ne0);
        float scale;
        if constexpr (kNorm) {
            double vs = 0.0;
            for (uint64_t c = threadIdx.x; c < ne0; c += 1024) {
                const float cf = __fsub_rn(xrow[(int64_t)c * st0], mean);
                if constexpr (kGeneric) {
                    vs += (double)__fmul_rn(cf, cf);
                } else {
                    const double d = (double)cf;
                    vs += d * d;
                }
            }
            vs = group_sum<1024>(vs, &s);
            if constexpr (kGeneric) {
                scale = __double2float_rn(__ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(vs / (double)ne0, (double)eps))));
            } else {
                const float variance = __double2float_rn(vs / (double)ne0);
                scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(variance, eps)));
            }
        } else if constexpr (kGeneric) {
            scale = __double2float_rn(__ddiv_rn(1.0, __dsqrt_rn(__dadd_rn((double)mean, (double)eps))));
        } else {
            scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
        }
        for (uint64_t c = threadIdx.x; c < ne0; c += 1024) {
            const float x = xrow[(int64_t)c * st0];
            float y = kNorm ? f_mul(f_sub(x, mean), scale) : f_mul(x, scale);
            if constexpr (OP == 2) y = f_mul(y, reinterpret_cast<const float*>(p.aux.ptr)[(int64_t)c * p.aux.st[0]]);
            dst_elem(p, r, c)[0] = y;
        }
    }
}

// soft_max over rows re-read per pass.  Dense layouts sum in f64 across the
// CTA; non-dense layouts keep the reference's sequential f32 sum by having
// thread 0 walk the row in order (correct for any width, slow by design).
template <bool FIRST_PIN>
__global__ void __launch_bounds__(1024) softmax_rows_stream(RowPlan p, bool apply_scale, float scale) {
    __shared__ GroupScratch<1024> s;
    __shared__ float total;
    const uint64_t ne0 = p.ne[0];
    for (uint64_t r = blockIdx.x; r < p.rows; r += gridDim.x) {
        const float* xrow = reinterpret_cast<const float*>(p.src.ptr) + row_base(p.src, r, p.ne[1], p.ne[2]);
        const int64_t mbase = p.has_aux ? mask_row_base(p.aux, r, p.ne[1], p.ne[2]) : 0;
        auto value = [&](uint64_t c) {
            float v = xrow[(int64_t)c * p.src.st[0]];
            if (apply_scale) {
                v = f_mul(v, scale);
                if (p.has_aux) v = f_add(v, load_aux(p.aux, p.aux_dtype, mbase + (int64_t)c * p.aux.st[0]));
            }
            return v;
        };
        float m = bitsf(0x7fc00000u);
        for (uint64_t c = threadIdx.x; c < ne0; c += 1024) m = max_nn(m, value(c));
        m = group_max<1024>(m, &s);
        const float v0 = value(0);
        if (FIRST_PIN && is_nan(v0)) m = v0;
        if (!FIRST_PIN && is_nan(m)) m = -INFINITY;
        if (p.dense) {
            double acc = 0.0;
            for (uint64_t c = threadIdx.x; c < ne0; c += 1024) acc += (double)lm_exp(f_sub(value(c), m));
            acc = group_sum<1024>(acc, &s);
            if (threadIdx.x == 0) total = __double2float_rn(acc);
        } else if (threadIdx.x == 0) {
            float acc = 0.0f;
            for (uint64_t c = 0; c < ne0; ++c) acc = f_add(acc, lm_exp(f_sub(value(c), m)));
            total = acc;
        }
        __syncthreads();
        const float denom = total;
        for (uint64_t c = threadIdx.x; c < ne0; c += 1024) dst_elem(p, r, c)[0] = f_div(lm_exp(f_sub(value(c), m)), denom);
        __syncthreads();
    }
}

}  // namespace

// Threads per row for register-resident rows: the smallest group whose
// registers hold the row.
static int resident_group(uint64_t ne0) {
    if (ne0 <= 32ull * kMaxE) return 32;
    if (ne0 <= 256ull * kMaxE) return 256;
    if (ne0 <= 1024ull * kMaxE) return 1024;
    return 0;
}

#define EMEL_NORM_LAUNCH(G, VEC, OP)                                                                          \
    norm_rows<G, VEC, OP><<<row_grid(env, p.rows, cta_of<G>() / G, 2048 / cta_of<G>()), cta_of<G>(), 0, env.stream>>>(p, eps)

cudaError_t launch_norm(const LaunchEnv& env, const RowPlan& p, int op, float eps) {
    cudaError_t ring_err;
    if (launch_row_ring(env, p, op, eps, false, &ring_err)) return ring_err;
    const int g = resident_group(p.ne[0]);
    if (g == 0) {
        const uint32_t grid = row_grid(env, p.rows, 1, 2);
        if (op == 0) norm_rows_stream<0><<<grid, 1024, 0, env.stream>>>(p, eps);
        else if (op == 1) norm_rows_stream<1><<<grid, 1024, 0, env.stream>>>(p, eps);
        else norm_rows_stream<2><<<grid, 1024, 0, env.stream>>>(p, eps);
        ++*env.launches;
        return cudaGetLastError();
    }
#define EMEL_NORM_G(G)                                                  \
    if (g == G) {                                                       \
        if (p.vec) {                                                    \
            if (op == 0) EMEL_NORM_LAUNCH(G, 4, 0);                     \
            else if (op == 1) EMEL_NORM_LAUNCH(G, 4, 1);                \
            else EMEL_NORM_LAUNCH(G, 4, 2);                             \
        } else {                                                        \
            if (op == 0) EMEL_NORM_LAUNCH(G, 1, 0);                     \
            else if (op == 1) EMEL_NORM_LAUNCH(G, 1, 1);                \
            else EMEL_NORM_LAUNCH(G, 1, 2);                             \
        }                                                               \
    }
    EMEL_NORM_G(32) else EMEL_NORM_G(256) else EMEL_NORM_G(1024)
#undef EMEL_NORM_G
    ++*env.launches;
    return cudaGetLastError();
}

// The generic envelope's norm (op 3) / rms_norm (op 4): the ring when the
// view qualifies, else one 1024-thread CTA per row.
cudaError_t launch_norm_generic(const LaunchEnv& env, const RowPlan& p, int op, float eps) {
    cudaError_t ring_err;
    if (!p.dst_ordinal && launch_row_ring(env, p, op == 3 ? 4 : 5, eps, false, &ring_err)) return ring_err;
    const uint32_t grid = row_grid(env, p.rows, 1, 2);
    if (op == 3) norm_rows_stream<3><<<grid, 1024, 0, env.stream>>>(p, eps);
    else norm_rows_stream<4><<<grid, 1024, 0, env.stream>>>(p, eps);
    ++*env.launches;
    return cudaGetLastError();
}

// The generic envelope's soft_max (generic.rs:1952-1989): maximum from -inf
// over non-NaN values, exp written out, a sequential binary32 sum per row,
// then a division.  Rows that fit in shared memory are staged there; longer
// ones are re-read.
cudaError_t launch_soft_max_generic(const LaunchEnv& env, const RowPlan& p) {
    if (!p.dst_ordinal && p.ne[0] * sizeof(float) <= 200 * 1024) {
        const size_t smem = p.ne[0] * sizeof(float);
        cudaFuncSetAttribute(softmax_rows_seq<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        softmax_rows_seq<false><<<row_grid(env, p.rows, 1, 8), 256, smem, env.stream>>>(p, false, 1.0f);
    } else {
        RowPlan q = p;
        q.dense = false;  // the sequential binary32 sum
        softmax_rows_stream<false><<<row_grid(env, p.rows, 1, 2), 1024, 0, env.stream>>>(q, false, 1.0f);
    }
    ++*env.launches;
    return cudaGetLastError();
}

uint64_t soft_max_cluster_capacity() { return 8ull * 1024 * kMaxE; }

cudaError_t launch_soft_max(const LaunchEnv& env, const RowPlan& p, bool apply_scale, float scale) {
    cudaError_t ring_err;
    if (launch_row_ring(env, p, 3, scale, apply_scale, &ring_err)) return ring_err;
    if (p.dense && split_rows_wanted(env, p)) return launch_soft_max_split(env, p, apply_scale, scale);
    const bool long_row = resident_group(p.ne[0]) == 0 && (!p.vec || p.ne[0] > soft_max_cluster_capacity());
    if (p.dst_ordinal || (!p.dense && p.ne[0] * sizeof(float) > 200 * 1024) || (p.dense && long_row)) {
        softmax_rows_stream<true><<<row_grid(env, p.rows, 1, 2), 1024, 0, env.stream>>>(p, apply_scale, scale);
        ++*env.launches;
        return cudaGetLastError();
    }
    if (!p.dense) {
        const size_t smem = p.ne[0] * sizeof(float);
        cudaFuncSetAttribute(softmax_rows_seq<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        softmax_rows_seq<true><<<row_grid(env, p.rows, 1, 8), 256, smem, env.stream>>>(p, apply_scale, scale);
        ++*env.launches;
        return cudaGetLastError();
    }
    const int g = resident_group(p.ne[0]);
    if (g != 0) {
#define EMEL_SM_LAUNCH(G, VEC) \
    softmax_rows<G, VEC><<<row_grid(env, p.rows, cta_of<G>() / G, 2048 / cta_of<G>()), cta_of<G>(), 0, env.stream>>>(p, apply_scale, scale)
        if (g == 32) {
            if (p.vec) EMEL_SM_LAUNCH(32, 4); else EMEL_SM_LAUNCH(32, 1);
        } else if (g == 256) {
            if (p.vec) EMEL_SM_LAUNCH(256, 4); else EMEL_SM_LAUNCH(256, 1);
        } else {
            if (p.vec) EMEL_SM_LAUNCH(1024, 4); else EMEL_SM_LAUNCH(1024, 1);
        }
#undef EMEL_SM_LAUNCH
        ++*env.launches;
        return cudaGetLastError();
    }
    if (!p.vec || p.ne[0] > soft_max_cluster_capacity()) return cudaErrorInvalidValue;
    // Smallest cluster (2, 4 or 8 CTAs) whose registers hold the row; the
    // chunk is a multiple of 4 so every CTA's first column stays 16-byte aligned.
    int cluster = 2;
    while ((uint64_t)cluster * 1024 * kMaxE < p.ne[0]) cluster *= 2;
    uint64_t chunk = (p.ne[0] + cluster - 1) / cluster;
    chunk = (chunk + 3) / 4 * 4;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(p.rows * cluster));
    cfg.blockDim = dim3(1024);
    cfg.stream = env.stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cluster;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t err;
    if (cluster == 2) err = cudaLaunchKernelEx(&cfg, softmax_rows_cluster<2>, p, apply_scale, scale, chunk);
    else if (cluster == 4) err = cudaLaunchKernelEx(&cfg, softmax_rows_cluster<4>, p, apply_scale, scale, chunk);
    else err = cudaLaunchKernelEx(&cfg, softmax_rows_cluster<8>, p, apply_scale, scale, chunk);
    ++*env.launches;
    return err != cudaSuccess ? err : cudaGetLastError();
}

static int stream_group(uint64_t ne0) {
    if (ne0 <= 2048) return 32;
    if (ne0 <= 65536) return 256;
    return 1024;
}

cudaError_t launch_sum_rows(const LaunchEnv& env, const RowPlan& p) {
    if (split_rows_wanted(env, p)) return launch_sum_rows_split(env, p);
    const int g = stream_group(p.ne[0]);
    if (g == 32) sum_rows_kernel<32><<<row_grid(env, p.rows, 8, 8), 256, 0, env.stream>>>(p);
    else if (g == 256) sum_rows_kernel<256><<<row_grid(env, p.rows, 1, 8), 256, 0, env.stream>>>(p);
    else sum_rows_kernel<1024><<<row_grid(env, p.rows, 1, 2), 1024, 0, env.stream>>>(p);
    ++*env.launches;
    return cudaGetLastError();
}

cudaError_t launch_argmax_rows(const LaunchEnv& env, const RowPlan& p, int dst_dtype) {
    if (split_rows_wanted(env, p)) return launch_argmax_rows_split(env, p, dst_dtype);
    const int g = stream_group(p.ne[0]);
    if (g == 32) argmax_rows_kernel<32><<<row_grid(env, p.rows, 8, 8), 256, 0, env.stream>>>(p, dst_dtype);
    else if (g == 256) argmax_rows_kernel<256><<<row_grid(env, p.rows, 1, 8), 256, 0, env.stream>>>(p, dst_dtype);
    else argmax_rows_kernel<1024><<<row_grid(env, p.rows, 1, 2), 1024, 0, env.stream>>>(p, dst_dtype);
    ++*env.launches;
    return cudaGetLastError();
}

}  // namespace emel
