// Row operators over few, long rows (vocabulary logits: 151,936 columns,
// tens of rows): one thread-block cluster of kSplitCluster CTAs per row, CTA
// k owning the k-th contiguous chunk of columns, partial results exchanged
// through distributed shared memory and folded in rank order (so the result
// does not depend on timing).  One CTA per row would leave most SMs idle.
//
//   * argmax_rows: one pass; partial (value, index) per CTA, earliest index
//     on ties, NaN at column 0 pins the index to 0 (reductions.rs:715-730);
//   * sum_rows: one pass; f64 partial per CTA (reductions.rs:684-700);
//   * soft_max (dense views): pass 1 reads the chunk from HBM for the
//     maximum, pass 2 re-reads it (from L2: a cluster's chunks are in flight
//     together) and writes e = exp(v - max) to dst, pass 3 divides dst by
//     the f64 sum in place.  The fast/exact split is the ring kernel's: plain
//     IEEE arithmetic unless a NaN or a non-finite maximum shows up, in which
//     case every CTA of the cluster redoes the row with the x86 NaN rules.
#include <cooperative_groups.h>

#include "common.cuh"
#include "launch.hpp"
#include "pdl.cuh"
#include "rowreduce.cuh"

namespace cg = cooperative_groups;

namespace emel {

namespace {

constexpr int kSplitThreads = 256;
constexpr int kSplitCluster = 8;
constexpr int kSplitCtasPerSm = 4;  // register cap: 148 SMs x 4 >= 64 vocabulary rows x 8 CTAs, all resident

__device__ __forceinline__ int64_t split_row_base(const RowOperand& o, uint64_t r, uint64_t ne1, uint64_t ne2) {
    const uint64_t i1 = r % ne1, q = r / ne1, i2 = q % ne2, i3 = q / ne2;
    return (int64_t)i1 * o.st[1] + (int64_t)i2 * o.st[2] + (int64_t)i3 * o.st[3];
}

__device__ __forceinline__ int64_t split_mask_base(const RowOperand& m, uint64_t r, uint64_t ne1, uint64_t ne2) {
    const uint64_t i1 = r % ne1, q = r / ne1, i2 = q % ne2, i3 = q / ne2;
    return (int64_t)i1 * m.st[1] + (int64_t)(i2 % m.ne[2]) * m.st[2] + (int64_t)(i3 % m.ne[3]) * m.st[3];
}

struct Chunk {
    uint64_t col0, col1;
};

// Visits the 16-byte vectors v0 + tid, v0 + tid + T, ... below v1, issuing U
// loads before using any of them, the last batch included (its loads past
// v1 are skipped): one load in flight per thread would leave the chunk's
// passes latency-bound.
template <int U, typename Load, typename Use>
__device__ __forceinline__ void batched(uint64_t v0, uint64_t v1, Load load, Use use) {
    uint64_t v = v0 + threadIdx.x;
    for (; v + (U - 1) * kSplitThreads < v1; v += U * kSplitThreads) {
        float4 q[U];
#pragma unroll
        for (int k = 0; k < U; ++k) q[k] = load(v + k * kSplitThreads);
#pragma unroll
        for (int k = 0; k < U; ++k) use(v + k * kSplitThreads, q[k]);
    }
    if (v < v1) {  // the partial last batch, its loads still issued together
        float4 q[U];
#pragma unroll
        for (int k = 0; k < U; ++k)
            if (v + k * kSplitThreads < v1) q[k] = load(v + k * kSplitThreads);
#pragma unroll
        for (int k = 0; k < U; ++k)
            if (v + k * kSplitThreads < v1) use(v + k * kSplitThreads, q[k]);
    }
}

// NaN-propagating maximum (PTX max.NaN): a NaN anywhere in a chunk reaches
// the row's maximum.
__device__ __forceinline__ float max_nan(float a, float b) {
    float d;
    asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
    return d;
}

__device__ __forceinline__ Chunk my_chunk(uint64_t ne0, uint64_t chunk, unsigned rank) {
    const uint64_t c0 = (uint64_t)rank * chunk;
    return Chunk{c0 < ne0 ? c0 : ne0, c0 + chunk < ne0 ? c0 + chunk : ne0};
}

__device__ __forceinline__ void arg_take(ArgBest& b, float v, int64_t i) {
    if ((!b.has && !is_nan(v)) || v > b.v) {
        b.v = v;
        b.i = i;
        b.has = 1;
    }
}

__global__ void __cluster_dims__(kSplitCluster, 1, 1) __launch_bounds__(kSplitThreads, kSplitCtasPerSm)
    argmax_rows_split(RowPlan p, int dst_dtype, uint64_t chunk) {
    pdl_enter();
    __shared__ GroupScratch<kSplitThreads> s;
    __shared__ float pv;
    __shared__ int64_t pi;
    __shared__ uint32_t ph;
    cg::cluster_group cluster = cg::this_cluster();
    const unsigned rank = cluster.block_rank();
    const uint64_t r = blockIdx.x / kSplitCluster;
    const Chunk ch = my_chunk(p.ne[0], chunk, rank);
    const float* row = reinterpret_cast<const float*>(p.src.ptr) + split_row_base(p.src, r, p.ne[1], p.ne[2]);
    ArgBest b{0.0f, 0, 0};
    if (p.vec) {
        // one (value, index) chain per vector lane, folded afterwards by
        // arg_better (larger value, then smaller index): the sequential
        // scan's answer, with four independent compare chains
        ArgBest bl[4] = {b, b, b, b};
        const float4* r4 = reinterpret_cast<const float4*>(row);
        batched<8>(ch.col0 / 4, ch.col1 / 4, [&](uint64_t v) { return __ldcs(r4 + v); },
                   [&](uint64_t v, float4 q) {
                       const int64_t c = (int64_t)v * 4;
                       arg_take(bl[0], q.x, c);
                       arg_take(bl[1], q.y, c + 1);
                       arg_take(bl[2], q.z, c + 2);
                       arg_take(bl[3], q.w, c + 3);
                   });
        b = arg_better(arg_better(bl[0], bl[1]), arg_better(bl[2], bl[3]));
    } else {
        for (uint64_t c = ch.col0 + threadIdx.x; c < ch.col1; c += kSplitThreads)
            arg_take(b, row[(int64_t)c * p.src.st[0]], (int64_t)c);
    }
    b = group_argmax<kSplitThreads>(b, &s);
    if (threadIdx.x == 0) {
        pv = b.v;
        pi = b.i;
        ph = b.has;
    }
    cluster.sync();
    if (rank == 0 && threadIdx.x == 0) {
        ArgBest best{0.0f, 0, 0};
        for (int k = 0; k < kSplitCluster; ++k)
            best = arg_better(best, ArgBest{*cluster.map_shared_rank(&pv, k), *cluster.map_shared_rank(&pi, k),
                                            *cluster.map_shared_rank(&ph, k)});
        const int64_t idx = (is_nan(row[0]) || !best.has) ? 0 : best.i;
        const int64_t off = split_row_base(p.dst, r, p.ne[1], p.ne[2]);
        if (dst_dtype == (int)DType::I64) reinterpret_cast<int64_t*>(p.dst.ptr)[off] = idx;
        else if (dst_dtype == (int)DType::I32) reinterpret_cast<int32_t*>(p.dst.ptr)[off] = (int32_t)idx;
        else reinterpret_cast<float*>(p.dst.ptr)[off] = (float)idx;
    }
    cluster.sync();  // peers' shared memory stays alive until rank 0 has read it
}

// argmax_rows without a cluster: the row's kSplitCluster CTAs are
// independent; each writes its chunk's (value, column) partial to the
// context workspace and takes a ticket on its row, and the CTA that takes
// the last ticket folds the row's partials in chunk order (earliest column
// on ties, NaN at column 0 pins 0) and re-arms the ticket.  No cluster
// scheduling and no cluster barrier; four (value, vector) chains per thread
// with fmaxf from a NaN start (three instructions per element).
struct ChunkPartial {
    float v;
    uint32_t has;
    int64_t i;
};

// early_batch: with `early` (the row is clear of the previous kernel's
// writes) the thread's first batch of U vectors of [v0, v1) is loaded before
// the wait for that kernel (pdl_enter) and used after it; returns where the
// batched walk continues.  Without it, waits first.
template <int U, typename Load, typename Use>
__device__ __forceinline__ uint64_t early_batch(bool early, uint64_t v0, uint64_t v1, Load load, Use use) {
    if (!early) {
        pdl_enter();
        return v0;
    }
    const uint64_t v = v0 + threadIdx.x;
    float4 q[U];
#pragma unroll
    for (int k = 0; k < U; ++k)
        if (v + k * kSplitThreads < v1) q[k] = load(v + k * kSplitThreads);
    pdl_enter();
#pragma unroll
    for (int k = 0; k < U; ++k)
        if (v + k * kSplitThreads < v1) use(v + k * kSplitThreads, q[k]);
    return v0 + (uint64_t)U * kSplitThreads;
}

__global__ void __launch_bounds__(kSplitThreads, kSplitCtasPerSm)
    argmax_rows_flat(RowPlan p, int dst_dtype, uint64_t chunk, ChunkPartial* partials, unsigned* tickets,
                     int early) {
    __shared__ GroupScratch<kSplitThreads> s;
    __shared__ bool is_last;
    const unsigned rank = blockIdx.x % kSplitCluster;
    const uint64_t r = blockIdx.x / kSplitCluster;
    const Chunk ch = my_chunk(p.ne[0], chunk, rank);
    const float* row = reinterpret_cast<const float*>(p.src.ptr) + split_row_base(p.src, r, p.ne[1], p.ne[2]);
    const float nan = __int_as_float(0x7fc00000);
    float bv[4] = {nan, nan, nan, nan};
    uint64_t bc[4] = {0, 0, 0, 0};
    const float4* r4 = reinterpret_cast<const float4*>(row);
    auto load = [&](uint64_t v) { return __ldcs(r4 + v); };
    auto use = [&](uint64_t v, float4 q) {
        const float q4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int l = 0; l < 4; ++l) {
            const float nb = fmaxf(bv[l], q4[l]);
            if (nb != bv[l]) bc[l] = v;
            bv[l] = nb;
        }
    };
    const uint64_t vstart = early_batch<8>(early != 0, ch.col0 / 4, ch.col1 / 4, load, use);
    batched<8>(vstart, ch.col1 / 4, load, use);
    ArgBest bl[4];
#pragma unroll
    for (int l = 0; l < 4; ++l) bl[l] = ArgBest{bv[l], (int64_t)(4 * bc[l] + l), is_nan(bv[l]) ? 0u : 1u};
    ArgBest b = arg_better(arg_better(bl[0], bl[1]), arg_better(bl[2], bl[3]));
    b = group_argmax<kSplitThreads>(b, &s);
    if (threadIdx.x == 0) {
        partials[r * kSplitCluster + rank] = ChunkPartial{b.v, b.has, b.i};
        __threadfence();
        is_last = atomicAdd(&tickets[r], 1u) == kSplitCluster - 1;
    }
    __syncthreads();
    if (!is_last || threadIdx.x != 0) return;
    __threadfence();
    ArgBest best{0.0f, 0, 0};
    for (int k = 0; k < kSplitCluster; ++k) {
        const ChunkPartial* q = partials + r * kSplitCluster + k;
        best = arg_better(best, ArgBest{__ldcg(&q->v), __ldcg(&q->i), __ldcg(&q->has)});
    }
    const int64_t idx = (is_nan(row[0]) || !best.has) ? 0 : best.i;
    const int64_t off = split_row_base(p.dst, r, p.ne[1], p.ne[2]);
    if (dst_dtype == (int)DType::I64) reinterpret_cast<int64_t*>(p.dst.ptr)[off] = idx;
    else if (dst_dtype == (int)DType::I32) reinterpret_cast<int32_t*>(p.dst.ptr)[off] = (int32_t)idx;
    else reinterpret_cast<float*>(p.dst.ptr)[off] = (float)idx;
    tickets[r] = 0u;
}

__global__ void __cluster_dims__(kSplitCluster, 1, 1) __launch_bounds__(kSplitThreads, kSplitCtasPerSm)
    sum_rows_split(RowPlan p, uint64_t chunk) {
    pdl_enter();
    __shared__ GroupScratch<kSplitThreads> s;
    __shared__ double part;
    cg::cluster_group cluster = cg::this_cluster();
    const unsigned rank = cluster.block_rank();
    const uint64_t r = blockIdx.x / kSplitCluster;
    const Chunk ch = my_chunk(p.ne[0], chunk, rank);
    const float* row = reinterpret_cast<const float*>(p.src.ptr) + split_row_base(p.src, r, p.ne[1], p.ne[2]);
    double acc = 0.0;
    if (p.vec) {
        const float4* r4 = reinterpret_cast<const float4*>(row);
        batched<8>(ch.col0 / 4, ch.col1 / 4, [&](uint64_t v) { return __ldcs(r4 + v); },
                   [&](uint64_t, float4 q) {
                       acc += (double)q.x;
                       acc += (double)q.y;
                       acc += (double)q.z;
                       acc += (double)q.w;
                   });
    } else {
        for (uint64_t c = ch.col0 + threadIdx.x; c < ch.col1; c += kSplitThreads) acc += (double)row[(int64_t)c * p.src.st[0]];
    }
    acc = group_sum<kSplitThreads>(acc, &s);
    if (threadIdx.x == 0) part = acc;
    cluster.sync();
    if (rank == 0 && threadIdx.x == 0) {
        double t = 0.0;
        for (int k = 0; k < kSplitCluster; ++k) t += *cluster.map_shared_rank(&part, k);
        reinterpret_cast<float*>(p.dst.ptr)[split_row_base(p.dst, r, p.ne[1], p.ne[2])] = __double2float_rn(t);
    }
    cluster.sync();
}

// --- soft_max -----------------------------------------------------------------
struct SoftmaxRow {
    const float* x;
    float* y;
    int64_t xs, ys;  // dim-0 strides (elements)
    int64_t mbase;
    bool has_mask;
};

__device__ __forceinline__ float mask_at(const RowPlan& p, const SoftmaxRow& w, uint64_t c) {
    const int64_t e = w.mbase + (int64_t)c * p.aux.st[0];
    return p.aux_dtype == (int)DType::F16 ? f16_bits_to_f32(reinterpret_cast<const uint16_t*>(p.aux.ptr)[e])
                                          : reinterpret_cast<const float*>(p.aux.ptr)[e];
}

template <bool EXACT>
__device__ __forceinline__ float value_at(const RowPlan& p, const SoftmaxRow& w, uint64_t c, bool apply_scale,
                                          float scale) {
    float v = w.x[(int64_t)c * w.xs];
    if (!apply_scale) return v;
    v = EXACT ? f_mul(v, scale) : __fmul_rn(v, scale);
    if (w.has_mask) v = EXACT ? f_add(v, mask_at(p, w, c)) : __fadd_rn(v, mask_at(p, w, c));
    return v;
}

__global__ void __cluster_dims__(kSplitCluster, 1, 1) __launch_bounds__(kSplitThreads, kSplitCtasPerSm)
    softmax_rows_split(RowPlan p, bool apply_scale, float scale, uint64_t chunk, int early) {
    __shared__ GroupScratch<kSplitThreads> s;
    __shared__ float part_max;
    __shared__ double part_sum;
    cg::cluster_group cluster = cg::this_cluster();
    const unsigned rank = cluster.block_rank();
    const uint64_t r = blockIdx.x / kSplitCluster;
    const Chunk ch = my_chunk(p.ne[0], chunk, rank);
    SoftmaxRow w;
    w.x = reinterpret_cast<const float*>(p.src.ptr) + split_row_base(p.src, r, p.ne[1], p.ne[2]);
    w.y = reinterpret_cast<float*>(p.dst.ptr) + split_row_base(p.dst, r, p.ne[1], p.ne[2]);
    w.xs = p.src.st[0];
    w.ys = p.dst.st[0];
    w.has_mask = apply_scale && p.has_aux;
    w.mbase = w.has_mask ? split_mask_base(p.aux, r, p.ne[1], p.ne[2]) : 0;
    const bool vec = p.vec && !w.has_mask;
    const float4* x4 = reinterpret_cast<const float4*>(w.x);
    float4* y4 = reinterpret_cast<float4*>(w.y);
    auto scale4 = [&](float4 q) {
        return apply_scale ? make_float4(__fmul_rn(q.x, scale), __fmul_rn(q.y, scale), __fmul_rn(q.z, scale),
                                         __fmul_rn(q.w, scale))
                           : q;
    };

    // pass 1: maximum of the fast values, NaN-propagating: a NaN anywhere,
    // or a maximum of +-inf, leaves the row's maximum non-finite
    float m = -INFINITY;
    if (vec) {
        auto load = [&](uint64_t v) { return __ldcg(x4 + v); };
        auto use = [&](uint64_t, float4 raw) {
            const float4 q = scale4(raw);
            m = max_nan(max_nan(m, q.x), max_nan(q.y, max_nan(q.z, q.w)));
        };
        const uint64_t vstart = early_batch<8>(early != 0, ch.col0 / 4, ch.col1 / 4, load, use);
        batched<8>(vstart, ch.col1 / 4, load, use);
    } else {
        pdl_enter();
        for (uint64_t c = ch.col0 + threadIdx.x; c < ch.col1; c += kSplitThreads)
            m = max_nan(m, value_at<false>(p, w, c, apply_scale, scale));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = max_nan(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & 31) == 0) s.f[threadIdx.x / 32] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        float cm = s.f[0];
        for (int k = 1; k < kSplitThreads / 32; ++k) cm = max_nan(cm, s.f[k]);
        part_max = cm;
    }
    cluster.sync();
    float gm = *cluster.map_shared_rank(&part_max, 0);
    for (int k = 1; k < kSplitCluster; ++k) gm = max_nan(gm, *cluster.map_shared_rank(&part_max, k));

    double acc = 0.0;
    float zmin = 0.0f;  // smallest v - max among this thread's values
    if (isfinite(gm)) {
        // pass 2: e = exp(v - max) into dst, f64 sum.  Vectors whose four
        // z = v - max are all >= kSoftmaxPlainDivFloor take the packed
        // exponential (softmax_exp2), the rest softmax_exp lane by lane; a
        // vector's four terms are added in binary32 (relative error <= 2^-23)
        // before the f64 sum.
        if (vec) {
            const float2 ngm = make_float2(-gm, -gm);  // z = q + (-max) is IEEE q - max
            batched<8>(ch.col0 / 4, ch.col1 / 4, [&](uint64_t v) { return __ldcg(x4 + v); },
                       [&](uint64_t v, float4 raw) {
                           const float4 q = scale4(raw);
                           const float2 zl = __fadd2_rn(lo2(q), ngm), zh = __fadd2_rn(hi2(q), ngm);
                           const float zm = fmin3(fminf(zl.x, zl.y), zh.x, zh.y);
                           float4 e;
                           if (zm >= kSoftmaxPlainDivFloor) {
                               e = cat2(softmax_exp2(zl), softmax_exp2(zh));
                           } else {
                               zmin = fminf(zmin, zm);
                               e = make_float4(softmax_exp(zl.x), softmax_exp(zl.y), softmax_exp(zh.x),
                                               softmax_exp(zh.y));
                           }
                           y4[v] = e;
                           const float2 pr = __fadd2_rn(lo2(e), hi2(e));
                           acc += (double)__fadd_rn(pr.x, pr.y);
                       });
        } else {
            for (uint64_t c = ch.col0 + threadIdx.x; c < ch.col1; c += kSplitThreads) {
                const float z = __fsub_rn(value_at<false>(p, w, c, apply_scale, scale), gm);
                zmin = fminf(zmin, z);
                const float e = softmax_exp(z);
                w.y[(int64_t)c * w.ys] = e;
                acc += (double)e;
            }
        }
    } else {
        // exact pass: the reference's NaN rules (first element pins a NaN max)
        const float v0 = value_at<true>(p, w, 0, apply_scale, scale);
        float em = bitsf(0x7fc00000u);
        __syncthreads();
        for (uint64_t c = ch.col0 + threadIdx.x; c < ch.col1; c += kSplitThreads)
            em = max_nn(em, value_at<true>(p, w, c, apply_scale, scale));
        em = group_max<kSplitThreads>(em, &s);
        if (threadIdx.x == 0) part_max = em;
        cluster.sync();
        gm = bitsf(0x7fc00000u);
        for (int k = 0; k < kSplitCluster; ++k) gm = max_nn(gm, *cluster.map_shared_rank(&part_max, k));
        if (is_nan(v0)) gm = v0;
        for (uint64_t c = ch.col0 + threadIdx.x; c < ch.col1; c += kSplitThreads) {
            const float e = lm_exp(f_sub(value_at<true>(p, w, c, apply_scale, scale), gm));
            w.y[(int64_t)c * w.ys] = e;
            acc += (double)e;
        }
    }
    acc = group_sum<kSplitThreads>(acc, &s);
    if (threadIdx.x == 0) part_sum = acc;
    cluster.sync();  // also orders every CTA's pass-2 stores before pass 3 reads its own
    double total = 0.0;
    for (int k = 0; k < kSplitCluster; ++k) total += *cluster.map_shared_rank(&part_sum, k);
    const float denom = __double2float_rn(total);
    // pass 3: divide in place (each thread rereads the values it wrote)
    if (isfinite(gm) && isfinite(denom)) {
        const float inv = __frcp_rn(denom);
        if (vec && zmin >= kSoftmaxPlainDivFloor) {
            const float2 d2 = make_float2(denom, denom), i2 = make_float2(inv, inv);
            batched<8>(ch.col0 / 4, ch.col1 / 4, [&](uint64_t v) { return y4[v]; },
                       [&](uint64_t v, float4 e) {
                           __stcs(y4 + v, cat2(markstein_div2(lo2(e), d2, i2), markstein_div2(hi2(e), d2, i2)));
                       });
        } else if (vec) {
            batched<8>(ch.col0 / 4, ch.col1 / 4, [&](uint64_t v) { return y4[v]; },
                       [&](uint64_t v, float4 e) {
                           __stcs(y4 + v, make_float4(softmax_div(e.x, denom, inv), softmax_div(e.y, denom, inv),
                                                      softmax_div(e.z, denom, inv), softmax_div(e.w, denom, inv)));
                       });
        } else {
            for (uint64_t c = ch.col0 + threadIdx.x; c < ch.col1; c += kSplitThreads) {
                float* o = w.y + (int64_t)c * w.ys;
                *o = softmax_div(*o, denom, inv);
            }
        }
    } else {
        for (uint64_t c = ch.col0 + threadIdx.x; c < ch.col1; c += kSplitThreads) {
            float* o = w.y + (int64_t)c * w.ys;
            *o = f_div(*o, denom);
        }
    }
    cluster.sync();  // peers' shared memory stays alive until every CTA has read it
}

uint64_t split_chunk(uint64_t ne0) {
    uint64_t c = (ne0 + kSplitCluster - 1) / kSplitCluster;
    return (c + 3) / 4 * 4;  // keeps every chunk's first column 16-byte aligned
}

}  // namespace

bool split_rows_wanted(const LaunchEnv& env, const RowPlan& p) {
    // few rows, each long enough to give eight CTAs real work
    return p.ne[0] >= 16384 && p.rows <= (uint64_t)env.sm_count && p.rows * kSplitCluster <= 0x7fffffffull &&
           !p.dst_ordinal;
}

cudaError_t launch_argmax_rows_split(const LaunchEnv& env, const RowPlan& p, int dst_dtype) {
    cudaError_t err;
    if (p.vec) {
        static_assert(kSplitCluster == kSplitRowChunks, "workspace slots per row");
        char* base = static_cast<char*>(env.workspace) + split_rows_workspace_offset(env.sm_count);
        auto* partials = reinterpret_cast<ChunkPartial*>(base);
        auto* tickets = reinterpret_cast<unsigned*>(base + (uint64_t)env.sm_count * kSplitRowChunks * 16);
        const int early = reads_clear(env, span_of(p.src, 4));
        err = launch_dependent(argmax_rows_flat, dim3((unsigned)(p.rows * kSplitCluster)), dim3(kSplitThreads), 0,
                               env.stream, p, dst_dtype, split_chunk(p.ne[0]), partials, tickets, early);
        if (err == cudaSuccess) stream_wrote(env.stream, span_of(p.dst, dst_dtype == (int)DType::I64 ? 8 : 4));
    } else {
        err = launch_dependent(argmax_rows_split, dim3((unsigned)(p.rows * kSplitCluster)), dim3(kSplitThreads), 0,
                               env.stream, p, dst_dtype, split_chunk(p.ne[0]));
    }
    ++*env.launches;
    return err != cudaSuccess ? err : cudaGetLastError();
}

cudaError_t launch_sum_rows_split(const LaunchEnv& env, const RowPlan& p) {
    const cudaError_t err = launch_dependent(sum_rows_split, dim3((unsigned)(p.rows * kSplitCluster)),
                                             dim3(kSplitThreads), 0, env.stream, p, split_chunk(p.ne[0]));
    ++*env.launches;
    return err != cudaSuccess ? err : cudaGetLastError();
}

cudaError_t launch_soft_max_split(const LaunchEnv& env, const RowPlan& p, bool apply_scale, float scale) {
    // early only for the vector pass without a mask (the kernel's `vec`)
    const int early = p.vec && !(apply_scale && p.has_aux) && reads_clear(env, span_of(p.src, 4));
    const cudaError_t err = launch_dependent(softmax_rows_split, dim3((unsigned)(p.rows * kSplitCluster)),
                                             dim3(kSplitThreads), 0, env.stream, p, apply_scale, scale,
                                             split_chunk(p.ne[0]), early);
    if (err == cudaSuccess) stream_wrote(env.stream, span_of(p.dst, 4));
    ++*env.launches;
    return err != cudaSuccess ? err : cudaGetLastError();
}

}  // namespace emel
