// Rotary position embedding (rope.rs): norm (pairs 2k, 2k + 1), neox
// (pairs k, k + n_dims / 2) and timestep (real / imaginary halves).
//
// A CTA owns one (position, batch) slice: all ne1 rows of that position.
// The reference recomputes cos / sin for every row; they depend only on the
// position and the pair, so the CTA computes them once into shared memory:
// the theta chain theta_k = theta_{k-1} * theta_scale (a sequential binary32
// product, kept sequential so every theta_k is the reference's) by one
// thread, then cos / sin of every pair by all threads; then every thread
// rotates pairs of every row (coalesced: consecutive threads take
// consecutive pairs).  Pairs are handled in chunks of kRopeChunk so any
// n_dims fits the shared-memory table.
//
// Numerics (rope.rs:523-646): rotated = theta * freq_scale, c = cos * attn,
// s = sin * attn, a' = fma(a, c, -(b * s)), b' = fma(a, s, b * c); timestep:
// frequency = exp(-log(base) * k / half), argument = position * frequency *
// freq_scale, a' = a c - b s, b' = a s + b c.  theta_scale = powf(base,
// -2 / n_dims) and -logf(base) come from the host (the same libm calls the
// reference makes).  cos / sin / exp are binary64 evaluations rounded once
// (cos and sin from one sincos).  Row and pair counters are 32-bit: the
// host routes only slices of fewer than 2^32 (row, pair) items here.
#include "common.cuh"
#include "launch.hpp"
#include "pdl.cuh"

namespace emel {

namespace {

constexpr int kRopeThreads = 256;
constexpr uint32_t kRopeChunk = 2048;  // pairs per shared-memory table

__device__ __forceinline__ float* at(char* base, const int64_t st[4], uint64_t c, uint64_t r, uint64_t p, uint64_t b) {
    return reinterpret_cast<float*>(base + (int64_t)c * st[0] + (int64_t)r * st[1] + (int64_t)p * st[2] +
                                    (int64_t)b * st[3]);
}

// fma(a, c, -(b * s)) and fma(a, s, b * c); a NaN result is rebuilt with the
// x86 rules, operands in source order.
__device__ __forceinline__ void rotate(float a, float b, float c, float s, float& ra, float& rb) {
    ra = __fmaf_rn(a, c, -__fmul_rn(b, s));
    rb = __fmaf_rn(a, s, __fmul_rn(b, c));
    if (is_nan(ra)) ra = x86_nan3(ra, a, c, f_neg(f_mul(b, s)));
    if (is_nan(rb)) rb = x86_nan3(rb, a, s, f_mul(b, c));
}

// Positions per CTA unit: enough that the table build keeps every thread
// busy (P * half >= kRopeThreads) when the pairs are few.
__host__ __device__ __forceinline__ uint32_t rope_group(uint64_t half) {
    return half >= kRopeThreads ? 1u : (uint32_t)(kRopeThreads / half);
}

template <int MODE>
__global__ void __launch_bounds__(kRopeThreads) rope_kernel(RopePlan p) {
    extern __shared__ float table[];  // cos[kRopeChunk], sin[kRopeChunk]
    pdl_enter();
    const uint64_t half = MODE == kRopeTimestep ? p.cols / 2 : p.n_dims / 2;
    const uint32_t group = rope_group(half);  // positions per unit (1 when half > kRopeChunk / group)
    const uint64_t pgroups = (p.npos + group - 1) / group;
    const uint64_t units = pgroups * p.batches;
    char* src = const_cast<char*>(p.src);
    for (uint64_t u = blockIdx.x; u < units; u += gridDim.x) {
        const uint64_t b = u / pgroups, p0 = (u % pgroups) * group;
        const uint32_t np = (uint32_t)(p.npos - p0 < group ? p.npos - p0 : group);
        float theta = 0.0f;  // with group == 1, thread 0 carries the chain across chunks
        if (threadIdx.x < np)
            theta = __int2float_rn(*reinterpret_cast<const int32_t*>(p.positions + (p0 + threadIdx.x) * p.pos_stride));
        for (uint64_t k0 = 0; k0 < half; k0 += kRopeChunk) {
            const uint32_t nk = (uint32_t)(half - k0 < kRopeChunk ? half - k0 : kRopeChunk);
            const uint32_t entries = np * nk;  // table entry e = j * nk + k for position p0 + j
            __syncthreads();  // the previous chunk's table readers are done
            if constexpr (MODE != kRopeTimestep) {
                if (threadIdx.x < np) {
                    // theta is finite and theta_scale finite positive: no NaN on this chain
                    for (uint32_t k = 0; k < nk; ++k) {
                        table[threadIdx.x * nk + k] = theta;
                        theta = __fmul_rn(theta, p.theta_scale);
                    }
                }
                __syncthreads();
            }
            for (uint32_t e = threadIdx.x; e < entries; e += kRopeThreads) {
                float angle;
                if constexpr (MODE == kRopeTimestep) {
                    const uint32_t j = e / nk, k = e - j * nk;
                    const float position =
                        __int2float_rn(*reinterpret_cast<const int32_t*>(p.positions + (p0 + j) * p.pos_stride));
                    const float frequency = lm_exp_cr(f_div(f_mul(p.neg_log_period, (float)(k0 + k)), (float)half));
                    angle = f_mul(f_mul(position, frequency), p.freq_scale);
                } else {
                    angle = f_mul(table[e], p.freq_scale);
                }
                // cos and sin of the same binary64 argument, each rounded once
                double sd, cd;
                sincos((double)angle, &sd, &cd);
                table[e] = f_mul(x86_nan1((float)cd, angle), p.attn_factor);
                table[kRopeChunk + e] = f_mul(x86_nan1((float)sd, angle), p.attn_factor);
            }
            __syncthreads();
            if constexpr (MODE != kRopeTimestep) {
                if (p.vec) {
                    // dense 16-byte rows: norm, four consecutive elements = two
                    // pairs; neox, pairs k..k+3 as one vector at k and one at k + half
                    constexpr uint32_t kPairsPerItem = MODE == kRopeNorm ? 2 : 4;
                    constexpr int U = 4;  // items in flight per thread
                    const uint32_t nq = nk / kPairsPerItem;
                    const uint32_t per_pos = (uint32_t)p.rows * nq;
                    const uint32_t work = np * per_pos;
                    for (uint32_t w0 = threadIdx.x; w0 < work; w0 += U * kRopeThreads) {
                        float4 va[U], vb[U];
                        float4* da[U];
                        float4* db[U];
                        uint32_t kq[U];
#pragma unroll
                        for (int u = 0; u < U; ++u) {
                            const uint32_t w = w0 + u * kRopeThreads;
                            if (w >= work) break;
                            const uint32_t j = w / per_pos, rem = w - j * per_pos;
                            const uint32_t r = rem / nq, q = rem - r * nq;
                            const uint64_t pi = p0 + j, kk = k0 + (uint64_t)q * kPairsPerItem;
                            kq[u] = j * nk + q * kPairsPerItem;
                            const uint64_t ea = MODE == kRopeNorm ? 2 * kk : kk;
                            va[u] = __ldcs(reinterpret_cast<const float4*>(at(src, p.src_st, ea, r, pi, b)));
                            da[u] = reinterpret_cast<float4*>(at(p.dst, p.dst_st, ea, r, pi, b));
                            if constexpr (MODE == kRopeNeox) {
                                vb[u] = __ldcs(reinterpret_cast<const float4*>(at(src, p.src_st, kk + half, r, pi, b)));
                                db[u] = reinterpret_cast<float4*>(at(p.dst, p.dst_st, kk + half, r, pi, b));
                            }
                        }
#pragma unroll
                        for (int u = 0; u < U; ++u) {
                            if (w0 + u * kRopeThreads >= work) break;
                            const uint32_t e = kq[u];
                            if constexpr (MODE == kRopeNorm) {
                                float4 o;
                                rotate(va[u].x, va[u].y, table[e], table[kRopeChunk + e], o.x, o.y);
                                rotate(va[u].z, va[u].w, table[e + 1], table[kRopeChunk + e + 1], o.z, o.w);
                                __stcs(da[u], o);
                            } else {
                                float4 oa, ob;
                                rotate(va[u].x, vb[u].x, table[e], table[kRopeChunk + e], oa.x, ob.x);
                                rotate(va[u].y, vb[u].y, table[e + 1], table[kRopeChunk + e + 1], oa.y, ob.y);
                                rotate(va[u].z, vb[u].z, table[e + 2], table[kRopeChunk + e + 2], oa.z, ob.z);
                                rotate(va[u].w, vb[u].w, table[e + 3], table[kRopeChunk + e + 3], oa.w, ob.w);
                                __stcs(da[u], oa);
                                __stcs(db[u], ob);
                            }
                        }
                    }
                    continue;
                }
            }
            // items (position j, row r, pair k), pair fastest
            const uint32_t per_pos = (uint32_t)p.rows * nk;
            const uint32_t work = np * per_pos;
            for (uint32_t w = threadIdx.x; w < work; w += kRopeThreads) {
                const uint32_t j = w / per_pos, rem = w - j * per_pos;
                const uint32_t r = rem / nk, k = rem - r * nk;
                const uint64_t kk = k0 + k, pi = p0 + j;
                const float c = table[j * nk + k], s = table[kRopeChunk + j * nk + k];
                uint64_t ia, ib, oa, ob;
                if constexpr (MODE == kRopeNorm) {
                    ia = oa = 2 * kk;
                    ib = ob = 2 * kk + 1;
                } else if constexpr (MODE == kRopeNeox) {
                    ia = oa = kk;
                    ib = ob = kk + half;
                } else {
                    ia = 2 * kk;
                    ib = 2 * kk + 1;
                    oa = kk;
                    ob = half + kk;
                }
                const float a = *at(src, p.src_st, ia, r, pi, b), bv = *at(src, p.src_st, ib, r, pi, b);
                float ra, rb;
                if constexpr (MODE == kRopeTimestep) {
                    // separate products, then one subtraction / addition
                    ra = f_sub(f_mul(a, c), f_mul(bv, s));
                    rb = f_add(f_mul(a, s), f_mul(bv, c));
                } else {
                    rotate(a, bv, c, s, ra, rb);
                }
                *at(p.dst, p.dst_st, oa, r, pi, b) = ra;
                *at(p.dst, p.dst_st, ob, r, pi, b) = rb;
            }
        }
        if constexpr (MODE != kRopeTimestep) {
            // columns n_dims .. cols - 1 are copied
            const uint32_t tail = (uint32_t)(p.cols - p.n_dims);
            const uint32_t per_pos = (uint32_t)p.rows * tail;
            for (uint32_t w = threadIdx.x; w < np * per_pos; w += kRopeThreads) {
                const uint32_t j = w / per_pos, rem = w - j * per_pos;
                const uint32_t r = rem / tail;
                const uint64_t c = p.n_dims + (rem - r * tail);
                *at(p.dst, p.dst_st, c, r, p0 + j, b) = *at(src, p.src_st, c, r, p0 + j, b);
            }
        }
    }
}

}  // namespace

cudaError_t launch_rope(const LaunchEnv& env, const RopePlan& p) {
    const uint64_t half = p.mode == kRopeTimestep ? p.cols / 2 : p.n_dims / 2;
    const uint64_t group = rope_group(half);
    const uint64_t units = (p.npos + group - 1) / group * p.batches;
    // eight CTAs per SM whatever the residency: the finer grid-stride split
    // balances the positions better than one exact wave
    const uint64_t cap = (uint64_t)env.sm_count * 8;
    const dim3 grid((unsigned)(units < cap ? units : cap));
    const size_t smem = 2 * kRopeChunk * sizeof(float);
    cudaError_t err;
    switch (p.mode) {
    case kRopeNorm: err = launch_dependent(rope_kernel<kRopeNorm>, grid, dim3(kRopeThreads), smem, env.stream, p); break;
    case kRopeNeox: err = launch_dependent(rope_kernel<kRopeNeox>, grid, dim3(kRopeThreads), smem, env.stream, p); break;
    default: err = launch_dependent(rope_kernel<kRopeTimestep>, grid, dim3(kRopeThreads), smem, env.stream, p); break;
    }
    ++*env.launches;
    return err != cudaSuccess ? err : cudaGetLastError();
}

}  // namespace emel
