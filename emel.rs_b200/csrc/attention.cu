// Single-query attention (flash_attn.rs OpFlashAttnExt) on the device.
//
// The reference (flash_attn.rs:329-404) walks the key/value tokens of one
// head in order with a running maximum, a binary32 score sum and a
// binary16 accumulator row that is rounded after every token.  Rounding
// to binary16 at each step makes the accumulator a strictly sequential
// recurrence per (head, column): no reordering, splitting or tree
// combination reproduces its bits.  What is independent is
//   * the score of each token (a binary64 dot product of the binary16 query
//     with the key row, flash_attn.rs:424-441),
//   * the running maximum before each token (a prefix maximum), and from it
//     each token's rescale / value factors (one exp each),
//   * the recurrence of each accumulator column (it reads only its own
//     column of V and the per-token factors).
//
// So one CTA per head runs three warp roles over tiles of TILE tokens:
//   score warps (TILE threads, one token each) compute tile i's scores,
//     scan them for the running maximum, turn them into the per-token
//     factors (rs, vs, and both rounded to binary16), store them in a
//     double-buffered shared tile, and prefetch the K rows of the next
//     tile into L2;
//   the sum warp has the TMA engine copy tile i's V rows into a
//     double-buffered shared tile (an mbarrier counts the bytes), and its
//     lane 0 carries the binary32 score sum over tile i - 1;
//   accumulator warps (one thread per DPT columns) consume tile i - 1:
//     per token and column one rescale when the maximum moved and one
//     fused a + v * vs (the product of two binary16 values is exact in
//     binary32, so the fused form rounds exactly as the reference's
//     separate multiply and add), each rounded to binary16, V read from
//     shared memory.
// A block barrier separates the iterations.  Shared memory holds two V
// tiles, so TILE shrinks as head_dim grows (256 tokens up to 192 columns,
// 32 tokens at 1536); beyond that V is read from global memory.  The
// accumulator chain (one FMA and one binary16 round trip per token) bounds
// the kernel: its time is tokens x the chain latency, whatever the number
// of heads.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "common.cuh"
#include "launch.hpp"
#include "pdl.cuh"
#include "tma.cuh"

namespace emel {
namespace {


// flash_attn.rs:528-557 as integer steps: binary32 -> binary16 bits.
// Normal results round to nearest even, results below 2^-24 become a
// signed zero, the subnormal range rounds half up, NaN is 0x7E00 | sign.
__device__ __noinline__ uint16_t fa_f16_bits(float value) {
    const uint32_t w = __float_as_uint(value);
    const uint32_t sign = (w >> 16) & 0x8000u;
    const uint32_t e = (w >> 23) & 0xffu, frac = w & 0x7fffffu;
    if (e == 0xffu) return (uint16_t)(sign | (frac == 0 ? 0x7c00u : 0x7e00u));
    if (e > 142u) return (uint16_t)(sign | 0x7c00u);
    if (e < 103u) return (uint16_t)sign;
    if (e < 113u) {
        const uint32_t shift = 113u - e, m = 0x800000u | frac;
        return (uint16_t)(sign | ((m + (1u << (shift + 12u))) >> (shift + 13u)));
    }
    uint32_t h = sign | ((e - 112u) << 10) | (frac >> 13);
    const uint32_t rem = frac & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1u;
    return (uint16_t)h;
}

// quant.rs:287-302 widening of binary16 bits: exact for numbers, a NaN
// comes back quiet with its sign.
__device__ __forceinline__ float fa_widen(uint16_t h) {
    if ((h & 0x7fffu) > 0x7c00u) return __uint_as_float(((uint32_t)(h & 0x8000u) << 16) | 0x7fc00000u);
    return __half2float(__ushort_as_half(h));
}

__device__ __noinline__ float fa_round16_slow(float x) { return fa_widen(fa_f16_bits(x)); }

// round_fp16_scalar (flash_attn.rs:420-422).  From the smallest normal
// binary16 up, the rule is IEEE round-to-nearest-even (overflow included),
// which the hardware conversion does; zero, the subnormal range and NaN
// take the integer restatement.
__device__ __forceinline__ float fa_round16(float x) {
    if (fabsf(x) >= 6.103515625e-05f) return __half2float(__float2half_rn(x));
    return fa_round16_slow(x);
}

// f16_to_f32 (f16_matmul.rs:508-532): exact widening of key / value bits.
__device__ __forceinline__ float fa_kv(uint16_t h) { return __half2float(__ushort_as_half(h)); }

__device__ __forceinline__ float fa_max(float a, float b) { return fmaxf(a, b); }  // a NaN operand is skipped

__device__ __forceinline__ void fa_prefetch_l2(const void* p) {
    asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// V staging modes: kFaVBulk, the TMA engine copies each tile's V rows into
// shared memory (unit-stride rows, 16-byte aligned); kFaVCopy, the score
// warps copy their own tokens' rows element by element (any strides);
// kFaVGlobal (head_dim beyond the shared-memory budget), the accumulator
// threads read V from global memory through a register ring.
enum FaVMode : int { kFaVBulk = 0, kFaVCopy = 1, kFaVGlobal = 2 };

constexpr int fa_threads(int dpt, int tile) { return (dpt == 8 ? 512 : 256) + tile + 32; }

template <int DPT, int TILE, int VMODE>
__global__ void __launch_bounds__(fa_threads(DPT, TILE), 1) fa_decode(FlashAttnPlan p) {
    constexpr int kScoreWarps = TILE / 32;
    constexpr int RING = 32 / DPT;  // kFaVGlobal only
    extern __shared__ __align__(16) unsigned char fa_smem[];
    uint64_t* bars = reinterpret_cast<uint64_t*>(fa_smem);               // [2] V tile arrivals (kFaVBulk)
    float4* tiles = reinterpret_cast<float4*>(fa_smem + 16);             // [2][TILE]: rs, vs, rs16, vs16
    float* wtot = reinterpret_cast<float*>(tiles + 2 * TILE);            // [kScoreWarps] warp maxima
    float* ssum = wtot + 8;                                              // final score sum
    int* failed = reinterpret_cast<int*>(wtot + 9);                      // a bounded wait expired
    uint32_t* flags = reinterpret_cast<uint32_t*>(wtot + 16);            // [2][8] tokens where the maximum moved
    double* qd = reinterpret_cast<double*>(wtot + 32);                   // [d] query through binary16
    uint16_t* vtile = reinterpret_cast<uint16_t*>(qd + p.d);             // [2][TILE][d] staged V rows
    pdl_enter();

    const uint64_t head = blockIdx.x;
    const uint64_t kvh = head / p.rep;
    const int tid = threadIdx.x;
    const int na = (int)blockDim.x - TILE - 32;  // accumulator threads
    const uint64_t d = p.d, T = p.tokens;
    const char* kbase = p.k + kvh * p.ks[2];
    const char* vbase = p.v + kvh * p.vs[2];

    // flash_attn.rs:346-350: the query row through binary16
    for (uint64_t c = tid; c < d; c += blockDim.x) qd[c] = (double)fa_widen(fa_f16_bits(p.q[head * d + c]));
    if (tid == 0) {
        failed[0] = 0;
        if constexpr (VMODE == kFaVBulk) {
            mbar_init(&bars[0], 1);
            mbar_init(&bars[1], 1);
            mbar_init_fence();
        }
    }
    __syncthreads();

    const int warp = tid >> 5, lane = tid & 31;
    const bool is_acc = tid < na;
    const bool is_score = !is_acc && tid < na + TILE;
    const bool is_sum = !is_acc && !is_score;
    const int sj = tid - na;  // score thread index
    const uint64_t ntiles = (T + TILE - 1) / TILE;

    float acc[DPT];
    uint64_t col[DPT];
#pragma unroll
    for (int k = 0; k < DPT; ++k) {
        acc[k] = 0.0f;
        const uint64_t c = (uint64_t)tid + (uint64_t)k * na;
        col[k] = c < d ? c : 0;
    }
    uint16_t ring[VMODE == kFaVGlobal ? RING : 1][DPT];
    if constexpr (VMODE == kFaVGlobal) {
        if (is_acc) {
#pragma unroll
            for (int j = 0; j < RING; ++j)
#pragma unroll
                for (int k = 0; k < DPT; ++k)
                    ring[j][k] = (uint64_t)j < T ? *reinterpret_cast<const uint16_t*>(vbase + col[k] * p.vs[0] +
                                                                                     (uint64_t)j * p.vs[1])
                                                 : 0;
        }
    }
    float carry = -INFINITY;  // running maximum before the tile (score threads)
    float sum = 0.0f;         // score sum (sum lane)

    for (uint64_t it = 0; it <= ntiles; ++it) {
        if (is_sum && it < ntiles && VMODE == kFaVBulk) {
            // V rows of tile `it` into buffer it & 1, consumed next iteration
            const uint64_t t0 = it * TILE;
            const uint64_t n = T - t0 < (uint64_t)TILE ? T - t0 : (uint64_t)TILE;
            uint16_t* dst = vtile + (it & 1) * (uint64_t)TILE * d;
            const uint32_t row_bytes = (uint32_t)(d * 2);
            if (lane == 0) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                mbar_expect_tx(&bars[it & 1], (uint32_t)(n * row_bytes));
            }
            __syncwarp();
            if (p.v_dense) {
                // one contiguous range, copied in pieces of at most 16 KB
                const uint32_t bytes = (uint32_t)(n * row_bytes);
                const char* src = vbase + t0 * p.vs[1];
                for (uint32_t off = (uint32_t)lane * 16384u; off < bytes; off += 32u * 16384u)
                    bulk_load(reinterpret_cast<char*>(dst) + off, src + off, bytes - off < 16384u ? bytes - off : 16384u,
                              &bars[it & 1]);
            } else {
                for (uint64_t j = lane; j < n; j += 32)
                    bulk_load(dst + j * d, vbase + (t0 + j) * p.vs[1], row_bytes, &bars[it & 1]);
            }
        }
        if (is_score && it < ntiles) {
            const uint64_t t = it * TILE + sj;
            float s = __uint_as_float(0x7fc00000u);  // out of range: skipped by the scan
            if (t < T) {
                const char* krow = kbase + t * p.ks[1];
                double dot = 0.0;
                if (p.k_rows) {
                    const auto pair = [&](uint32_t word, uint64_t c) {
                        dot = __dadd_rn(dot, __dmul_rn(qd[c], (double)fa_kv((uint16_t)(word & 0xffffu))));
                        dot = __dadd_rn(dot, __dmul_rn(qd[c + 1], (double)fa_kv((uint16_t)(word >> 16))));
                    };
                    uint64_t c0 = 0;
                    for (; c0 + 64 <= d; c0 += 64) {  // eight 16-byte loads in flight
                        const uint4* r4 = reinterpret_cast<const uint4*>(krow + c0 * 2);
                        uint4 w[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e) w[e] = r4[e];
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            const uint64_t c = c0 + 8 * e;
                            pair(w[e].x, c), pair(w[e].y, c + 2), pair(w[e].z, c + 4), pair(w[e].w, c + 6);
                        }
                    }
                    for (; c0 < d; c0 += 8) {
                        const uint4 w = *reinterpret_cast<const uint4*>(krow + c0 * 2);
                        pair(w.x, c0), pair(w.y, c0 + 2), pair(w.z, c0 + 4), pair(w.w, c0 + 6);
                    }
                } else {
                    for (uint64_t c = 0; c < d; ++c)
                        dot = __dadd_rn(dot, __dmul_rn(qd[c], (double)fa_kv(*reinterpret_cast<const uint16_t*>(
                                                                    krow + c * p.ks[0]))));
                }
                s = __fmul_rn(__double2float_rn(dot), p.scale);
                if (p.k_rows && t + TILE < T) {
                    const char* knext = kbase + (t + TILE) * p.ks[1];
                    for (uint64_t b = 0; b < d * 2; b += 128) fa_prefetch_l2(knext + b);
                }
                if constexpr (VMODE == kFaVCopy) {
                    uint16_t* dst = vtile + (it & 1) * (uint64_t)TILE * d + (uint64_t)sj * d;
                    const char* vrow = vbase + t * p.vs[1];
                    for (uint64_t c = 0; c < d; ++c) dst[c] = *reinterpret_cast<const uint16_t*>(vrow + c * p.vs[0]);
                }
            }
            // running maximum before each token: strict '>' updates never
            // take a NaN, so it is the prefix maximum over the numbers
            float m = s;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const float o = __shfl_up_sync(0xffffffffu, m, off);
                if (lane >= off) m = fa_max(m, o);
            }
            const int sw = warp - na / 32;
            if (lane == 31) wtot[sw] = m;
            asm volatile("bar.sync 1, %0;" ::"r"(TILE));
            float before = carry, total = carry;
#pragma unroll
            for (int i = 0; i < kScoreWarps; ++i) {
                if (i < sw) before = fa_max(before, wtot[i]);
                total = fa_max(total, wtot[i]);
            }
            const float prev = __shfl_up_sync(0xffffffffu, m, 1);
            const float mb = lane == 0 ? before : fa_max(before, prev);
            carry = total;
            float rs = 1.0f, vs = 1.0f;
            if (t < T) {
                // flash_attn.rs:364-375
                if (s > mb)
                    rs = lm_exp_cr(__fsub_rn(mb, s));
                else
                    vs = lm_exp_cr(__fsub_rn(s, mb));
                tiles[(it & 1) * TILE + sj] = make_float4(rs, vs, fa_round16(rs), fa_round16(vs));
            }
            // tokens whose binary16 rescale factor is not 1 (a rescale by 1 leaves
            // a binary16 accumulator unchanged)
            const uint32_t moved = __ballot_sync(0xffffffffu, t < T && fa_round16(rs) != 1.0f);
            if (lane == 0) flags[(it & 1) * 8 + sw] = moved;
        } else if (is_acc && it > 0) {
            const uint64_t t0 = (it - 1) * TILE;
            const float4* sc = tiles + ((it - 1) & 1) * TILE;
            const int n = T - t0 < (uint64_t)TILE ? (int)(T - t0) : TILE;
            if constexpr (VMODE == kFaVGlobal) {
                for (int base = 0; base < TILE; base += RING) {
#pragma unroll
                    for (int j = 0; j < RING; ++j) {
                        const uint64_t t = t0 + base + j;
                        if (t < T) {
                            const float4 f = sc[base + j];
#pragma unroll
                            for (int k = 0; k < DPT; ++k) {
                                float a = acc[k];
                                if (f.z != 1.0f) a = fa_round16(__fmul_rn(a, f.z));
                                acc[k] = fa_round16(__fmaf_rn(fa_kv(ring[j][k]), f.w, a));
                            }
                            const uint64_t tn = t + RING;
#pragma unroll
                            for (int k = 0; k < DPT; ++k)
                                if (tn < T)
                                    ring[j][k] = *reinterpret_cast<const uint16_t*>(vbase + col[k] * p.vs[0] +
                                                                                    tn * p.vs[1]);
                        }
                    }
                }
            } else {
                if constexpr (VMODE == kFaVBulk) {
                    if (!failed[0] && !mbar_wait(&bars[(it - 1) & 1], (uint32_t)(((it - 1) >> 1) & 1))) {
                        failed[0] = 1;
                        atomicExch(p.fault, 1u);
                    }
                }
                const uint16_t* vt = vtile + ((it - 1) & 1) * (uint64_t)TILE * d;
                // one binary16 recurrence step per token and column
                // (scale_f16_buffer_scalar where the maximum moved, then
                // axpy_f16_buffer_scalar).  The fast pass rounds with the
                // hardware conversion and only records whether a value fell
                // in (0, 2^-14), where the reference's rounding differs;
                // a thread that saw one replays its tile with the exact rule.
                float a0[DPT];
                uint32_t off[DPT];
#pragma unroll
                for (int k = 0; k < DPT; ++k) {
                    a0[k] = acc[k];
                    off[k] = (uint32_t)col[k];
                }
                const uint32_t d32 = (uint32_t)d;
                bool suspect = false;
                // The hardware conversion rounds to nearest even; the reference
                // (flash_attn.rs:528-557) differs only below 2^-14, where it
                // flushes (2^-25, 2^-24) to zero and rounds exact ties up.  A
                // tie is |x - r| = 2^-25 (the difference is exact there); a
                // flushed value is |x| < 2^-24 rounded to nonzero.  Only those
                // inputs mark the tile for an exact replay; the test uses
                // compares only, so it adds no conversion to the chain's pipe.
                const auto fast = [&](float x) {
                    const float r = __half2float(__float2half_rn(x));
                    const float ax = fabsf(x);
                    suspect |= ax < 6.103515625e-05f && (fabsf(__fsub_rn(x, r)) == 2.98023223876953125e-08f ||
                                                          (ax < 5.9604644775390625e-08f && r != 0.0f));
                    return r;
                };
                const uint32_t* fl = flags + ((it - 1) & 1) * 8;
                const auto step = [&](int j, bool rescale) {
                    const float4 f = sc[j];
                    float v[DPT];
#pragma unroll
                    for (int k = 0; k < DPT; ++k) v[k] = fa_kv(vt[(uint32_t)j * d32 + off[k]]);
                    if (rescale && f.z != 1.0f) {
#pragma unroll
                        for (int k = 0; k < DPT; ++k) acc[k] = fast(__fmul_rn(acc[k], f.z));
                    }
#pragma unroll
                    for (int k = 0; k < DPT; ++k) acc[k] = fast(__fmaf_rn(v[k], f.w, acc[k]));
                };
                int j = 0;
                for (; j + 8 <= n; j += 8) {
                    // one uniform test per 8 tokens: most groups never move the maximum
                    if (((fl[j >> 5] >> (j & 31)) & 0xffu) == 0u) {
#pragma unroll
                        for (int u = 0; u < 8; ++u) step(j + u, false);
                    } else {
#pragma unroll
                        for (int u = 0; u < 8; ++u) step(j + u, true);
                    }
                }
                for (; j < n; ++j) step(j, true);
                if (suspect) {
#pragma unroll
                    for (int k = 0; k < DPT; ++k) acc[k] = a0[k];
                    for (int jj = 0; jj < n; ++jj) {
                        const float4 f = sc[jj];
#pragma unroll
                        for (int k = 0; k < DPT; ++k) {
                            float a = acc[k];
                            if (f.z != 1.0f) a = fa_round16(__fmul_rn(a, f.z));
                            acc[k] = fa_round16(__fmaf_rn(fa_kv(vt[(uint32_t)jj * d32 + off[k]]), f.w, a));
                        }
                    }
                }
            }
        } else if (is_sum && lane == 0 && it > 0) {
            const uint64_t t0 = (it - 1) * TILE;
            const float4* sc = tiles + ((it - 1) & 1) * TILE;
            const int n = T - t0 < (uint64_t)TILE ? (int)(T - t0) : TILE;
            int j = 0;
            for (; j + 8 <= n; j += 8) {
                float2 f[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) f[u] = make_float2(sc[j + u].x, sc[j + u].y);
#pragma unroll
                for (int u = 0; u < 8; ++u) sum = __fadd_rn(__fmul_rn(sum, f[u].x), f[u].y);
            }
            for (; j < n; ++j) sum = __fadd_rn(__fmul_rn(sum, sc[j].x), sc[j].y);
        }
        __syncthreads();
    }
    if (is_sum && lane == 0) ssum[0] = sum;
    __syncthreads();
    if (is_acc) {
        // finalize_attention_output (flash_attn.rs:382-404)
        const float total = ssum[0];
        const float inv = total == 0.0f ? 0.0f : __fdiv_rn(1.0f, total);
#pragma unroll
        for (int k = 0; k < DPT; ++k) {
            const uint64_t c = (uint64_t)tid + (uint64_t)k * na;
            if (c < d) p.dst[head * d + c] = total == 0.0f ? 0.0f : __fmul_rn(acc[k], inv);
        }
    }
}

template <int DPT, int TILE, int VMODE>
cudaError_t launch_fa(const LaunchEnv& env, const FlashAttnPlan& p) {
    const int na = (int)(((p.d + DPT - 1) / DPT + 31) / 32 * 32);
    const int threads = na + TILE + 32;
    const size_t smem = 16 + 2 * TILE * sizeof(float4) + 32 * sizeof(float) + p.d * sizeof(double) +
                        (VMODE == kFaVGlobal ? 0 : 2 * (size_t)TILE * p.d * 2);
    if (smem > 48 * 1024) {
        const cudaError_t err =
            cudaFuncSetAttribute(fa_decode<DPT, TILE, VMODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (err != cudaSuccess) return err;
    }
    return launch_dependent(fa_decode<DPT, TILE, VMODE>, dim3((unsigned)p.heads), dim3(threads), smem, env.stream,
                            p);
}

// head_dim -> (columns per thread, tokens per tile) such that two staged V
// tiles stay within about 192 KB of shared memory.
template <int VMODE>
cudaError_t launch_fa_mode(const LaunchEnv& env, const FlashAttnPlan& p) {
    if (p.d <= 192) return launch_fa<1, 256, VMODE>(env, p);
    if (p.d <= 256) return launch_fa<1, 128, VMODE>(env, p);
    if (p.d <= 384) return launch_fa<2, 128, VMODE>(env, p);
    if (p.d <= 512) return launch_fa<2, 64, VMODE>(env, p);
    if (p.d <= 768) return launch_fa<4, 64, VMODE>(env, p);
    if (p.d <= 1024) return launch_fa<4, 32, VMODE>(env, p);
    return launch_fa<8, 32, VMODE>(env, p);
}

}  // namespace

cudaError_t launch_flash_attn(const LaunchEnv& env, const FlashAttnPlan& p) {
    cudaError_t err;
    if (p.d > 1536)
        err = launch_fa<8, 32, kFaVGlobal>(env, p);
    else if (p.v_bulk)
        err = launch_fa_mode<kFaVBulk>(env, p);
    else
        err = launch_fa_mode<kFaVCopy>(env, p);
    ++*env.launches;
    return err != cudaSuccess ? err : cudaGetLastError();
}

}  // namespace emel
