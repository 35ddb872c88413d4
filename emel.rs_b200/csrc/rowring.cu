// Row operators on a shared-memory ring fed by the TMA bulk-copy engine:
// norm, rms_norm, rms_norm * weight and soft_max (with scale and mask).
//
// Each of these needs every element of a row more than once (a statistic,
// then the output), so the row must stay on chip between the passes.  A
// persistent CTA owns the rows blockIdx.x, blockIdx.x + gridDim.x, ... and
// keeps S of them in flight in a ring of shared-memory stages:
//
//   * one thread issues `cp.async.bulk` copies (global -> shared, completion
//     counted in bytes on the stage's mbarrier) S rows ahead, so HBM sees
//     S row reads per CTA in flight while the CTA computes;
//   * all threads wait for the stage's phase (bounded by the global timer),
//     then run the passes over the staged row from shared memory (16-byte
//     reads, conflict-free), with f64 block reductions between passes;
//   * results go straight from registers to global memory (16-byte
//     streaming stores when the destination rows allow it);
//   * after a barrier the stage is refilled with the row S ahead.
//
// The soft_max_ext mask row, when it is contiguous and 16-byte aligned, is
// copied into the same stage by a second bulk copy on the same mbarrier; the
// rms_norm weight row is loaded into shared memory once per CTA.
//
// Arithmetic is the resident-row kernels' (rows.cu), term for term; only the
// grouping of the f64 partial sums differs.
//
// A wait that does not complete within two seconds sets the context's fault
// word (read back by emel_cuda_stream_synchronize as EMEL_CUDA_TIMEOUT);
// the CTA then waits, again bounded, for the copies it still has in flight
// and returns.
#include "common.cuh"
#include "launch.hpp"
#include "rowreduce.cuh"
#include "pdl.cuh"
#include "tma.cuh"

namespace emel {

namespace {

constexpr int kRingStagesMax = 4;
constexpr int kRingThreads = 256;
constexpr uint32_t kRingSmemPerSm = 220 * 1024;
constexpr uint32_t kStageAlign = 128;

// 4 / 5: the generic envelope's norm / rms_norm numerics (generic.rs:1992-2050).
enum RingOp { kRingNorm = 0, kRingRms = 1, kRingRmsMul = 2, kRingSoftMax = 3, kRingNormGeneric = 4, kRingRmsGeneric = 5 };

// aux_mode
enum { kAuxNone = 0, kAuxWeight = 1, kAuxMaskStaged = 2, kAuxMaskLoads = 3 };

struct RingArgs {
    const char* src;
    char* dst;
    const char* aux;
    uint32_t* fault;
    uint32_t ne0;  // multiple of 4
    uint32_t rows;
    uint32_t ne1, ne2;
    FastDiv d1, d2;
    int64_t src_st[4];  // element strides; src_st[0] == 1
    int64_t dst_st[4];
    int64_t aux_st[4];
    uint32_t aux_ne2, aux_ne3;
    FastDiv a2, a3;
    int aux_mode;
    int aux_f16;
    int dst_vec;
    int apply_scale;
    uint32_t stage_bytes;
    uint32_t mask_offset;
    uint32_t weight_bytes;
    int stages;
    float param;  // eps (norms) or scale (soft_max)
    int early;    // inputs clear of the previous kernel's writes: first copies before the wait
};

__device__ __forceinline__ void row_coords(uint32_t r, const RingArgs& a, uint32_t& i1, uint32_t& i2, uint32_t& i3) {
    const uint32_t q = fdiv(r, a.d1);
    i1 = r - q * a.ne1;
    i3 = fdiv(q, a.d2);
    i2 = q - i3 * a.ne2;
}

__device__ __forceinline__ int64_t row_offset(uint32_t r, const RingArgs& a, const int64_t* st) {
    uint32_t i1, i2, i3;
    row_coords(r, a, i1, i2, i3);
    return (int64_t)i1 * st[1] + (int64_t)i2 * st[2] + (int64_t)i3 * st[3];
}

// Mask row (i1, i2 % m2, i3 % m3) of soft_max_ext (reductions.rs:597-606).
__device__ __forceinline__ int64_t mask_offset(uint32_t r, const RingArgs& a) {
    uint32_t i1, i2, i3;
    row_coords(r, a, i1, i2, i3);
    const uint32_t m2 = i2 - fdiv(i2, a.a2) * a.aux_ne2;
    const uint32_t m3 = i3 - fdiv(i3, a.a3) * a.aux_ne3;
    return (int64_t)i1 * a.aux_st[1] + (int64_t)m2 * a.aux_st[2] + (int64_t)m3 * a.aux_st[3];
}

template <int T>
__device__ __forceinline__ double block_sum(double v, GroupScratch<T>* s) {
    return group_sum<T>(v, s);
}

__device__ __forceinline__ float4 ld_f4(const float* p) { return *reinterpret_cast<const float4*>(p); }

template <int OP>
__device__ __forceinline__ void store4(const RingArgs& a, float* drow, uint32_t v, float4 y) {
    if (a.dst_vec) {
        __stcs(reinterpret_cast<float4*>(drow) + v, y);
    } else {
        const int64_t s0 = a.dst_st[0];
        const int64_t c = (int64_t)v * 4;
        drow[c * s0] = y.x;
        drow[(c + 1) * s0] = y.y;
        drow[(c + 2) * s0] = y.z;
        drow[(c + 3) * s0] = y.w;
    }
}

// The four mask values of vector v (columns 4v .. 4v+3).
__device__ __forceinline__ float4 mask4(const RingArgs& a, const unsigned char* stage, int64_t moff, uint32_t v) {
    if (a.aux_mode == kAuxMaskStaged) {
        const unsigned char* m = stage + a.mask_offset;
        if (a.aux_f16) {
            const uint2 h = reinterpret_cast<const uint2*>(m)[v];
            return make_float4(f16_bits_to_f32(h.x & 0xffffu), f16_bits_to_f32(h.x >> 16), f16_bits_to_f32(h.y & 0xffffu),
                               f16_bits_to_f32(h.y >> 16));
        }
        return reinterpret_cast<const float4*>(m)[v];
    }
    const int64_t s0 = a.aux_st[0];
    const int64_t c = (int64_t)v * 4;
    float r[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int64_t e = moff + (c + k) * s0;
        r[k] = a.aux_f16 ? f16_bits_to_f32(reinterpret_cast<const uint16_t*>(a.aux)[e])
                         : reinterpret_cast<const float*>(a.aux)[e];
    }
    return make_float4(r[0], r[1], r[2], r[3]);
}

// v = x * scale (+ mask) for the fast soft_max pass: plain IEEE operations
// and hardware binary16 conversion (NaN payloads are irrelevant there: a
// NaN sends the row to the exact pass).
__device__ __forceinline__ float4 scaled4_fast(const RingArgs& a, const float* row, const unsigned char* stage,
                                               int64_t moff, uint32_t v) {
    float4 x = ld_f4(row + 4 * v);
    if (!a.apply_scale) return x;
    x = make_float4(__fmul_rn(x.x, a.param), __fmul_rn(x.y, a.param), __fmul_rn(x.z, a.param), __fmul_rn(x.w, a.param));
    if (a.aux_mode == kAuxNone) return x;
    float4 mk;
    if (a.aux_mode == kAuxMaskStaged && a.aux_f16) {
        const uint2 h = reinterpret_cast<const uint2*>(stage + a.mask_offset)[v];
        const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&h.x));
        const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&h.y));
        mk = make_float4(lo.x, lo.y, hi.x, hi.y);
    } else {
        mk = mask4(a, stage, moff, v);
    }
    return make_float4(__fadd_rn(x.x, mk.x), __fadd_rn(x.y, mk.y), __fadd_rn(x.z, mk.z), __fadd_rn(x.w, mk.w));
}

// Reductions for the register-resident soft_max rows.  They skip the
// leading barrier of group_max / group_sum: each uses its own scratch array
// and, between two uses of the same array, every thread passes the other
// reduction's barrier, so no reader of the previous value is left.  fmaxf
// skips NaN; the sign of a zero maximum does not change any exp(v - max).
// The maximum's barrier also carries every thread's stage-wait outcome
// (ok): *all_ok is the same AND of them in every thread, so the row needs
// no barrier of its own after the stage wait.
template <int T>
__device__ __forceinline__ float row_max_fast(float v, GroupScratch<T>* s, bool ok, bool* all_ok) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int lane = threadIdx.x & 31, warp = threadIdx.x / 32;
    const uint32_t warp_ok = __all_sync(0xffffffffu, ok) ? 1u : 0u;
    if (lane == 0) {
        s->f[warp] = v;
        s->h[warp] = warp_ok;
    }
    __syncthreads();
    v = s->f[0];
    uint32_t all = s->h[0];
#pragma unroll
    for (int w = 1; w < T / 32; ++w) {
        v = fmaxf(v, s->f[w]);
        all &= s->h[w];
    }
    *all_ok = all != 0;
    return v;
}

template <int T>
__device__ __forceinline__ double row_sum_fast(double v, GroupScratch<T>* s) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int lane = threadIdx.x & 31, warp = threadIdx.x / 32;
    if (lane == 0) s->d[warp] = v;
    __syncthreads();
    v = 0.0;
#pragma unroll
    for (int w = 0; w < T / 32; ++w) v += s->d[w];
    return v;
}

// soft_max operand modes of the register-resident pass (compile-time, so
// the per-vector work has no mode branches): v = x; v = x * scale; and
// v = x * scale + mask with the mask row staged as f16 or f32, or read with
// loads (any strides).
enum SmMode { kSmPlain = 0, kSmScale = 1, kSmMaskF16 = 2, kSmMaskF32 = 3, kSmMaskLoads = 4 };

template <int MODE>
__device__ __forceinline__ float4 sm_operand4(const RingArgs& a, const float* row, const unsigned char* stage,
                                              int64_t moff, uint32_t v) {
    float4 x = ld_f4(row + 4 * v);
    if constexpr (MODE == kSmPlain) return x;
    const float2 s2 = make_float2(a.param, a.param);
    x = cat2(__fmul2_rn(lo2(x), s2), __fmul2_rn(hi2(x), s2));
    if constexpr (MODE == kSmScale) return x;
    float4 mk;
    if constexpr (MODE == kSmMaskF16) {
        const uint2 h = reinterpret_cast<const uint2*>(stage + a.mask_offset)[v];
        const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&h.x));
        const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&h.y));
        mk = make_float4(lo.x, lo.y, hi.x, hi.y);
    } else if constexpr (MODE == kSmMaskF32) {
        mk = reinterpret_cast<const float4*>(stage + a.mask_offset)[v];
    } else {
        mk = mask4(a, stage, moff, v);
    }
    return cat2(__fadd2_rn(lo2(x), lo2(mk)), __fadd2_rn(hi2(x), hi2(mk)));
}

// Maximum, exps and their sum for the thread's R vectors (kept in sv).  A
// vector whose four v - max are all >= kSoftmaxPlainDivFloor takes the
// packed exponential (softmax_exp2); any other vector (a masked -inf, a
// tiny or NaN term) takes the scalar softmax_exp and sets its bit in
// *slow, which routes its division through the range-checked softmax_div.
// The thread's terms (at most 32, each <= 1) are summed in binary32 pairs,
// then the thread sums meet in binary64.  GUARD: the row does not fill all
// R * T vector slots.
// ok: this thread's stage wait succeeded; *all_ok comes back false in
// every thread (and nothing past the maximum runs) if any thread's did not.
template <int T, int R, int MODE, bool GUARD>
__device__ __forceinline__ double sm_exp_pass(const RingArgs& a, const float* row, const unsigned char* stage,
                                              int64_t moff, uint32_t nvec, float4 (&sv)[R], uint32_t* slow,
                                              GroupScratch<T>* red, bool ok, bool* all_ok) {
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < R; ++i) {
        const uint32_t v = threadIdx.x + (uint32_t)(i * T);
        if (!GUARD || v < nvec) {
            sv[i] = sm_operand4<MODE>(a, row, stage, moff, v);
            m = fmax3(fmax3(m, sv[i].x, sv[i].y), sv[i].z, sv[i].w);
        }
    }
    m = row_max_fast<T>(m, red, ok, all_ok);
    if (!*all_ok) return 0.0;
    const float2 nm2 = make_float2(-m, -m);  // x + (-m) is IEEE x - m
    float2 acc2 = make_float2(0.0f, 0.0f);
    uint32_t bits = 0;
#pragma unroll
    for (int i = 0; i < R; ++i) {
        const uint32_t v = threadIdx.x + (uint32_t)(i * T);
        if (!GUARD || v < nvec) {
            const float2 zl = __fadd2_rn(lo2(sv[i]), nm2), zh = __fadd2_rn(hi2(sv[i]), nm2);
            if (fmin3(fminf(zl.x, zl.y), zh.x, zh.y) >= kSoftmaxPlainDivFloor) {
                sv[i] = cat2(softmax_exp2(zl), softmax_exp2(zh));
            } else {
                sv[i] = make_float4(softmax_exp(zl.x), softmax_exp(zl.y), softmax_exp(zh.x), softmax_exp(zh.y));
                bits |= 1u << i;
            }
            acc2 = __fadd2_rn(acc2, lo2(sv[i]));
            acc2 = __fadd2_rn(acc2, hi2(sv[i]));
        }
    }
    *slow = bits;
    return row_sum_fast<T>((double)acc2.x + (double)acc2.y, red);
}

// e / denom for the thread's vectors: the packed Markstein quotient for the
// vectors whose terms are all >= e^kSoftmaxPlainDivFloor, the range-checked
// scalar form for the vectors flagged in slow.
template <int OP, int T, int R, bool GUARD>
__device__ __forceinline__ void sm_div_pass(const RingArgs& a, float* drow, uint32_t nvec, const float4 (&sv)[R],
                                            float denom, float inv, uint32_t slow) {
    const float2 d2 = make_float2(denom, denom), i2 = make_float2(inv, inv);
#pragma unroll
    for (int i = 0; i < R; ++i) {
        const uint32_t v = threadIdx.x + (uint32_t)(i * T);
        if (!GUARD || v < nvec) {
            if (!(slow >> i & 1u))
                store4<OP>(a, drow, v, cat2(markstein_div2(lo2(sv[i]), d2, i2), markstein_div2(hi2(sv[i]), d2, i2)));
            else
                store4<OP>(a, drow, v,
                           make_float4(softmax_div(sv[i].x, denom, inv), softmax_div(sv[i].y, denom, inv),
                                       softmax_div(sv[i].z, denom, inv), softmax_div(sv[i].w, denom, inv)));
        }
    }
}

// R > 0 (soft_max only): each thread keeps its R vectors of the row in
// registers (rows of at most 4 * T * R elements), MODE being the operand
// mode (SmMode); R == 0 loops over the staged row for every pass.
template <int OP, int T, int R, int MODE>
__global__ void __launch_bounds__(T, R >= 8 ? 2 : (R >= 4 ? 3 : 1024 / T)) row_ring(RingArgs a) {
    extern __shared__ __align__(128) unsigned char ring_smem[];
    __shared__ __align__(8) uint64_t full[kRingStagesMax];
    __shared__ GroupScratch<T> red;
    if (!a.early) pdl_enter();
    const int tid = threadIdx.x;
    const int S = a.stages;
    const uint32_t mine = a.rows > blockIdx.x ? (a.rows - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    const float* wsm = reinterpret_cast<const float*>(ring_smem);
    unsigned char* stage0 = ring_smem + a.weight_bytes;
    const uint32_t nvec = a.ne0 / 4;
    const uint32_t msize = a.aux_f16 ? 2u : 4u;

    if (tid == 0) {
        for (int s = 0; s < S; ++s) mbar_init(&full[s], 1);
        mbar_init_fence();
    }
    if constexpr (OP == kRingRmsMul) {
        float* w = reinterpret_cast<float*>(ring_smem);
        for (uint32_t c = tid; c < a.ne0; c += T) w[c] = reinterpret_cast<const float*>(a.aux)[(int64_t)c * a.aux_st[0]];
    }
    __syncthreads();

    auto issue = [&](uint32_t k, int s) {  // row k into stage s
        const uint32_t r = blockIdx.x + k * gridDim.x;
        unsigned char* st = stage0 + (size_t)s * a.stage_bytes;
        const uint32_t rb = a.ne0 * 4u;
        const uint32_t mb = a.aux_mode == kAuxMaskStaged ? a.ne0 * msize : 0u;
        mbar_expect_tx(&full[s], rb + mb);
        bulk_load(st, a.src + row_offset(r, a, a.src_st) * 4, rb, &full[s]);
        if (mb) bulk_load(st + a.mask_offset, a.aux + mask_offset(r, a) * msize, mb, &full[s]);
    };
    if (tid == 0)
        for (uint32_t k = 0; k < mine && k < (uint32_t)S; ++k) issue(k, (int)k);
    if (a.early) pdl_enter();  // every global store comes after this

    int s = 0;            // stage of row k: k % S
    uint32_t parity = 0;  // phase parity of row k: (k / S) & 1
    for (uint32_t k = 0; k < mine; ++k, s = s + 1 == S ? 0 : s + 1, parity ^= (s == 0)) {
        const bool ok = mbar_wait(&full[s], parity);
        // an expired wait: every thread returns together, thread 0 records
        // the fault and waits (bounded) for the copies still in flight
        auto fail = [&]() {
            if (tid == 0) {
                atomicExch(a.fault, 1u);
                for (uint32_t j = k; j < mine && j < k + (uint32_t)S; ++j)
                    mbar_wait(&full[j % (uint32_t)S], (j / (uint32_t)S) & 1u);
            }
        };
        // the register-resident soft_max folds the outcome into its maximum's
        // barrier (row_max_fast); every other pass agrees on it here
        constexpr bool kFoldedWait = OP == kRingSoftMax && R > 0;
        if constexpr (!kFoldedWait) {
            if (!__syncthreads_and(ok)) {
                fail();
                return;
            }
        }
        unsigned char* stage = stage0 + (size_t)s * a.stage_bytes;
        float* row = reinterpret_cast<float*>(stage);
        const uint32_t r = blockIdx.x + k * gridDim.x;
        float* drow = reinterpret_cast<float*>(a.dst) + row_offset(r, a, a.dst_st);

        if constexpr (OP == kRingNorm || OP == kRingNormGeneric) {
            double acc = 0.0;
            for (uint32_t v = tid; v < nvec; v += T) {
                const float4 x = ld_f4(row + 4 * v);
                acc += (double)x.x;
                acc += (double)x.y;
                acc += (double)x.z;
                acc += (double)x.w;
            }
            acc = block_sum<T>(acc, &red);
            const float mean = __double2float_rn(acc / (double)a.ne0);
            double vs = 0.0;
            for (uint32_t v = tid; v < nvec; v += T) {
                const float4 x = ld_f4(row + 4 * v);
                const float cs[4] = {__fsub_rn(x.x, mean), __fsub_rn(x.y, mean), __fsub_rn(x.z, mean),
                                     __fsub_rn(x.w, mean)};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    if constexpr (OP == kRingNormGeneric) {
                        vs += (double)__fmul_rn(cs[k], cs[k]);  // squared in binary32
                    } else {
                        const double c = (double)cs[k];
                        vs += c * c;
                    }
                }
            }
            vs = block_sum<T>(vs, &red);
            float scale;
            if constexpr (OP == kRingNormGeneric) {
                scale = __double2float_rn(__ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(vs / (double)a.ne0, (double)a.param))));
            } else {
                const float variance = __double2float_rn(vs / (double)a.ne0);
                scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(variance, a.param)));
            }
            for (uint32_t v = tid; v < nvec; v += T) {
                const float4 x = ld_f4(row + 4 * v);
                store4<OP>(a, drow, v,
                           make_float4(f_mul(f_sub(x.x, mean), scale), f_mul(f_sub(x.y, mean), scale),
                                       f_mul(f_sub(x.z, mean), scale), f_mul(f_sub(x.w, mean), scale)));
            }
        } else if constexpr (OP == kRingRms || OP == kRingRmsMul || OP == kRingRmsGeneric) {
            double acc = 0.0;
            for (uint32_t v = tid; v < nvec; v += T) {
                const float4 x = ld_f4(row + 4 * v);
                acc += (double)__fmul_rn(x.x, x.x);
                acc += (double)__fmul_rn(x.y, x.y);
                acc += (double)__fmul_rn(x.z, x.z);
                acc += (double)__fmul_rn(x.w, x.w);
            }
            acc = block_sum<T>(acc, &red);
            const float mean = __double2float_rn(acc / (double)a.ne0);
            const float scale = OP == kRingRmsGeneric
                                    ? __double2float_rn(__ddiv_rn(1.0, __dsqrt_rn(__dadd_rn((double)mean, (double)a.param))))
                                    : __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, a.param)));
            for (uint32_t v = tid; v < nvec; v += T) {
                const float4 x = ld_f4(row + 4 * v);
                float4 y = make_float4(f_mul(x.x, scale), f_mul(x.y, scale), f_mul(x.z, scale), f_mul(x.w, scale));
                if constexpr (OP == kRingRmsMul) {
                    const float4 w = ld_f4(wsm + 4 * v);
                    y = make_float4(f_mul(y.x, w.x), f_mul(y.y, w.y), f_mul(y.z, w.z), f_mul(y.w, w.w));
                }
                store4<OP>(a, drow, v, y);
            }
        } else {
            // soft_max (reductions.rs:565-638): v = x * scale (+ mask); max
            // (starting from element 0); e = exp(v - max); sum in f64; e / sum.
            //
            // Fast pass: plain IEEE arithmetic.  While no v is NaN and the
            // maximum is finite no step can produce a NaN, so the x86 NaN
            // rules never apply and the plain results are the reference's
            // bits.  A NaN lane reports +inf to the max reduction; a row
            // whose maximum comes back non-finite is redone exactly below.
            const int64_t moff = a.aux_mode == kAuxMaskLoads ? mask_offset(r, a) : 0;
            if constexpr (R > 0) {
                // Register-resident fast pass: the row is read from the stage
                // once.  No NaN check is needed while reading: a NaN v, or a
                // maximum of +-inf (inf - inf, -inf - -inf), makes some
                // v - max NaN, its exp NaN and the f64 sum NaN, while
                // otherwise every exp is at most 1 and the sum is finite.  A
                // row whose sum comes back non-finite is redone exactly
                // below from the untouched stage.
                float4 sv[R];
                uint32_t slow;
                const bool guard = nvec != (uint32_t)(R * T);
                bool all_ok;
                const double acc = guard ? sm_exp_pass<T, R, MODE, true>(a, row, stage, moff, nvec, sv, &slow, &red, ok,
                                                                        &all_ok)
                                         : sm_exp_pass<T, R, MODE, false>(a, row, stage, moff, nvec, sv, &slow, &red,
                                                                         ok, &all_ok);
                if (!all_ok) {
                    fail();
                    return;
                }
                if (isfinite(acc)) {
                    // every thread has finished reading the stage: refill it now
                    if (tid == 0 && k + (uint32_t)S < mine) {
                        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                        issue(k + (uint32_t)S, s);
                    }
                    const float denom = __double2float_rn(acc);  // >= 1: the maximum contributes exp(0)
                    const float inv = __frcp_rn(denom);
                    if (guard) sm_div_pass<OP, T, R, true>(a, drow, nvec, sv, denom, inv, slow);
                    else sm_div_pass<OP, T, R, false>(a, drow, nvec, sv, denom, inv, slow);
                    continue;
                }
            }
            float m = bitsf(0x7fc00000u);  // NaN = "no value yet" (fmaxf skips it)
            if constexpr (R == 0) {
                bool odd = false;
                for (uint32_t v = tid; v < nvec; v += T) {
                    const float4 s = scaled4_fast(a, row, stage, moff, v);
                    odd = odd || is_nan(s.x) || is_nan(s.y) || is_nan(s.z) || is_nan(s.w);
                    m = fmaxf(fmaxf(m, s.x), fmaxf(s.y, fmaxf(s.z, s.w)));
                }
                m = group_max<T>(odd ? INFINITY : m, &red);
            }
            if (R == 0 && isfinite(m)) {
                double acc = 0.0;
                for (uint32_t v = tid; v < nvec; v += T) {
                    const float4 s = scaled4_fast(a, row, stage, moff, v);
                    const float4 e = make_float4(softmax_exp(__fsub_rn(s.x, m)), softmax_exp(__fsub_rn(s.y, m)),
                                                 softmax_exp(__fsub_rn(s.z, m)), softmax_exp(__fsub_rn(s.w, m)));
                    reinterpret_cast<float4*>(row)[v] = e;
                    acc += (double)e.x;
                    acc += (double)e.y;
                    acc += (double)e.z;
                    acc += (double)e.w;
                }
                acc = block_sum<T>(acc, &red);
                const float denom = __double2float_rn(acc);  // >= 1: the maximum contributes exp(0)
                const float inv = __frcp_rn(denom);
                for (uint32_t v = tid; v < nvec; v += T) {
                    const float4 e = ld_f4(row + 4 * v);
                    store4<OP>(a, drow, v,
                               make_float4(softmax_div(e.x, denom, inv), softmax_div(e.y, denom, inv), softmax_div(e.z, denom, inv),
                                           softmax_div(e.w, denom, inv)));
                }
            } else {
                m = bitsf(0x7fc00000u);
                for (uint32_t v = tid; v < nvec; v += T) {
                    float4 x = ld_f4(row + 4 * v);
                    if (a.apply_scale) {
                        x = make_float4(f_mul(x.x, a.param), f_mul(x.y, a.param), f_mul(x.z, a.param), f_mul(x.w, a.param));
                        if (a.aux_mode != kAuxNone) {
                            const float4 mk = mask4(a, stage, moff, v);
                            x = make_float4(f_add(x.x, mk.x), f_add(x.y, mk.y), f_add(x.z, mk.z), f_add(x.w, mk.w));
                        }
                        reinterpret_cast<float4*>(row)[v] = x;
                    }
                    m = max_nn(m, x.x);
                    m = max_nn(m, x.y);
                    m = max_nn(m, x.z);
                    m = max_nn(m, x.w);
                }
                m = group_max<T>(m, &red);  // its barriers also publish row[0]
                const float first = row[0];
                if (is_nan(first)) m = first;  // reductions.rs:572: the scan starts from element 0
                double acc = 0.0;
                for (uint32_t v = tid; v < nvec; v += T) {
                    const float4 x = ld_f4(row + 4 * v);
                    const float4 e = make_float4(lm_exp(f_sub(x.x, m)), lm_exp(f_sub(x.y, m)), lm_exp(f_sub(x.z, m)),
                                                 lm_exp(f_sub(x.w, m)));
                    reinterpret_cast<float4*>(row)[v] = e;
                    acc += (double)e.x;
                    acc += (double)e.y;
                    acc += (double)e.z;
                    acc += (double)e.w;
                }
                acc = block_sum<T>(acc, &red);
                const float denom = __double2float_rn(acc);
                for (uint32_t v = tid; v < nvec; v += T) {
                    const float4 e = ld_f4(row + 4 * v);
                    store4<OP>(a, drow, v,
                               make_float4(f_div(e.x, denom), f_div(e.y, denom), f_div(e.z, denom), f_div(e.w, denom)));
                }
            }
        }
        __syncthreads();  // every thread is done with this stage
        if (tid == 0 && k + (uint32_t)S < mine) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue(k + (uint32_t)S, s);
        }
    }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

uint32_t round_up(uint64_t v, uint32_t a) { return (uint32_t)((v + a - 1) / a * a); }

bool fits_u32(uint64_t v) { return v > 0 && v <= 0xffffffffull; }

// Occupancy first: as many CTAs per SM as registers and two stages each
// allow (each CTA's row passes are a chain of dependent steps and barriers,
// so throughput comes from several rows in progress per SM); then deeper
// rings (up to kRingStagesMax) while shared memory lasts.
template <int OP, int T, int R = 0, int MODE = 0>
cudaError_t launch_ring_kernel(const LaunchEnv& env, RingArgs a, uint64_t rows, bool* launched) {
    static DeviceFlags configured;  // devices with the attribute set
    if (!configured.done(env.device)) {
        const cudaError_t err =
            cudaFuncSetAttribute(row_ring<OP, T, R, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kRingSmemPerSm);
        if (err != cudaSuccess) return err;
        configured.mark(env.device);
    }
    *launched = false;
    const uint32_t two = a.weight_bytes + 2 * a.stage_bytes;
    if (two > kRingSmemPerSm) return cudaSuccess;
    int ctas = 0;
    cudaError_t err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&ctas, row_ring<OP, T, R, MODE>, T, two);
    if (err != cudaSuccess) return err;
    if (ctas < 1) return cudaSuccess;
    if (ctas > 8) ctas = 8;
    auto stages_for = [&](int c) -> uint32_t {
        const uint32_t budget = kRingSmemPerSm / (uint32_t)c;
        return budget > a.weight_bytes ? (budget - a.weight_bytes) / a.stage_bytes : 0u;
    };
    uint32_t stages = stages_for(ctas);
    while (stages < 2 && ctas > 1) stages = stages_for(--ctas);
    if (stages < 2) return cudaSuccess;
    a.stages = (int)(stages > (uint32_t)kRingStagesMax ? kRingStagesMax : stages);
    const uint32_t smem = a.weight_bytes + (uint32_t)a.stages * a.stage_bytes;
    const uint64_t cap = (uint64_t)env.sm_count * ctas;
    const uint32_t grid = (uint32_t)(rows < cap ? rows : cap);
    err = launch_dependent(row_ring<OP, T, R, MODE>, dim3(grid), dim3(T), smem, env.stream, a);
    *launched = true;
    return err != cudaSuccess ? err : cudaGetLastError();
}

template <int R>
cudaError_t launch_softmax_ring(const LaunchEnv& env, const RingArgs& a, uint64_t rows, bool* launched) {
    if (!a.apply_scale) return launch_ring_kernel<kRingSoftMax, kRingThreads, R, kSmPlain>(env, a, rows, launched);
    switch (a.aux_mode) {
    case kAuxNone: return launch_ring_kernel<kRingSoftMax, kRingThreads, R, kSmScale>(env, a, rows, launched);
    case kAuxMaskStaged:
        return a.aux_f16 ? launch_ring_kernel<kRingSoftMax, kRingThreads, R, kSmMaskF16>(env, a, rows, launched)
                         : launch_ring_kernel<kRingSoftMax, kRingThreads, R, kSmMaskF32>(env, a, rows, launched);
    default: return launch_ring_kernel<kRingSoftMax, kRingThreads, R, kSmMaskLoads>(env, a, rows, launched);
    }
}

}  // namespace

// Plans and launches the ring kernel when the view qualifies: rows of
// ne0 % 4 == 0 floats, unit stride in dim 0, every row start 16-byte
// aligned, and (for soft_max) dense src/dst so the f64 sum applies.  Returns
// false (nothing launched) otherwise.  op: 0 norm, 1 rms_norm, 2 rms_norm *
// weight, 3 soft_max, 4 / 5 the generic envelope's norm / rms_norm.
bool launch_row_ring(const LaunchEnv& env, const RowPlan& p, int op, float param, bool apply_scale,
                     cudaError_t* err) {
    const uint64_t ne0 = p.ne[0];
    if (ne0 < 1024 || ne0 % 4 != 0 || !fits_u32(p.rows) || !fits_u32(p.ne[1]) || !fits_u32(p.ne[2])) return false;
    if (p.dst_ordinal || p.src.st[0] != 1 || !aligned16(p.src.ptr)) return false;
    for (int d = 1; d < 4; ++d)
        if (p.src.st[d] % 4 != 0) return false;
    if (op == 3 && !p.dense) return false;
    RingArgs a{};
    a.src = p.src.ptr;
    a.dst = p.dst.ptr;
    a.fault = reinterpret_cast<uint32_t*>(static_cast<char*>(env.workspace) + kFaultWordOffset);
    a.ne0 = (uint32_t)ne0;
    a.rows = (uint32_t)p.rows;
    a.ne1 = (uint32_t)p.ne[1];
    a.ne2 = (uint32_t)p.ne[2];
    a.d1 = make_fastdiv(a.ne1);
    a.d2 = make_fastdiv(a.ne2);
    for (int d = 0; d < 4; ++d) {
        a.src_st[d] = p.src.st[d];
        a.dst_st[d] = p.dst.st[d];
    }
    a.dst_vec = p.dst.st[0] == 1 && aligned16(p.dst.ptr) && p.dst.st[1] % 4 == 0 && p.dst.st[2] % 4 == 0 &&
                p.dst.st[3] % 4 == 0;
    a.apply_scale = apply_scale ? 1 : 0;
    a.param = param;
    a.aux_mode = kAuxNone;
    uint32_t mask_bytes = 0;
    if (op == 2) {
        a.aux_mode = kAuxWeight;
        a.aux = p.aux.ptr;
        a.aux_st[0] = p.aux.st[0];
        a.weight_bytes = round_up(ne0 * 4, kStageAlign);
    } else if (op == 3 && apply_scale && p.has_aux) {
        a.aux = p.aux.ptr;
        a.aux_f16 = p.aux_dtype == (int)DType::F16 ? 1 : 0;
        for (int d = 0; d < 4; ++d) a.aux_st[d] = p.aux.st[d];
        if (!fits_u32(p.aux.ne[2]) || !fits_u32(p.aux.ne[3])) return false;
        a.aux_ne2 = (uint32_t)p.aux.ne[2];
        a.aux_ne3 = (uint32_t)p.aux.ne[3];
        a.a2 = make_fastdiv(a.aux_ne2);
        a.a3 = make_fastdiv(a.aux_ne3);
        const uint32_t ms = a.aux_f16 ? 2 : 4;
        bool staged = p.aux.st[0] == 1 && (ne0 * ms) % 16 == 0 && aligned16(p.aux.ptr);
        for (int d = 1; d < 4; ++d) staged = staged && ((uint64_t)p.aux.st[d] * ms) % 16 == 0;
        a.aux_mode = staged ? kAuxMaskStaged : kAuxMaskLoads;
        if (staged) mask_bytes = round_up(ne0 * ms, kStageAlign);
    }
    const uint32_t row_bytes = round_up(ne0 * 4, kStageAlign);
    a.mask_offset = row_bytes;
    a.stage_bytes = row_bytes + mask_bytes;
    a.early = reads_clear(env, span_of(p.src, 4)) &&
              (a.aux_mode == kAuxNone || reads_clear(env, span_of(p.aux, a.aux_f16 && op == 3 ? 2 : 4)));
    cudaError_t e;
    bool launched = false;
    switch (op) {
    case 0: e = launch_ring_kernel<kRingNorm, kRingThreads>(env, a, p.rows, &launched); break;
    case 1: e = launch_ring_kernel<kRingRms, kRingThreads>(env, a, p.rows, &launched); break;
    case 2: e = launch_ring_kernel<kRingRmsMul, kRingThreads>(env, a, p.rows, &launched); break;
    case 3: {
        // vectors per thread, rounded up to a power of two, up to 8
        const uint64_t per = (ne0 / 4 + kRingThreads - 1) / kRingThreads;
        if (per <= 1) e = launch_softmax_ring<1>(env, a, p.rows, &launched);
        else if (per <= 2) e = launch_softmax_ring<2>(env, a, p.rows, &launched);
        else if (per <= 4) e = launch_softmax_ring<4>(env, a, p.rows, &launched);
        else if (per <= 8) e = launch_softmax_ring<8>(env, a, p.rows, &launched);
        else e = launch_ring_kernel<kRingSoftMax, kRingThreads>(env, a, p.rows, &launched);
        break;
    }
    case 4: e = launch_ring_kernel<kRingNormGeneric, kRingThreads>(env, a, p.rows, &launched); break;
    default: e = launch_ring_kernel<kRingRmsGeneric, kRingThreads>(env, a, p.rows, &launched); break;
    }
    if (e == cudaSuccess && !launched) return false;
    if (e == cudaSuccess) stream_wrote(env.stream, span_of(p.dst, 4));
    ++*env.launches;
    *err = e;
    return true;
}

}  // namespace emel
