// Row gather (get_rows.rs): dst row r = source row idx[r] of the source
// batch the index's outer coordinates select, decoded to f32.  Sources:
// F32 (strided rows), byte-backed F32 (rows at any byte offset), F16 and BF16
// (any strides), and the Q4_0 / Q8_0 / Q4_K block formats (dense rows of
// packed blocks).
//
// Indices live in device memory, so the reference's index guard (every
// index in [0, rows) before anything is written) runs on the device: a
// check kernel scans them and raises the call's flag (and the context's
// sticky "rejected" word, reported by emel_cuda_stream_synchronize as
// EMEL_CUDA_INDEX_OUT_OF_BOUNDS); the gather kernel, a programmatic
// dependent of the check, returns without a store when the flag is up.
//
// Work: one CTA per destination row at a time (grid-stride over rows).
// F32 / F16 / BF16 rows move as 16-byte vectors when the source row is
// contiguous and aligned; quantized rows are staged chunk by chunk in shared
// memory with the widest aligned loads the row allows, then every thread
// decodes four consecutive values (one block, one nibble half) and stores
// them as one 16-byte vector.
#include <cuda_fp16.h>

#include "common.cuh"
#include "launch.hpp"
#include "pdl.cuh"

namespace emel {

namespace {

constexpr int kGatherThreads = 256;
constexpr int kQuantChunkValues = 4096;  // values staged per chunk (16 KB of output)

__device__ __forceinline__ void row_coords(const GatherPlan& p, uint64_t r, uint64_t& i1, uint64_t& i2) {
    const uint64_t t = r / p.idx_ne[0];
    i1 = t % p.idx_ne[1];
    i2 = t / p.idx_ne[1];
}

__device__ __forceinline__ int32_t index_of(const GatherPlan& p, uint64_t r) {
    const uint64_t i0 = r % p.idx_ne[0], t = r / p.idx_ne[0];
    const uint64_t i1 = t % p.idx_ne[1], i2 = t / p.idx_ne[1];
    return p.idx[(int64_t)i0 * p.idx_st[0] + (int64_t)i1 * p.idx_st[1] + (int64_t)i2 * p.idx_st[2]];
}

__global__ void __launch_bounds__(kGatherThreads) gather_check(GatherPlan p) {
    pdl_enter();
    const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
    bool bad = false;
    for (uint64_t r = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; r < p.dst_rows; r += stride) {
        const int32_t i = index_of(p, r);
        bad = bad || i < 0 || (uint64_t)i >= p.rows;
    }
    if (__syncthreads_or(bad) && threadIdx.x == 0) {
        atomicOr(p.flag, 1u);
        atomicExch(p.reject, p.reject_code);
    }
}

// f16_to_f32 of f16_matmul.rs:508-532: exact, a NaN keeps its payload bits.
__device__ __forceinline__ float f16_exact_bits(uint16_t h) {
    if ((h & 0x7c00u) == 0x7c00u) return bitsf(((uint32_t)(h & 0x8000u) << 16) | 0x7f800000u | ((uint32_t)(h & 0x3ffu) << 13));
    return __half2float(__ushort_as_half(h));
}

// fp16_to_f32 of quant.rs:287-302 (exact for numbers; its binary32 multiply
// quietens a NaN, keeping sign and payload).
__device__ __forceinline__ float f16_quant_scale(uint16_t h) {
    if ((h & 0x7c00u) == 0x7c00u && (h & 0x3ffu) != 0)
        return bitsf(((uint32_t)(h & 0x8000u) << 16) | 0x7fc00000u | ((uint32_t)(h & 0x3ffu) << 13));
    return __half2float(__ushort_as_half(h));
}

template <int KIND>
__device__ __forceinline__ float half_value(uint16_t h) {
    if constexpr (KIND == kGatherF16) return f16_exact_bits(h);
    return bitsf((uint32_t)h << 16);
}

// ---- F32 / F16 / BF16 ---------------------------------------------------------
template <int KIND>
__device__ __forceinline__ void half_store8(float* out, uint64_t v, uint4 u) {
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
    float f[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        f[2 * k] = half_value<KIND>((uint16_t)(w[k] & 0xffffu));
        f[2 * k + 1] = half_value<KIND>((uint16_t)(w[k] >> 16));
    }
    __stcs(reinterpret_cast<float4*>(out) + 2 * v, make_float4(f[0], f[1], f[2], f[3]));
    __stcs(reinterpret_cast<float4*>(out) + 2 * v + 1, make_float4(f[4], f[5], f[6], f[7]));
}

template <int KIND>
__global__ void __launch_bounds__(kGatherThreads) gather_plain(GatherPlan p) {
    constexpr int U = 4;  // 16-byte loads in flight per thread
    pdl_enter();
    if (*reinterpret_cast<volatile uint32_t*>(p.flag) != 0u) return;
    const uint64_t cols = p.cols;
    uint64_t r = blockIdx.x;
    int32_t next = r < p.dst_rows ? index_of(p, r) : 0;
    for (; r < p.dst_rows; r += gridDim.x) {
        uint64_t i1, i2;
        row_coords(p, r, i1, i2);
        const uint64_t index = (uint64_t)next;
        if (r + gridDim.x < p.dst_rows) next = index_of(p, r + gridDim.x);  // in flight during this row
        const char* row = p.src + index * p.src_st[1] + i1 * p.src_st[2] + i2 * p.src_st[3];
        float* out = p.dst + r * cols;
        const bool vec = p.vec && (reinterpret_cast<uintptr_t>(row) & 15u) == 0;
        constexpr bool kF32 = KIND == kGatherF32 || KIND == kGatherF32Bytes;
        if (vec) {
            // F32: 4 floats per vector (read_row_contiguous, tensor_view.rs:756-769:
            // columns 4 bytes apart); F16 / BF16: 8 halves per vector
            const uint64_t nv = kF32 ? cols / 4 : cols / 8;
            const uint4* in = reinterpret_cast<const uint4*>(row);
            uint64_t v = threadIdx.x;
            for (; v + (U - 1) * kGatherThreads < nv; v += U * kGatherThreads) {
                uint4 q[U];
#pragma unroll
                for (int k = 0; k < U; ++k) q[k] = __ldcs(in + v + k * kGatherThreads);
#pragma unroll
                for (int k = 0; k < U; ++k) {
                    if constexpr (kF32)
                        __stcs(reinterpret_cast<uint4*>(out) + v + k * kGatherThreads, q[k]);
                    else
                        half_store8<KIND>(out, v + k * kGatherThreads, q[k]);
                }
            }
            for (; v < nv; v += kGatherThreads) {
                const uint4 q = __ldcs(in + v);
                if constexpr (kF32) __stcs(reinterpret_cast<uint4*>(out) + v, q);
                else half_store8<KIND>(out, v, q);
            }
        } else if constexpr (KIND == kGatherF32) {
            const float* in = reinterpret_cast<const float*>(row);
            for (uint64_t c = threadIdx.x; c < cols; c += kGatherThreads) out[c] = in[c];
        } else if constexpr (KIND == kGatherF32Bytes) {
            // ByteTensorView::read_row_contiguous (tensor_view.rs:645-680): the 4 little-endian
            // bytes at row + 4c.  A row off a word boundary is read as the aligned
            // words that hold its bytes, each joined with the next by a funnel
            // shift; every word read holds at least one byte of the row.
            const uintptr_t a = reinterpret_cast<uintptr_t>(row);
            const uint32_t sh = (uint32_t)(a & 3u) * 8u;
            if (p.vec) {
                // 16-byte destination vectors: output vector v is bytes
                // [16v, 16v + 16) of the row, held by aligned source chunks v
                // and v + 1 (the row is off a 16-byte boundary, so both hold
                // bytes of the row); rotate by (a & 15) / 4 words, then funnel.
                const uint4* base = reinterpret_cast<const uint4*>(a & ~(uintptr_t)15);
                const uint32_t q = (uint32_t)(a & 15u) >> 2;
                const uint64_t nv = cols / 4;
                for (uint64_t v = threadIdx.x; v < nv; v += kGatherThreads) {
                    const uint4 x = __ldg(base + v), y = __ldg(base + v + 1);
                    uint32_t w[8] = {x.x, x.y, x.z, x.w, y.x, y.y, y.z, y.w};
                    if (q & 2u) {
#pragma unroll
                        for (int i = 0; i < 6; ++i) w[i] = w[i + 2];
                    }
                    if (q & 1u) {
#pragma unroll
                        for (int i = 0; i < 7; ++i) w[i] = w[i + 1];
                    }
                    __stcs(reinterpret_cast<uint4*>(out) + v,
                           make_uint4(__funnelshift_r(w[0], w[1], sh), __funnelshift_r(w[1], w[2], sh),
                                      __funnelshift_r(w[2], w[3], sh), __funnelshift_r(w[3], w[4], sh)));
                }
            } else if (sh == 0) {
                const float* in = reinterpret_cast<const float*>(row);
                for (uint64_t c = threadIdx.x; c < cols; c += kGatherThreads) out[c] = in[c];
            } else {
                const uint32_t* w = reinterpret_cast<const uint32_t*>(a & ~(uintptr_t)3);
                for (uint64_t c = threadIdx.x; c < cols; c += kGatherThreads)
                    out[c] = __uint_as_float(__funnelshift_r(__ldg(w + c), __ldg(w + c + 1), sh));
            }
        } else {
            for (uint64_t c = threadIdx.x; c < cols; c += kGatherThreads)
                out[c] = half_value<KIND>(*reinterpret_cast<const uint16_t*>(row + c * p.src_st[0]));
        }
    }
}

// ---- quantized blocks -----------------------------------------------------------
template <int KIND>
struct QuantFormat;
template <>
struct QuantFormat<kGatherQ4_0> {
    static constexpr int kValues = 32, kBytes = 18;
};
template <>
struct QuantFormat<kGatherQ8_0> {
    static constexpr int kValues = 32, kBytes = 34;
};
template <>
struct QuantFormat<kGatherQ4_K> {
    static constexpr int kValues = 256, kBytes = 144;
};

__device__ __forceinline__ uint16_t ld_le16(const unsigned char* b) { return (uint16_t)(b[0] | (b[1] << 8)); }

// Values v .. v + 3 (v % 4 == 0) of the block at `b` (quant.rs:106-134,
// 178-205; quant_more.rs:438-468, 952-961) in the reference's binary32
// operation order.  EXACT applies the x86 NaN rules to every operation; the
// plain pass agrees with it on every non-NaN result, so a NaN result is
// recomputed exactly.
template <int KIND, bool EXACT>
__device__ __forceinline__ float4 decode4_as(const unsigned char* b, int v) {
    using A = Arith<EXACT>;
    float r[4];
    if constexpr (KIND == kGatherQ8_0) {
        const float scale = f16_quant_scale(ld_le16(b));
#pragma unroll
        for (int k = 0; k < 4; ++k) r[k] = A::mul((float)(int8_t)b[2 + v + k], scale);
    } else if constexpr (KIND == kGatherQ4_0) {
        const float scale = f16_quant_scale(ld_le16(b));
        const bool high = v >= 16;
        const int j = high ? v - 16 : v;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const unsigned q = high ? (b[2 + j + k] >> 4) : (b[2 + j + k] & 0x0fu);
            r[k] = A::mul(__fsub_rn((float)q, 8.0f), scale);
        }
    } else {
        const float scale = f16_quant_scale(ld_le16(b));
        const float minimum = f16_quant_scale(ld_le16(b + 2));
        const unsigned char* sc = b + 4;
        const int g = v / 64, within = v % 64;
        const bool high = within >= 32;
        const int s = 2 * g + (high ? 1 : 0);
        unsigned sv, mv;
        if (s < 4) {
            sv = sc[s] & 0x3fu;
            mv = sc[s + 4] & 0x3fu;
        } else {
            sv = (sc[s + 4] & 0x0fu) | ((unsigned)(sc[s - 4] >> 6) << 4);
            mv = (unsigned)(sc[s + 4] >> 4) | ((unsigned)(sc[s] >> 6) << 4);
        }
        const float d = A::mul(scale, (float)sv), m = A::mul(minimum, (float)mv);
        const unsigned char* q = b + 16 + 32 * g + (high ? within - 32 : within);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const unsigned n = high ? (q[k] >> 4) : (q[k] & 0x0fu);
            r[k] = A::sub(A::mul(d, (float)n), m);
        }
    }
    return make_float4(r[0], r[1], r[2], r[3]);
}

template <int KIND>
__device__ __noinline__ float4 decode4_exact(const unsigned char* b, int v) {
    return decode4_as<KIND, true>(b, v);
}

template <int KIND>
__device__ __forceinline__ float4 decode4(const unsigned char* b, int v) {
    const float4 r = decode4_as<KIND, false>(b, v);
    if (!(is_nan(r.x) || is_nan(r.y) || is_nan(r.z) || is_nan(r.w))) return r;
    return decode4_exact<KIND>(b, v);
}

// Copies `bytes` bytes from global `src` into shared `dst` with the widest
// loads both ends allow (16, 4 or 2 bytes; rows are whole blocks, so even).
__device__ __forceinline__ void stage(unsigned char* dst, const unsigned char* src, uint32_t bytes) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(src);
    if ((a & 15u) == 0 && (bytes & 15u) == 0) {
        for (uint32_t i = threadIdx.x; i < bytes / 16; i += kGatherThreads)
            reinterpret_cast<uint4*>(dst)[i] = __ldcs(reinterpret_cast<const uint4*>(src) + i);
    } else if ((a & 3u) == 0 && (bytes & 3u) == 0) {
        for (uint32_t i = threadIdx.x; i < bytes / 4; i += kGatherThreads)
            reinterpret_cast<uint32_t*>(dst)[i] = __ldcs(reinterpret_cast<const unsigned int*>(src) + i);
    } else {
        for (uint32_t i = threadIdx.x; i < bytes / 2; i += kGatherThreads)
            reinterpret_cast<uint16_t*>(dst)[i] = __ldcs(reinterpret_cast<const unsigned short*>(src) + i);
    }
}

template <int KIND>
__global__ void __launch_bounds__(kGatherThreads) gather_quant(GatherPlan p) {
    using F = QuantFormat<KIND>;
    constexpr int kChunkBlocks = kQuantChunkValues / F::kValues;
    __shared__ __align__(16) unsigned char smem[kChunkBlocks * F::kBytes];
    pdl_enter();
    if (*reinterpret_cast<volatile uint32_t*>(p.flag) != 0u) return;
    const uint64_t blocks = p.cols / F::kValues;
    for (uint64_t r = blockIdx.x; r < p.dst_rows; r += gridDim.x) {
        uint64_t i1, i2;
        row_coords(p, r, i1, i2);
        const uint64_t index = (uint64_t)index_of(p, r);
        const unsigned char* row =
            reinterpret_cast<const unsigned char*>(p.src) + ((i2 * p.batches + i1) * p.rows + index) * p.row_bytes;
        float4* out = reinterpret_cast<float4*>(p.dst + r * p.cols);
        for (uint64_t b0 = 0; b0 < blocks; b0 += kChunkBlocks) {
            const uint32_t nb = (uint32_t)(blocks - b0 < (uint64_t)kChunkBlocks ? blocks - b0 : kChunkBlocks);
            __syncthreads();  // the previous chunk's readers are done
            stage(smem, row + b0 * F::kBytes, nb * F::kBytes);
            __syncthreads();
            const uint32_t nv = nb * (F::kValues / 4);
            for (uint32_t v = threadIdx.x; v < nv; v += kGatherThreads) {
                const uint32_t blk = v / (F::kValues / 4), within = (v % (F::kValues / 4)) * 4;
                __stcs(out + (b0 * F::kValues) / 4 + v, decode4<KIND>(smem + blk * F::kBytes, (int)within));
            }
        }
    }
}

// Resident CTAs per SM of `kernel` (registers decide it): the gather grid
// is one full wave, so no CTA waits behind the rows of another.
// Cached per device and per kernel instantiation.
template <typename K>
int resident_ctas(const LaunchEnv& env, K kernel) {
    static DeviceKeyedValue cached;
    uint32_t n = 0;
    if (!cached.get(env.device, 0u, &n)) {
        int m = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&m, kernel, kGatherThreads, 0) != cudaSuccess || m < 1) m = 1;
        n = (uint32_t)m;
        cached.put(env.device, 0u, n);
    }
    return (int)n;
}

template <typename K>
cudaError_t launch_pair(const LaunchEnv& env, const GatherPlan& p, K kernel) {
    const uint64_t check_grid = (p.dst_rows + kGatherThreads - 1) / kGatherThreads;
    gather_check<<<(unsigned)(check_grid < (uint64_t)env.sm_count * 4 ? check_grid : (uint64_t)env.sm_count * 4),
                   kGatherThreads, 0, env.stream>>>(p);
    ++*env.launches;
    cudaError_t err = cudaGetLastError();
    if (err != cudaSuccess) return err;
    const uint64_t cap = (uint64_t)env.sm_count * resident_ctas(env, kernel);
    err = launch_dependent(kernel, dim3((unsigned)(p.dst_rows < cap ? p.dst_rows : cap)), dim3(kGatherThreads), 0,
                           env.stream, p);
    ++*env.launches;
    return err != cudaSuccess ? err : cudaGetLastError();
}

}  // namespace

cudaError_t launch_get_rows(const LaunchEnv& env, const GatherPlan& p) {
    cudaError_t err = cudaMemsetAsync(p.flag, 0, sizeof(uint32_t), env.stream);
    if (err != cudaSuccess) return err;
    switch (p.kind) {
    case kGatherF32: return launch_pair(env, p, gather_plain<kGatherF32>);
    case kGatherF32Bytes: return launch_pair(env, p, gather_plain<kGatherF32Bytes>);
    case kGatherF16: return launch_pair(env, p, gather_plain<kGatherF16>);
    case kGatherBF16: return launch_pair(env, p, gather_plain<kGatherBF16>);
    case kGatherQ4_0: return launch_pair(env, p, gather_quant<kGatherQ4_0>);
    case kGatherQ8_0: return launch_pair(env, p, gather_quant<kGatherQ8_0>);
    default: return launch_pair(env, p, gather_quant<kGatherQ4_K>);
    }
}

}  // namespace emel
