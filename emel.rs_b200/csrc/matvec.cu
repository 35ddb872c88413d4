// Vocabulary matvec + argmax (matmul.rs OpMulMatArgmax, F32): score of row
// r = sum over i of lhs[r, i] * rhs[i] as ONE sequential binary32 sum of
// separate products (the reference's accumulation order: a parallel or
// fused sum would change the bits), then the first row with the largest
// score (row 0 starts the scan; a later row needs a strictly larger score).
//
// One thread owns one row and keeps its accumulator across the whole row,
// so the order is exactly the reference's.  The rows reach the threads
// through shared memory: a persistent CTA of kMvRows threads walks tiles of
// kMvRows rows; each tile is consumed in chunks of kMvChunk columns, every
// chunk brought in by four 2-D TMA tensor loads (boxes of 32 columns x 128
// rows, 128-byte swizzle so that threads reading down a column hit distinct
// banks) plus one bulk copy of the rhs chunk, three stages deep on
// mbarriers, so the next chunks stream from HBM while the threads sum the
// current one.  A row whose plain-IEEE sum comes out NaN is summed again
// with the x86 NaN rules (rare).  Each CTA keeps its best (score, row); the
// last CTA to finish (atomic ticket) folds the partials.
//
// Rows whose length is not a multiple of 4 floats (the tensor map needs
// 16-byte row strides) take a plain kernel: one thread per row reading
// global memory.
#include <cuda.h>

#include "common.cuh"
#include "launch.hpp"
#include "pdl.cuh"
#include "tma.cuh"

namespace emel {

namespace {

constexpr int kMvRows = 128;                 // threads = rows per tile
constexpr int kMvChunk = 128;                // columns per chunk
constexpr int kMvBoxCols = 32;               // 128 bytes: the widest box the 128-byte swizzle allows
constexpr int kMvBoxes = kMvChunk / kMvBoxCols;
constexpr int kMvBoxBytes = kMvRows * kMvBoxCols * 4;
constexpr int kMvStageBytes = (kMvBoxes * kMvBoxBytes + kMvChunk * 4 + 1023) / 1024 * 1024;
constexpr int kMvStages = 3;                 // 3 x 65 KB of shared memory

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

struct MvPart {
    float v;
    int32_t i;
    uint32_t has;  // a comparable (non-NaN) score
    uint32_t pin;  // row 0 scored NaN: the scan never moves off it
};

// The reference's scan (row 0 starts it, a later row needs a strictly larger
// score) in a form that combines in any order: a NaN at row 0 pins the
// answer to row 0; otherwise the largest non-NaN score, earliest row on ties.
__device__ __forceinline__ MvPart mv_better(MvPart a, MvPart b) {
    if (a.pin) return a;
    if (b.pin) return b;
    if (!b.has) return a;
    if (!a.has) return b;
    if (b.v > a.v) return b;
    if (a.v > b.v) return a;
    return b.i < a.i ? b : a;
}

__device__ __forceinline__ float row_exact(const float* lhs, const float* rhs, uint64_t k, uint64_t row) {
    float acc = 0.0f;
    for (uint64_t i = 0; i < k; ++i) acc = f_add(acc, f_mul(lhs[row * k + i], rhs[i]));
    return acc;
}

__device__ __forceinline__ bool last_cta(unsigned* ticket) {
    __shared__ bool is_last;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) is_last = atomicAdd(ticket, 1u) == gridDim.x - 1;
    __syncthreads();
    return is_last;
}

__device__ void finish(const MvArgmaxPlan& p, MvPart best) {
    MvPart* parts = reinterpret_cast<MvPart*>(p.partials);
    if (threadIdx.x == 0) parts[blockIdx.x] = best;
    if (!last_cta(p.ticket)) return;
    if (threadIdx.x == 0) {
        __threadfence();
        MvPart total = parts[0];
        for (unsigned c = 1; c < gridDim.x; ++c) total = mv_better(total, parts[c]);
        *p.dst_value = total.v;
        *p.dst_index = total.i;
        *p.ticket = 0u;
    }
}

// rows owned by this CTA form a sequence of tiles t = blockIdx.x + j * gridDim.x
__global__ void __launch_bounds__(kMvRows, 1) mv_argmax_tma(const __grid_constant__ CUtensorMap lhs_map, MvArgmaxPlan p) {
    extern __shared__ unsigned char smem_raw[];
    __shared__ __align__(8) uint64_t full[kMvStages];
    __shared__ MvPart scratch[kMvRows];
    pdl_enter();
    // the 128-byte swizzle pattern repeats every 1024 bytes: align the stages to it
    unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    const uint64_t k = p.k, rows = p.rows;
    const uint64_t tiles = (rows + kMvRows - 1) / kMvRows;
    const uint64_t chunks = (k + kMvChunk - 1) / kMvChunk;
    const uint64_t mine = tiles > blockIdx.x ? (tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    const uint64_t steps = mine * chunks;  // (tile, chunk) pairs in order
    if (threadIdx.x == 0) {
        for (int s = 0; s < kMvStages; ++s) mbar_init(&full[s], 1);
        mbar_init_fence();
    }
    __syncthreads();
    auto issue = [&](uint64_t step) {  // one thread
        const uint64_t tile = blockIdx.x + (step / chunks) * gridDim.x, c = step % chunks;
        const int s = (int)(step % kMvStages);
        unsigned char* st = smem + (size_t)s * kMvStageBytes;
        const uint64_t c0 = c * kMvChunk;
        const uint32_t cols = (uint32_t)(k - c0 < (uint64_t)kMvChunk ? k - c0 : kMvChunk);
        const int boxes = (int)((cols + kMvBoxCols - 1) / kMvBoxCols);
        // a box counts its full size, rows past the end included (filled with zeros)
        mbar_expect_tx(&full[s], (uint32_t)boxes * kMvBoxBytes + cols * 4u);
        for (int bx = 0; bx < boxes; ++bx)
            tma_load_2d(st + bx * kMvBoxBytes, &lhs_map, (int)(c0 + bx * kMvBoxCols), (int)(tile * kMvRows), &full[s]);
        bulk_load(st + kMvBoxes * kMvBoxBytes, p.rhs + c0, cols * 4u, &full[s]);
    };
    if (threadIdx.x == 0)
        for (uint64_t j = 0; j < steps && j < (uint64_t)kMvStages; ++j) issue(j);
    MvPart best{0.0f, 0, 0u, 0u};
    float acc = 0.0f;
    const uint32_t sw = threadIdx.x & 7u;  // this row's swizzle phase
    for (uint64_t step = 0; step < steps; ++step) {
        const int s = (int)(step % kMvStages);
        const uint32_t parity = (uint32_t)((step / kMvStages) & 1u);
        const bool ok = mbar_wait(&full[s], parity);
        if (!__syncthreads_and(ok)) {
            if (threadIdx.x == 0) {
                atomicExch(p.fault, 1u);
                for (uint64_t j = step; j < steps && j < step + kMvStages; ++j)
                    mbar_wait(&full[j % kMvStages], (uint32_t)((j / kMvStages) & 1u));
            }
            // still take part in the ticket so the fold completes and re-arms it
            finish(p, MvPart{0.0f, 0, 0u, 0u});
            return;
        }
        const uint64_t tile = blockIdx.x + (step / chunks) * gridDim.x, c = step % chunks;
        const uint64_t row = tile * kMvRows + threadIdx.x;
        const unsigned char* st = smem + (size_t)s * kMvStageBytes;
        const uint64_t c0 = c * kMvChunk;
        const uint32_t n = (uint32_t)(k - c0 < (uint64_t)kMvChunk ? k - c0 : kMvChunk);
        if (row < rows) {
            const float4* v4 = reinterpret_cast<const float4*>(st + kMvBoxes * kMvBoxBytes);
            for (uint32_t q = 0; q < n / 4; ++q) {
                // 16-byte chunk (q % 8) of this row's 128-byte line in box q / 8, swizzled
                const float4 a = *reinterpret_cast<const float4*>(st + (q / 8) * kMvBoxBytes + threadIdx.x * 128u +
                                                                  (((q & 7u) ^ sw) << 4));
                const float4 v = v4[q];
                acc = __fadd_rn(acc, __fmul_rn(a.x, v.x));
                acc = __fadd_rn(acc, __fmul_rn(a.y, v.y));
                acc = __fadd_rn(acc, __fmul_rn(a.z, v.z));
                acc = __fadd_rn(acc, __fmul_rn(a.w, v.w));
            }
        }
        __syncthreads();  // every thread is done with this stage
        if (threadIdx.x == 0 && step + kMvStages < steps) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue(step + kMvStages);
        }
        if (c == chunks - 1) {
            // row complete
            if (row < rows) {
                float score = acc;
                if (is_nan(score)) score = row_exact(p.lhs, p.rhs, k, row);
                const bool nan = is_nan(score);
                const MvPart cand{score, (int32_t)row, nan ? 0u : 1u, (nan && row == 0) ? 1u : 0u};
                best = mv_better(best, cand);
            }
            acc = 0.0f;
        }
    }
    // fold the threads' candidates (the rule is order-free)
    scratch[threadIdx.x] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        MvPart b = scratch[0];
        for (int t = 1; t < kMvRows; ++t) b = mv_better(b, scratch[t]);
        scratch[0] = b;
    }
    __syncthreads();
    finish(p, scratch[0]);
}

// rows whose length is not whole 16-byte vectors: one thread per row
__global__ void __launch_bounds__(kMvRows) mv_argmax_plain(MvArgmaxPlan p) {
    __shared__ MvPart scratch[kMvRows];
    pdl_enter();
    MvPart best{0.0f, 0, 0u, 0u};
    for (uint64_t row = (uint64_t)blockIdx.x * kMvRows + threadIdx.x; row < p.rows;
         row += (uint64_t)gridDim.x * kMvRows) {
        float acc = 0.0f;
        for (uint64_t i = 0; i < p.k; ++i) acc = __fadd_rn(acc, __fmul_rn(p.lhs[row * p.k + i], p.rhs[i]));
        if (is_nan(acc)) acc = row_exact(p.lhs, p.rhs, p.k, row);
        const bool nan = is_nan(acc);
        best = mv_better(best, MvPart{acc, (int32_t)row, nan ? 0u : 1u, (nan && row == 0) ? 1u : 0u});
    }
    scratch[threadIdx.x] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        MvPart b = scratch[0];
        for (int t = 1; t < kMvRows; ++t) b = mv_better(b, scratch[t]);
        scratch[0] = b;
    }
    __syncthreads();
    finish(p, scratch[0]);
}

// ---- Q8_0 rows (matmul.rs OpMulMatArgmaxQ8_0) -------------------------------
// The rhs is quantized to Q8_0 in every CTA's shared memory (quantize_q8_0,
// matmul.rs:1629-1653: one warp per 32-value block, amax by a max-reduction,
// which is exact).  A warp owns 32 rows at a time.  For each row in turn the
// lanes form the block terms float(integer dot) * (d_lhs * d_rhs) of 128
// consecutive blocks (lane l: blocks l, l + 32, l + 64, l + 96, all loads
// issued first; dp4a on 32-bit words rebuilt from the 2-byte-aligned 34-byte
// blocks) into a padded shared tile [32 rows][129]; then lane r folds row r's
// terms in block order, one binary32 add each -- dot_q8_0's order
// (matmul.rs:1893-1910) -- so the 32 sequential sums run side by side.
constexpr int kQ8Threads = 128;
constexpr int kQ8Warps = kQ8Threads / 32;
constexpr int kQ8Chunk = 128;                       // blocks per pass
constexpr int kQ8TermStride = kQ8Chunk + 1;         // conflict-free column walk

__device__ __forceinline__ float q8_block_term(const uint8_t* rp, uint32_t b, const uint32_t* rq, const float* rd,
                                               const uint32_t (&w)[9], bool odd) {
    const uint32_t dbits = odd ? (w[0] >> 16) : (w[0] & 0xffffu);
    const uint32_t* r = rq + b * 9;
    int integer = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint32_t qw = odd ? w[j + 1] : __byte_perm(w[j], w[j + 1], 0x5432);
        integer = __dp4a((int)qw, (int)r[j], integer);
    }
    return __fmul_rn((float)integer, __fmul_rn(f16_bits_to_f32((uint16_t)dbits), rd[b]));
}

__global__ void __launch_bounds__(kQ8Threads) mv_argmax_q8_0(MvArgmaxPlan p, const uint8_t* lhs) {
    extern __shared__ __align__(16) uint32_t q8_smem[];
    __shared__ MvPart warp_best[kQ8Warps];
    const uint32_t blocks = (uint32_t)(p.k / 32);
    uint32_t* rq = q8_smem;                                            // [blocks][9]: 8 words of quants + pad
    float* rd = reinterpret_cast<float*>(q8_smem + blocks * 9);        // [blocks]: rhs scales
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float* terms = rd + blocks + warp * 32 * kQ8TermStride;            // this warp's [32][129] tile
    pdl_enter();
    for (uint32_t b = warp; b < blocks; b += kQ8Warps) {
        const float x = p.rhs[(uint64_t)b * 32 + lane];
        float amax = fabsf(x);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        const float scale = __fdiv_rn(amax, 127.0f);
        const float inverse = scale == 0.0f ? 0.0f : __fdiv_rn(1.0f, scale);
        float q = roundf(__fmul_rn(x, inverse));
        q = is_nan(q) ? 0.0f : fminf(fmaxf(q, -127.0f), 127.0f);
        reinterpret_cast<int8_t*>(rq + b * 9)[lane] = (int8_t)(int)q;
        if (lane == 0) rd[b] = f16_bits_to_f32(f32_to_f16_bits(scale));
    }
    __syncthreads();
    const uint64_t row_bytes = (uint64_t)blocks * 34;
    MvPart best{0.0f, 0, 0u, 0u};
    for (uint64_t g0 = ((uint64_t)blockIdx.x * kQ8Warps + warp) * 32; g0 < p.rows;
         g0 += (uint64_t)gridDim.x * kQ8Warps * 32) {
        const uint32_t nrows = p.rows - g0 < 32u ? (uint32_t)(p.rows - g0) : 32u;
        float sum = 0.0f;  // lane r: row g0 + r
        for (uint32_t b0 = 0; b0 < blocks; b0 += kQ8Chunk) {
            for (uint32_t r = 0; r < nrows; ++r) {
                const uint8_t* rp = lhs + (g0 + r) * row_bytes;
                uint32_t w[4][9];
                bool odd[4];
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const uint32_t b = b0 + 32 * c + lane;
                    odd[c] = false;
                    if (b < blocks) {
                        const uint64_t off = (uint64_t)b * 34;
                        odd[c] = ((uintptr_t)(rp + off) & 3u) != 0;  // block starts 2 bytes into a word
                        const uint32_t* wp = reinterpret_cast<const uint32_t*>(rp + off - (odd[c] ? 2 : 0));
#pragma unroll
                        for (int j = 0; j < 8; ++j) w[c][j] = __ldg(wp + j);
                        // the last word: whole when the block ends on it, else its first half
                        w[c][8] = odd[c] ? __ldg(wp + 8) : (uint32_t)__ldg(reinterpret_cast<const uint16_t*>(wp + 8));
                    }
                }
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const uint32_t b = b0 + 32 * c + lane;
                    if (b < blocks) terms[r * kQ8TermStride + 32 * c + lane] = q8_block_term(rp, b, rq, rd, w[c], odd[c]);
                }
            }
            __syncwarp();
            if ((uint32_t)lane < nrows) {
                const uint32_t n = blocks - b0 < (uint32_t)kQ8Chunk ? blocks - b0 : (uint32_t)kQ8Chunk;
                const float* t = terms + lane * kQ8TermStride;
                uint32_t j = 0;
                for (; j + 8 <= n; j += 8) {
                    float v[8];
#pragma unroll
                    for (int u = 0; u < 8; ++u) v[u] = t[j + u];
#pragma unroll
                    for (int u = 0; u < 8; ++u) sum = __fadd_rn(sum, v[u]);
                }
                for (; j < n; ++j) sum = __fadd_rn(sum, t[j]);
            }
            __syncwarp();
        }
        if ((uint32_t)lane < nrows) {
            const uint64_t row = g0 + lane;
            const bool nan = is_nan(sum);
            best = mv_better(best, MvPart{sum, (int32_t)row, nan ? 0u : 1u, (nan && row == 0) ? 1u : 0u});
        }
    }
    // order-free fold of the lanes' and warps' candidates
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        MvPart other;
        other.v = __shfl_xor_sync(0xffffffffu, best.v, o);
        other.i = __shfl_xor_sync(0xffffffffu, best.i, o);
        other.has = __shfl_xor_sync(0xffffffffu, best.has, o);
        other.pin = __shfl_xor_sync(0xffffffffu, best.pin, o);
        best = mv_better(best, other);
    }
    if (lane == 0) warp_best[warp] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        MvPart b = warp_best[0];
        for (int w = 1; w < kQ8Warps; ++w) b = mv_better(b, warp_best[w]);
        warp_best[0] = b;
    }
    __syncthreads();
    finish(p, warp_best[0]);
}

}  // namespace

namespace {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled from the driver the runtime already loaded
EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = nullptr;
    if (fn == nullptr) {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(f);
    }
    return fn;
}

}  // namespace

cudaError_t launch_mul_mat_argmax(const LaunchEnv& env, const MvArgmaxPlan& p) {
    const uint64_t tiles = (p.rows + kMvRows - 1) / kMvRows;
    cudaError_t err;
    bool tma = p.vec && p.k <= 0xffffffffull && p.rows <= 0x7fffffffull;
    CUtensorMap map;
    if (tma) {
        // lhs as a 2-D tensor: x = column (k), y = row; boxes of 32 columns x 128 rows
        const EncodeTiledFn enc = encode_tiled();
        const cuuint64_t dims[2] = {(cuuint64_t)p.k, (cuuint64_t)p.rows};
        const cuuint64_t strides[1] = {(cuuint64_t)p.k * 4};
        const cuuint32_t box[2] = {(cuuint32_t)kMvBoxCols, (cuuint32_t)kMvRows};
        const cuuint32_t estr[2] = {1, 1};
        tma = enc != nullptr &&
              enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(p.lhs), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    }
    if (tma) {
        static int configured_device_mask = 0;
        const int bit = env.device < 31 ? (1 << env.device) : 0;
        const int smem = kMvStages * kMvStageBytes + 1024;  // + alignment slack
        if (!(configured_device_mask & bit)) {
            err = cudaFuncSetAttribute(mv_argmax_tma, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            if (err != cudaSuccess) return err;
            configured_device_mask |= bit;
        }
        const uint64_t cap = (uint64_t)env.sm_count;  // one CTA per SM: its stages fill shared memory
        err = launch_dependent(mv_argmax_tma, dim3((unsigned)(tiles < cap ? tiles : cap)), dim3(kMvRows),
                               (size_t)smem, env.stream, map, p);
    } else {
        const uint64_t cap = (uint64_t)env.sm_count * 8;
        err = launch_dependent(mv_argmax_plain, dim3((unsigned)(tiles < cap ? tiles : cap)), dim3(kMvRows), 0,
                               env.stream, p);
    }
    ++*env.launches;
    return err != cudaSuccess ? err : cudaGetLastError();
}

cudaError_t launch_mul_mat_argmax_q8_0(const LaunchEnv& env, const MvArgmaxPlan& p, const uint8_t* lhs) {
    const uint64_t groups = (p.rows + kQ8Warps * 32 - 1) / (kQ8Warps * 32);
    const uint64_t cap = (uint64_t)env.sm_count * 3;
    const size_t smem = (size_t)(p.k / 32) * (9 * 4 + 4) + (size_t)kQ8Warps * 32 * kQ8TermStride * 4;
    static int configured_device_mask = 0;
    const int bit = env.device < 31 ? (1 << env.device) : 0;
    if (!(configured_device_mask & bit)) {
        const cudaError_t e =
            cudaFuncSetAttribute(mv_argmax_q8_0, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 1024 * 40 + kQ8Warps * 32 * kQ8TermStride * 4);
        if (e != cudaSuccess) return e;
        configured_device_mask |= bit;
    }
    const cudaError_t err = launch_dependent(mv_argmax_q8_0, dim3((unsigned)(groups < cap ? groups : cap)),
                                             dim3(kQ8Threads), smem, env.stream, p, lhs);
    ++*env.launches;
    return err != cudaSuccess ? err : cudaGetLastError();
}

}  // namespace emel
