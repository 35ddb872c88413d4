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

__device__ __forceinline__ MvPart mv_shfl(MvPart a, int o) {
    MvPart b;
    b.v = __shfl_xor_sync(0xffffffffu, a.v, o);
    b.i = __shfl_xor_sync(0xffffffffu, a.i, o);
    b.has = __shfl_xor_sync(0xffffffffu, a.has, o);
    b.pin = __shfl_xor_sync(0xffffffffu, a.pin, o);
    return b;
}

// Stores the CTA's partial; the last CTA folds all partials (mv_better is a
// maximum under a total order -- only the partial holding row 0 can pin --
// so every thread folds a strided share and the shares combine in any order).
__device__ void finish(const MvArgmaxPlan& p, MvPart best) {
    __shared__ MvPart fold[32];
    MvPart* parts = reinterpret_cast<MvPart*>(p.partials);
    if (threadIdx.x == 0) parts[blockIdx.x] = best;
    if (!last_cta(p.ticket)) return;
    __threadfence();
    MvPart t{0.0f, 0, 0u, 0u};
    for (unsigned c = threadIdx.x; c < gridDim.x; c += blockDim.x) {
        const int4 w = __ldcg(reinterpret_cast<const int4*>(parts + c));
        t = mv_better(t, MvPart{__int_as_float(w.x), w.y, (uint32_t)w.z, (uint32_t)w.w});
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t = mv_better(t, mv_shfl(t, o));
    if ((threadIdx.x & 31) == 0) fold[threadIdx.x >> 5] = t;
    __syncthreads();
    if (threadIdx.x == 0) {
        MvPart total = fold[0];
        for (unsigned w = 1; w < blockDim.x / 32; ++w) total = mv_better(total, fold[w]);
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

// ---- packed rows (matmul.rs OpMulMatArgmaxQ4_0 / Q4_1 / Q5_0 / Q8_0) ---------
// The rhs is quantized to Q8_0 in every CTA's shared memory (quantize_q8_0,
// matmul.rs:1629-1653: one warp per 32-value block, amax by a max-reduction,
// which is exact; Q4_1 also keeps each block's quant sum).  A warp owns 32
// rows at a time.  For each row in turn the lanes form the block terms of 128
// consecutive blocks (lane l: blocks l, l + 32, l + 64, l + 96; the next
// row's loads are issued before this row's terms are formed) into a padded
// shared tile [32 rows][129]; then lane r folds
// row r's terms in block order, one binary32 add each -- the order of
// dot_q4_0 / dot_q4_1 / dot_q5_0 / dot_q8_0 (matmul.rs:1804-1910) -- so the
// 32 sequential sums run side by side.  A block is read as aligned 32-bit
// words (predicated so no byte past it is touched), realigned when it starts
// 2 bytes into a word, and its quants rebuilt as 8 words of 4 signed bytes in
// the rhs order (positions 0-15 from the low nibbles, 16-31 from the high
// ones) for dp4a.
constexpr int kQ8Threads = 128;
constexpr int kQ8Warps = kQ8Threads / 32;
constexpr int kQ8Chunk = 128;                       // blocks per pass
constexpr int kQ8TermStride = kQ8Chunk + 1;         // conflict-free column walk

template <int CODE>
struct PackedFmt;
template <>
struct PackedFmt<kDtypeQ4_0> { static constexpr int kBytes = 18; };
template <>
struct PackedFmt<kDtypeQ4_1> { static constexpr int kBytes = 20; };
template <>
struct PackedFmt<kDtypeQ5_0> { static constexpr int kBytes = 22; };
template <>
struct PackedFmt<kDtypeQ8_0> { static constexpr int kBytes = 34; };
template <>
struct PackedFmt<kDtypeQ6_K> { static constexpr int kBytes = 210; };
template <>
struct PackedFmt<kDtypeQ3_K> { static constexpr int kBytes = 110; };

// byte i of a nibble bit pattern (4 bits) moved to bit 4 of byte i
__device__ __forceinline__ uint32_t q5_spread(uint32_t b4) {
    return ((b4 & 1u) << 4) | ((b4 & 2u) << 11) | ((b4 & 4u) << 18) | ((b4 & 8u) << 25);
}

template <int CODE>
struct PackedBlock {
    static constexpr int BB = PackedFmt<CODE>::kBytes;
    static constexpr int NW = (BB + 2 + 3) / 4;  // words a block can touch
    uint32_t w[NW];
    bool odd;

    // SHARED: `blk` points into a shared-memory staging window
    template <bool SHARED = false>
    __device__ __forceinline__ void load(const uint8_t* blk) {
        odd = ((uintptr_t)blk & 3u) != 0;  // starts 2 bytes into a word
        const uint32_t* wp = reinterpret_cast<const uint32_t*>(blk - (odd ? 2 : 0));
        const int end = BB + (odd ? 2 : 0);  // bytes of the aligned window in use
#pragma unroll
        for (int j = 0; j < NW; ++j) {
            if (4 * j + 4 <= end)
                w[j] = SHARED ? wp[j] : __ldg(wp + j);
            else if (4 * j + 2 <= end)
                w[j] = SHARED ? (uint32_t)*reinterpret_cast<const uint16_t*>(wp + j)
                              : (uint32_t)__ldg(reinterpret_cast<const uint16_t*>(wp + j));
            else
                w[j] = 0u;
        }
    }
    // word j of the block's bytes (block byte 4j at its low byte)
    __device__ __forceinline__ uint32_t word(int j) const {
        if (j + 1 < NW) return odd ? __byte_perm(w[j], w[j + 1], 0x5432) : w[j];
        return odd ? (w[j] >> 16) : w[j];
    }
    // the 4 bytes starting at block byte 4j + 2
    __device__ __forceinline__ uint32_t word2(int j) const { return __byte_perm(word(j), word(j + 1), 0x5432); }
};

template <int CODE>
__device__ __forceinline__ float packed_block_term(const PackedBlock<CODE>& k, uint32_t b, const uint32_t* rq,
                                                   const float* rd, const int* rs) {
    const uint32_t* r = rq + b * 9;
    const uint32_t w0 = k.word(0);
    const float dl = f16_bits_to_f32((uint16_t)(w0 & 0xffffu));
    int integer = 0;
    if constexpr (CODE == kDtypeQ8_0) {
#pragma unroll
        for (int j = 0; j < 8; ++j) integer = __dp4a((int)k.word2(j), (int)r[j], integer);
    } else if constexpr (CODE == kDtypeQ4_0) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t pk = k.word2(j);
            integer = __dp4a((int)__vsub4(pk & 0x0f0f0f0fu, 0x08080808u), (int)r[j], integer);
            integer = __dp4a((int)__vsub4((pk >> 4) & 0x0f0f0f0fu, 0x08080808u), (int)r[4 + j], integer);
        }
    } else if constexpr (CODE == kDtypeQ5_0) {
        const uint32_t qh = k.word2(0);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t pk = __byte_perm(k.word(j + 1), k.word(j + 2), 0x5432);  // bytes 6 + 4j ..
            const uint32_t lo = (pk & 0x0f0f0f0fu) | q5_spread((qh >> (4 * j)) & 0xfu);
            const uint32_t hi = ((pk >> 4) & 0x0f0f0f0fu) | q5_spread((qh >> (16 + 4 * j)) & 0xfu);
            integer = __dp4a((int)__vsub4(lo, 0x10101010u), (int)r[j], integer);
            integer = __dp4a((int)__vsub4(hi, 0x10101010u), (int)r[4 + j], integer);
        }
    } else {  // Q4_1: unsigned nibbles, min term (matmul.rs:1832-1858)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t pk = k.word(j + 1);  // bytes 4 + 4j ..
            integer = __dp4a((int)(pk & 0x0f0f0f0fu), (int)r[j], integer);
            integer = __dp4a((int)((pk >> 4) & 0x0f0f0f0fu), (int)r[4 + j], integer);
        }
        const float ml = f16_bits_to_f32((uint16_t)(w0 >> 16));
        return __fmul_rn(rd[b], __fadd_rn(__fmul_rn(dl, (float)integer), __fmul_rn(ml, (float)rs[b])));
    }
    return __fmul_rn((float)integer, __fmul_rn(dl, rd[b]));
}

template <int CODE>
__global__ void __launch_bounds__(kQ8Threads, 3) mv_argmax_packed(MvArgmaxPlan p, const uint8_t* lhs) {
    extern __shared__ __align__(16) uint32_t q8_smem[];
    __shared__ MvPart warp_best[kQ8Warps];
    constexpr int BB = PackedFmt<CODE>::kBytes;
    const uint32_t blocks = (uint32_t)(p.k / 32);
    uint32_t* rq = q8_smem;                                            // [blocks][9]: 8 words of quants + pad
    float* rd = reinterpret_cast<float*>(q8_smem + blocks * 9);        // [blocks]: rhs scales
    int* rs = reinterpret_cast<int*>(rd + blocks);                     // [blocks]: rhs quant sums
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float* terms = reinterpret_cast<float*>(rs + blocks) + warp * 32 * kQ8TermStride;  // [32][129]
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
        const int qi = (int)q;
        reinterpret_cast<int8_t*>(rq + b * 9)[lane] = (int8_t)qi;
        int qsum = qi;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) qsum += __shfl_xor_sync(0xffffffffu, qsum, o);
        if (lane == 0) {
            rd[b] = f16_bits_to_f32(f32_to_f16_bits(scale));
            rs[b] = qsum;
        }
    }
    __syncthreads();
    const uint64_t row_bytes = (uint64_t)blocks * BB;
    MvPart best{0.0f, 0, 0u, 0u};
    for (uint64_t g0 = ((uint64_t)blockIdx.x * kQ8Warps + warp) * 32; g0 < p.rows;
         g0 += (uint64_t)gridDim.x * kQ8Warps * 32) {
        const uint32_t nrows = p.rows - g0 < 32u ? (uint32_t)(p.rows - g0) : 32u;
        float sum = 0.0f;  // lane r: row g0 + r
        for (uint32_t b0 = 0; b0 < blocks; b0 += kQ8Chunk) {
            // row r's blocks are in registers while row r + 1's loads are in flight
            PackedBlock<CODE> cur[4], nxt[4];
            const auto load_row = [&](PackedBlock<CODE>(&dst)[4], uint32_t r) {
                const uint8_t* rp = lhs + (g0 + r) * row_bytes;
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const uint32_t b = b0 + 32 * c + lane;
                    if (b < blocks) dst[c].load(rp + (uint64_t)b * BB);
                }
            };
            load_row(cur, 0);
            for (uint32_t r = 0; r < nrows; ++r) {
                if (r + 1 < nrows) load_row(nxt, r + 1);
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    const uint32_t b = b0 + 32 * c + lane;
                    if (b < blocks) terms[r * kQ8TermStride + 32 * c + lane] = packed_block_term<CODE>(cur[c], b, rq, rd, rs);
                }
#pragma unroll
                for (int c = 0; c < 4; ++c) cur[c] = nxt[c];
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

template <int CODE>
cudaError_t launch_packed(const LaunchEnv& env, const MvArgmaxPlan& p, const uint8_t* lhs) {
    const uint64_t groups = (p.rows + kQ8Warps * 32 - 1) / (kQ8Warps * 32);
    const uint64_t cap = (uint64_t)env.sm_count * 3;
    const size_t table = (size_t)kQ8Warps * 32 * kQ8TermStride * 4;
    const size_t smem = (size_t)(p.k / 32) * (9 * 4 + 4 + 4) + table;
    static DeviceFlags configured;
    if (!configured.done(env.device)) {
        const cudaError_t e = cudaFuncSetAttribute(mv_argmax_packed<CODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   (int)(1024 * (9 * 4 + 4 + 4) + table));
        if (e != cudaSuccess) return e;
        configured.mark(env.device);
    }
    return launch_dependent(mv_argmax_packed<CODE>, dim3((unsigned)(groups < cap ? groups : cap)), dim3(kQ8Threads),
                            smem, env.stream, p, lhs);
}

// ---- K-quant rows (matmul.rs OpMulMatArgmaxQ2K / Q3K / Q4K / Q6K) ---------------
// quantize_q8_k (matmul.rs:1703-1745) per 256-value block in every CTA's
// shared memory, stored for dp4a: word [b][g][j] holds the quants at
// positions 32g + j, + 8, + 16, + 24 of block b -- the positions dot_q4_k
// (matmul.rs:2040-2114) adds into lane sum j of group g.  A warp owns 32
// rows; its lanes take (row, block) items of a 16-block chunk, each forming
// that block's eight lane terms d * float(acc[j]) and its minimum term
// dmin * float(min sum) into a padded shared tile; lane r then folds row r
// block by block (eight lane sums and the running total, the reference's
// order) and adds the lane sums to the total after the last block.
constexpr int kKThreads = 128;
constexpr int kKWarps = kKThreads / 32;
constexpr int kKTerms = 9;                        // eight lane terms + the minimum term

// Staging window of one block: the aligned words that hold its BB bytes
// (a block may start 2 bytes into a word), at an odd word stride per row so
// the lanes' word reads fall in distinct banks.
template <int CODE>
struct KWindow {
    static constexpr int BB = CODE == kDtypeQ2_K ? 84 : CODE == kDtypeQ3_K ? 110 : CODE == kDtypeQ4_K ? 144 : 210;
    static constexpr int NW = (BB + 2 + 3) / 4;
    static constexpr int SW = NW | 1;
    // 16-byte staging (16-byte aligned rows): the 16-byte chunks that hold
    // the block's bytes, at an odd number of chunks per row
    static constexpr int NC = (15 + BB + 15) / 16;
    static constexpr int SW16 = 4 * (NC | 1);
    static constexpr int SWM = SW > SW16 ? SW : SW16;
};

__device__ __forceinline__ int32_t q8k_nearest(float v) {
    return (int32_t)(__float_as_uint(__fadd_rn(v, 12582912.0f)) & 0x007fffffu) - 0x00400000;
}

// Q4_K term: eight lane terms d * float(acc[j]) and the minimum term.
// ALIGNED16: w is 16-byte aligned (the window is read as nine 16-byte words).
template <bool ALIGNED16 = false>
__device__ __forceinline__ void q4k_block_terms(const uint32_t* w, const uint32_t* r4, const int* bs, float rdb,
                                                float* o) {
    uint32_t W[36];
    if constexpr (ALIGNED16) {
#pragma unroll
        for (int i = 0; i < 9; ++i) {
            const uint4 q = reinterpret_cast<const uint4*>(w)[i];
            W[4 * i] = q.x;
            W[4 * i + 1] = q.y;
            W[4 * i + 2] = q.z;
            W[4 * i + 3] = q.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 36; ++i) W[i] = w[i];  // shared-memory window
    }
    // scales / minimums (dot_q4_k's unpacking)
    const uint32_t s0 = W[1], s1 = W[2], s2 = W[3];
    uint32_t sc[8], mn[8];
#pragma unroll
    for (int l = 0; l < 4; ++l) {
        const uint32_t a = (s0 >> (8 * l)) & 0xffu, bb = (s1 >> (8 * l)) & 0xffu, c = (s2 >> (8 * l)) & 0xffu;
        sc[l] = a & 0x3fu;
        sc[4 + l] = (c & 0x0fu) | ((a >> 6) << 4);
        mn[l] = bb & 0x3fu;
        mn[4 + l] = (c >> 4) | ((bb >> 6) << 4);
    }
    int min_sum = 0;
#pragma unroll
    for (int h = 0; h < 16; ++h) min_sum += bs[h] * (int)mn[h >> 1];
    int acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
    for (int gg = 0; gg < 8; ++gg) {
        const int h = gg >> 1;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int k0 = 4 + 8 * h + (j >> 2), bt = j & 3;
            const uint32_t sel = (uint32_t)bt | ((uint32_t)(bt + 4) << 4);
            const uint32_t lo = __byte_perm(W[k0], W[k0 + 2], sel);
            const uint32_t hi = __byte_perm(W[k0 + 4], W[k0 + 6], sel);
            uint32_t v = __byte_perm(lo, hi, 0x5410);
            v = (gg & 1) ? ((v >> 4) & 0x0f0f0f0fu) : (v & 0x0f0f0f0fu);
            acc[j] += (int)sc[gg] * __dp4a((int)v, (int)r4[gg * 8 + j], 0);
        }
    }
    const float dd = __fmul_rn(f16_bits_to_f32((uint16_t)(W[0] & 0xffffu)), rdb);
    const float dm = __fmul_rn(f16_bits_to_f32((uint16_t)(W[0] >> 16)), rdb);
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = __fmul_rn(dd, (float)acc[j]);
    o[8] = __fmul_rn(dm, (float)min_sum);
}

// Q6_K term (dot_q6_k, matmul.rs:2117-2190): eight lane terms
// (d_rhs * d) * float(sums[j]); decoded 4 values at a time with byte-SIMD
// ops, and each lane sum's two positions of a 16-value group paired for dp4a.
__device__ __forceinline__ void q6k_block_terms(const uint8_t* blk_ptr, const uint32_t* r4, float rdb, float* o) {
    PackedBlock<kDtypeQ6_K> blk;
    blk.load<true>(blk_ptr);
    int sums[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
    for (int g = 0; g < 16; ++g) {
        const int c = g >> 3, sgrp = (g & 7) >> 1, i0 = 16 * (g & 1);
        const int scale = (int)(int8_t)((blk.word(48 + (g >> 2)) >> (8 * (g & 3))) & 0xffu);
        uint32_t D[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int i = i0 + 4 * k;
            const uint32_t ql = blk.word(c * 16 + ((sgrp & 1) ? 8 : 0) + (i >> 2));
            const uint32_t nib = (sgrp < 2) ? (ql & 0x0f0f0f0fu) : ((ql >> 4) & 0x0f0f0f0fu);
            const uint32_t qh = blk.word(32 + c * 8 + (i >> 2));
            const uint32_t hb = ((qh >> (2 * sgrp)) & 0x03030303u) << 4;
            D[k] = __vsub4(nib | hb, 0x20202020u);
        }
        const uint32_t* R = r4 + 4 * g;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int a = j < 4 ? 0 : 1, bt = j & 3;
            const uint32_t sel = (uint32_t)bt | ((uint32_t)(bt + 4) << 4);
            const uint32_t x = __byte_perm(D[a], D[a + 2], sel) & 0xffffu;
            const uint32_t y = __byte_perm(R[a], R[a + 2], sel);
            sums[j] += scale * __dp4a((int)x, (int)y, 0);
        }
    }
    const float sc = __fmul_rn(rdb, f16_bits_to_f32((uint16_t)(blk.word(52) & 0xffffu)));
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = __fmul_rn(sc, (float)sums[j]);
    o[8] = 0.0f;
}

// Q2_K term (dot_q2_k, matmul.rs:1918-1962): one term per block,
// (d_rhs * d) * float(sum) - (d_rhs * dmin) * float(minimum sum), in o[8].
__device__ __forceinline__ void q2k_block_terms(const uint32_t* w, const uint32_t* r4, const int* bs, float rdb,
                                                float* o) {
    uint32_t W[21];
#pragma unroll
    for (int i = 0; i < 21; ++i) W[i] = w[i];  // shared-memory window
    int sum_mins = 0;
#pragma unroll
    for (int g = 0; g < 16; ++g) sum_mins += bs[g] * (int)((W[g >> 2] >> (8 * (g & 3) + 4)) & 0x0fu);
    int sum = 0;
#pragma unroll
    for (int c = 0; c < 2; ++c) {
#pragma unroll
        for (int t = 0; t < 4; ++t) {
            const int si = 8 * c + 2 * t;
            const int s0 = (int)((W[si >> 2] >> (8 * (si & 3))) & 0x0fu);
            const int s1 = (int)((W[(si + 1) >> 2] >> (8 * ((si + 1) & 3))) & 0x0fu);
            int low = 0, high = 0;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                low = __dp4a((int)((W[4 + 8 * c + k] >> (2 * t)) & 0x03030303u), (int)r4[32 * c + 8 * t + k], low);
                high = __dp4a((int)((W[8 + 8 * c + k] >> (2 * t)) & 0x03030303u), (int)r4[32 * c + 8 * t + 4 + k], high);
            }
            sum += s0 * low + s1 * high;
        }
    }
    const float d_all = __fmul_rn(rdb, f16_bits_to_f32((uint16_t)(W[20] & 0xffffu)));
    const float d_min = __fmul_rn(rdb, f16_bits_to_f32((uint16_t)(W[20] >> 16)));
    o[8] = __fsub_rn(__fmul_rn(d_all, (float)sum), __fmul_rn(d_min, (float)sum_mins));
}

// Q3_K term (unpack_q3_scales and dot_q3_k, matmul.rs:1964-2036): eight lane
// terms (d_rhs * d) * float(acc[j]); values (2 bits | 4 where the hmask bit
// is set) - 4 decoded four at a time, each lane sum's two positions of a
// 16-value group paired for dp4a.
__device__ __forceinline__ void q3k_block_terms(const uint8_t* blk_ptr, const uint32_t* r4, float rdb, float* o) {
    PackedBlock<kDtypeQ3_K> blk;
    blk.load<true>(blk_ptr);
    uint32_t a0 = blk.word(24), a1 = blk.word(25);
    const uint32_t tmp = blk.word(26);
    const uint32_t a2 = ((a0 >> 4) & 0x0f0f0f0fu) | (((tmp >> 4) & 0x03030303u) << 4);
    const uint32_t a3 = ((a1 >> 4) & 0x0f0f0f0fu) | (((tmp >> 6) & 0x03030303u) << 4);
    a0 = (a0 & 0x0f0f0f0fu) | ((tmp & 0x03030303u) << 4);
    a1 = (a1 & 0x0f0f0f0fu) | (((tmp >> 2) & 0x03030303u) << 4);
    const uint32_t aux[4] = {a0, a1, a2, a3};
    int acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
    for (int g = 0; g < 16; ++g) {
        const int scale = (int)(int8_t)(uint8_t)(((aux[g >> 2] >> (8 * (g & 3))) & 0xffu) - 32u);
        const int qbase = (g >> 3) * 32, half = (g & 1) * 16, shift = ((g >> 1) & 3) * 2, mbit = g >> 1;
        uint32_t D[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t qw = (blk.word(8 + (qbase + half) / 4 + k) >> shift) & 0x03030303u;
            const uint32_t hb = ((blk.word(half / 4 + k) >> mbit) & 0x01010101u) << 2;
            D[k] = __vsub4(qw | hb, 0x04040404u);
        }
        const uint32_t* R = r4 + 4 * g;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int a = j < 4 ? 0 : 1, bt = j & 3;
            const uint32_t sel = (uint32_t)bt | ((uint32_t)(bt + 4) << 4);
            const uint32_t x = __byte_perm(D[a], D[a + 2], sel) & 0xffffu;
            const uint32_t y = __byte_perm(R[a], R[a + 2], sel);
            acc[j] += scale * __dp4a((int)x, (int)y, 0);
        }
    }
    const float sc = __fmul_rn(rdb, f16_bits_to_f32((uint16_t)(blk.word(27) & 0xffffu)));
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j] = __fmul_rn(sc, (float)acc[j]);
    o[8] = 0.0f;
}

// The rhs quantized to Q8_K blocks (quantize_row_q8_k, the reference's
// rhs step of dot_q*_k) into shared memory: rq [blocks][64] quant words in
// the order the format's decode reads them, rd [blocks] scales, rb
// [blocks][16] sums of each 16-value group.  One warp per block.
// qs / bsz: words of rq and ints of rb per block (64 and 16 packed; a
// padded stride puts different blocks in different banks when lanes read
// different blocks at once).
template <int CODE>
__device__ __forceinline__ void quantize_rhs_q8k(const MvArgmaxPlan& p, uint32_t blocks, uint32_t* rq, float* rd,
                                                 int* rb, int nwarps, uint32_t qs = 64, uint32_t bsz = 16) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (uint32_t b = warp; b < blocks; b += (uint32_t)nwarps) {
        // lane l holds positions 8l .. 8l + 7
        float x[8];
        float absolute = 0.0f, maximum = 0.0f;
        int first = 256;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            x[i] = p.rhs[(uint64_t)b * 256 + lane * 8 + i];
            if (fabsf(x[i]) > absolute) {
                absolute = fabsf(x[i]);
                maximum = x[i];
                first = lane * 8 + i;
            }
        }
        // the first position of the largest magnitude (a strict '>' scan)
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float oa = __shfl_xor_sync(0xffffffffu, absolute, o);
            const float om = __shfl_xor_sync(0xffffffffu, maximum, o);
            const int of = __shfl_xor_sync(0xffffffffu, first, o);
            if (oa > absolute || (oa == absolute && of < first)) {
                absolute = oa;
                maximum = om;
                first = of;
            }
        }
        int8_t q[8];
        float d = 0.0f;
        if (absolute == 0.0f) {
#pragma unroll
            for (int i = 0; i < 8; ++i) q[i] = 0;
        } else {
            const float inverse = __fdiv_rn(-127.0f, maximum);
            d = __fdiv_rn(1.0f, inverse);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int32_t v = q8k_nearest(__fmul_rn(inverse, x[i]));
                q[i] = (int8_t)(v < 127 ? v : 127);
            }
        }
        if constexpr (CODE == kDtypeQ4_K) {
            // position 8 * lane + i = 32 g + 8 t + i: group g = lane / 4, t = lane % 4
            const int g = lane >> 2, t = lane & 3;
            int8_t* words = reinterpret_cast<int8_t*>(rq + b * qs + g * 8);
#pragma unroll
            for (int i = 0; i < 8; ++i) words[i * 4 + t] = q[i];
        } else {
            int8_t* bytes = reinterpret_cast<int8_t*>(rq + b * qs);  // natural order
#pragma unroll
            for (int i = 0; i < 8; ++i) bytes[lane * 8 + i] = q[i];
        }
        int gsum = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) gsum += q[i];
        gsum += __shfl_xor_sync(0xffffffffu, gsum, 1);  // lanes 2h, 2h + 1 hold group h of 16
        if ((lane & 1) == 0) rb[b * bsz + (lane >> 1)] = (int)(int16_t)gsum;
        if (lane == 0) rd[b] = d;
    }
}

template <int CODE>
__global__ void __launch_bounds__(kKThreads, CODE == kDtypeQ6_K || CODE == kDtypeQ3_K ? 6 : 8)
    mv_argmax_k(MvArgmaxPlan p, const uint8_t* lhs) {
    extern __shared__ __align__(16) uint32_t k_smem[];
    __shared__ MvPart warp_best[kKWarps];
    const uint32_t blocks = (uint32_t)(p.k / 256);
    uint32_t* rq = k_smem;                                           // [blocks][8 groups][8 lanes] quant words
    float* rd = reinterpret_cast<float*>(rq + blocks * 64);          // [blocks] scales
    int* rb = reinterpret_cast<int*>(rd + blocks);                   // [blocks][16] group sums
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    using KW = KWindow<CODE>;
    // [2][32 rows][SWM] staging windows, 16-byte aligned
    uint32_t* stage = k_smem + ((blocks * 81u + 3u) & ~3u) + warp * 2 * 32 * KW::SWM;
    pdl_enter();
    quantize_rhs_q8k<CODE>(p, blocks, rq, rd, rb, kKWarps);
    __syncthreads();
    constexpr uint64_t BB = KW::BB;
    const uint64_t row_bytes = (uint64_t)blocks * BB;
    // 16-byte aligned rows: block b sits at the same 16-byte offset in every
    // row and every 16-byte chunk holding its bytes lies inside the tensor
    const bool v16 = ((reinterpret_cast<uintptr_t>(lhs) | (uintptr_t)row_bytes) & 15u) == 0;
    const uint32_t sw = v16 ? (uint32_t)KW::SW16 : (uint32_t)KW::SW;
    MvPart best{0.0f, 0, 0u, 0u};
    // One lane per row.  The warp stages its rows' block windows in shared
    // memory with asynchronous word copies (every word read holds bytes of
    // the block; a trailing half word copies 2 bytes), block b + 1 in flight
    // while block b is consumed; every lane forms its row's terms from the
    // window and folds them in block order.
    for (uint64_t g0 = ((uint64_t)blockIdx.x * kKWarps + warp) * 32; g0 < p.rows;
         g0 += (uint64_t)gridDim.x * kKWarps * 32) {
        const uint32_t nrows = p.rows - g0 < 32u ? (uint32_t)(p.rows - g0) : 32u;
        const uint8_t* group = lhs + g0 * row_bytes;
        float ls[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
        float total = 0.0f;
        const auto issue = [&](uint32_t b) {
            uint32_t* buf = stage + (b & 1u) * 32 * KW::SWM;
            if (v16) {
                const uint32_t off16 = (uint32_t)(((uint64_t)b * BB) & 15u);
                const uint8_t* first = group + (uint64_t)b * BB - off16;
                for (uint32_t v = lane; v < nrows * (uint32_t)KW::NC; v += 32) {
                    const uint32_t r = v / KW::NC, c = v % KW::NC;
                    if (16 * c < off16 + (uint32_t)BB) {
                        const uint32_t dst = (uint32_t)__cvta_generic_to_shared(buf + r * KW::SW16 + 4 * c);
                        const void* src = first + r * row_bytes + 16 * c;
                        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src) : "memory");
                    }
                }
                asm volatile("cp.async.commit_group;\n" ::: "memory");
                return;
            }
            for (uint32_t v = lane; v < nrows * (uint32_t)KW::NW; v += 32) {
                const uint32_t r = v / KW::NW, j = v % KW::NW;
                const uintptr_t at = reinterpret_cast<uintptr_t>(group + r * row_bytes + (uint64_t)b * BB);
                const uint32_t off = (uint32_t)(at & 3u);
                const uint32_t end = off + (uint32_t)BB;
                if (4 * j + 2 <= end) {
                    const uint32_t bytes = 4 * j + 4 <= end ? 4u : 2u;
                    const uint32_t dst = (uint32_t)__cvta_generic_to_shared(buf + r * KW::SW + j);
                    const void* src = reinterpret_cast<const void*>(at - off + 4 * j);
                    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(dst), "l"(src), "r"(bytes)
                                 : "memory");
                }
            }
            asm volatile("cp.async.commit_group;\n" ::: "memory");
        };
        __syncwarp();  // the previous group's readers are done with both buffers
        issue(0);
        for (uint32_t b = 0; b < blocks; ++b) {
            if (b + 1 < blocks) {
                issue(b + 1);
                asm volatile("cp.async.wait_group 1;\n" ::: "memory");
            } else {
                asm volatile("cp.async.wait_group 0;\n" ::: "memory");
            }
            __syncwarp();  // every lane's copies of block b are visible
            if ((uint32_t)lane < nrows) {
                const uintptr_t at = reinterpret_cast<uintptr_t>(group + lane * row_bytes + (uint64_t)b * BB);
                const uint32_t off = v16 ? (uint32_t)(((uint64_t)b * BB) & 15u) : (uint32_t)(at & 3u);
                const uint8_t* bp = reinterpret_cast<const uint8_t*>(stage + (b & 1u) * 32 * KW::SWM + lane * sw) + off;
                float o[kKTerms];
                if constexpr (CODE == kDtypeQ2_K)
                    q2k_block_terms(reinterpret_cast<const uint32_t*>(bp), rq + b * 64, rb + b * 16, rd[b], o);
                else if constexpr (CODE == kDtypeQ3_K)
                    q3k_block_terms(bp, rq + b * 64, rd[b], o);
                else if constexpr (CODE == kDtypeQ4_K)
                    q4k_block_terms(reinterpret_cast<const uint32_t*>(bp), rq + b * 64, rb + b * 16, rd[b], o);
                else
                    q6k_block_terms(bp, rq + b * 64, rd[b], o);
                if constexpr (CODE == kDtypeQ2_K) {
                    total = __fadd_rn(total, o[8]);
                } else {
#pragma unroll
                    for (int j = 0; j < 8; ++j) ls[j] = __fadd_rn(ls[j], o[j]);
                    if constexpr (CODE == kDtypeQ4_K) total = __fsub_rn(total, o[8]);
                }
            }
            __syncwarp();  // block b's readers are done before its buffer is refilled
        }
        if ((uint32_t)lane < nrows) {
            if constexpr (CODE != kDtypeQ2_K) {
#pragma unroll
                for (int j = 0; j < 8; ++j) total = __fadd_rn(total, ls[j]);
            }
            const uint64_t row = g0 + lane;
            const bool nan = is_nan(total);
            best = mv_better(best, MvPart{total, (int32_t)row, nan ? 0u : 1u, (nan && row == 0) ? 1u : 0u});
        }
    }
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
        for (int w = 1; w < kKWarps; ++w) b = mv_better(b, warp_best[w]);
        warp_best[0] = b;
    }
    __syncthreads();
    finish(p, warp_best[0]);
}

// Balanced K-quant rows (the vocabulary case).  One lane per row (the
// kernel above) makes a warp's unit 32 rows: 151,936 rows are 4,748 units,
// 2.005 per resident warp, so the last round runs a few warps alone and the
// kernel takes three unit-times for two units of work.  Here a warp's unit
// is two rows, 16 lanes per row: the unit's rows (contiguous, 16-byte
// multiples) come in with one bulk copy into the warp's double-buffered
// stage, lane j of a row forms the terms of blocks j, j + 16, ... into a
// shared term tile, and the row's reference fold -- lane sums j = 0..7 and
// the minimum chain, each over the blocks in order, then total + ls[0] + ...
// + ls[7] -- runs as nine independent chains on nine lanes.  Units: 75,968,
// 32 per warp; the rounding of the last round costs 3 % instead of 33 %.
constexpr int kK2Warps = 4;
constexpr int kK2Threads = kK2Warps * 32;

// shared memory of one warp: two stages of two rows and the [2][blocks][9]
// term tile, rounded to 128 bytes (every stage starts 16-byte aligned)
__host__ __device__ __forceinline__ uint32_t k2_warp_words(uint32_t stage_bytes, uint32_t blocks) {
    return ((2 * stage_bytes) / 4 + 18 * blocks + 31u) & ~31u;
}
// rq rows of 65 words and rb rows of 17 ints: sixteen lanes decoding
// sixteen different blocks read sixteen different banks
constexpr uint32_t kK2Qs = 65, kK2Bs = 17;
__host__ __device__ __forceinline__ uint32_t k2_pre_words(uint32_t blocks) {
    return (blocks * (kK2Qs + 1 + kK2Bs) + 31u) & ~31u;
}

template <int CODE>
__global__ void __launch_bounds__(kK2Threads, CODE == kDtypeQ6_K || CODE == kDtypeQ3_K ? 6 : 8)
    mv_argmax_k2(MvArgmaxPlan p, const uint8_t* lhs, uint32_t stage_bytes) {
    extern __shared__ __align__(128) uint32_t k2_smem[];
    __shared__ __align__(8) uint64_t bars[kK2Warps][2];
    __shared__ MvPart warp_best[kK2Warps];
    const uint32_t blocks = (uint32_t)(p.k / 256);
    constexpr uint32_t BB = KWindow<CODE>::BB;
    const uint32_t row_bytes = blocks * BB;
    uint32_t* rq = k2_smem;
    float* rd = reinterpret_cast<float*>(rq + blocks * kK2Qs);
    int* rb = reinterpret_cast<int*>(rd + blocks);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t pre_words = k2_pre_words(blocks);                          // 128-byte aligned
    const uint32_t warp_words = k2_warp_words(stage_bytes, blocks);         // two stages + term tile
    unsigned char* stage0 = reinterpret_cast<unsigned char*>(k2_smem + pre_words + warp * warp_words);
    float* terms = reinterpret_cast<float*>(stage0 + 2 * stage_bytes);     // [2 rows][blocks][9]
    if (lane == 0) {
        mbar_init(&bars[warp][0], 1);
        mbar_init(&bars[warp][1], 1);
        mbar_init_fence();
    }
    pdl_enter();
    quantize_rhs_q8k<CODE>(p, blocks, rq, rd, rb, kK2Warps, kK2Qs, kK2Bs);
    __syncthreads();

    const uint64_t units = (p.rows + 1) / 2;
    const uint64_t W = (uint64_t)gridDim.x * kK2Warps;
    const uint64_t gw = (uint64_t)blockIdx.x * kK2Warps + warp;
    const auto issue = [&](uint64_t u, uint32_t s) {
        if (lane == 0) {
            const uint32_t nr = p.rows - 2 * u < 2 ? 1u : 2u;
            mbar_expect_tx(&bars[warp][s], nr * row_bytes);
            bulk_load(stage0 + s * stage_bytes, lhs + 2 * u * (uint64_t)row_bytes, nr * row_bytes, &bars[warp][s]);
        }
    };
    const uint32_t rr = (uint32_t)lane >> 4, j = (uint32_t)lane & 15u;
    MvPart best{0.0f, 0, 0u, 0u};
    if (gw < units) issue(gw, 0);
    uint32_t it = 0;
    for (uint64_t u = gw; u < units; u += W, ++it) {
        const uint32_t s = it & 1u;
        const bool next = u + W < units;
        if (next) issue(u + W, s ^ 1u);
        if (!mbar_wait(&bars[warp][s], (it >> 1) & 1u)) {
            // a copy that never landed: flag it, let the other stage's copy
            // finish (bounded) before the shared memory is released, and stop
            if (lane == 0) atomicExch(p.fault, 1u);
            if (next) mbar_wait(&bars[warp][s ^ 1u], ((it + 1) >> 1) & 1u);
            break;
        }
        const uint64_t row = 2 * u + rr;
        const unsigned char* rowp = stage0 + s * stage_bytes + rr * row_bytes;
        if (row < p.rows) {
            for (uint32_t b = j; b < blocks; b += 16) {
                float o[kKTerms];
                if constexpr (CODE == kDtypeQ2_K)
                    q2k_block_terms(reinterpret_cast<const uint32_t*>(rowp + b * BB), rq + b * kK2Qs, rb + b * kK2Bs,
                                    rd[b], o);
                else if constexpr (CODE == kDtypeQ3_K)
                    q3k_block_terms(rowp + b * BB, rq + b * kK2Qs, rd[b], o);
                else if constexpr (CODE == kDtypeQ4_K)  // 144-byte blocks of 16-byte multiple rows: aligned
                    q4k_block_terms<true>(reinterpret_cast<const uint32_t*>(rowp + b * BB), rq + b * kK2Qs,
                                          rb + b * kK2Bs, rd[b], o);
                else
                    q6k_block_terms(rowp + b * BB, rq + b * kK2Qs, rd[b], o);
                float* t = terms + (rr * blocks + b) * 9;
                if constexpr (CODE == kDtypeQ2_K) {
                    t[8] = o[8];
                } else {
#pragma unroll
                    for (int q = 0; q < kKTerms; ++q) t[q] = o[q];
                }
            }
        }
        __syncwarp();
        // chain j of the row: j < 8 the lane sum ls[j], j == 8 the running
        // total (Q4_K subtracts the minimum terms, Q2_K adds its one term)
        float chain = 0.0f;
        if (row < p.rows && j < 9) {
            const float* t = terms + rr * blocks * 9 + j;
            if (j < 8) {
                if constexpr (CODE != kDtypeQ2_K)
                    for (uint32_t b = 0; b < blocks; ++b) chain = __fadd_rn(chain, t[b * 9]);
            } else {
                if constexpr (CODE == kDtypeQ2_K)
                    for (uint32_t b = 0; b < blocks; ++b) chain = __fadd_rn(chain, t[b * 9]);
                else if constexpr (CODE == kDtypeQ4_K)
                    for (uint32_t b = 0; b < blocks; ++b) chain = __fsub_rn(chain, t[b * 9]);
            }
        }
        float total = __shfl_sync(0xffffffffu, chain, (int)(rr * 16 + 8));
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            const float lsq = __shfl_sync(0xffffffffu, chain, (int)(rr * 16 + q));
            if constexpr (CODE != kDtypeQ2_K) total = __fadd_rn(total, lsq);
        }
        if (j == 0 && row < p.rows) {
            const bool nan = is_nan(total);
            best = mv_better(best, MvPart{total, (int32_t)row, nan ? 0u : 1u, (nan && row == 0) ? 1u : 0u});
        }
        __syncwarp();  // the stage and the term tile are consumed before they are refilled
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) best = mv_better(best, mv_shfl(best, o));
    if (lane == 0) warp_best[warp] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        MvPart b = warp_best[0];
        for (int w = 1; w < kK2Warps; ++w) b = mv_better(b, warp_best[w]);
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
        static DeviceFlags configured;
        const int smem = kMvStages * kMvStageBytes + 1024;  // + alignment slack
        if (!configured.done(env.device)) {
            err = cudaFuncSetAttribute(mv_argmax_tma, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
            if (err != cudaSuccess) return err;
            configured.mark(env.device);
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

// The balanced kernel when the rows are 16-byte multiples on a 16-byte
// aligned base (one bulk copy per two rows) and four warps' stages fit
// twice per SM; false to fall back to the one-lane-per-row kernel.
template <int CODE>
bool launch_k2(const LaunchEnv& env, const MvArgmaxPlan& p, const uint8_t* lhs, cudaError_t* err) {
    const uint32_t blocks = (uint32_t)(p.k / 256);
    const uint64_t row_bytes = (uint64_t)blocks * KWindow<CODE>::BB;
    if (((reinterpret_cast<uintptr_t>(lhs) | (uintptr_t)row_bytes) & 15u) != 0 || p.rows > 0x7fffffffull) return false;
    const uint32_t stage_bytes = (uint32_t)(2 * row_bytes);
    const size_t smem = ((size_t)k2_pre_words(blocks) + (size_t)kK2Warps * k2_warp_words(stage_bytes, blocks)) * 4;
    if (smem > 110 * 1024) return false;
    static DeviceFlags configured;
    if (!configured.done(env.device)) {
        *err = cudaFuncSetAttribute(mv_argmax_k2<CODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, 110 * 1024);
        if (*err != cudaSuccess) return true;
        configured.mark(env.device);
    }
    static DeviceKeyedValue resident;
    uint32_t ctas = 0;
    if (!resident.get(env.device, (uint32_t)smem, &ctas)) {
        int n = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, mv_argmax_k2<CODE>, kK2Threads, smem) != cudaSuccess || n < 1)
            n = 1;
        ctas = (uint32_t)n;
        resident.put(env.device, (uint32_t)smem, ctas);
    }
    const uint64_t units = (p.rows + 1) / 2;
    const uint64_t want = (units + kK2Warps - 1) / kK2Warps;
    const uint64_t cap = (uint64_t)env.sm_count * ctas;
    *err = launch_dependent(mv_argmax_k2<CODE>, dim3((unsigned)(want < cap ? want : cap)), dim3(kK2Threads), smem,
                            env.stream, p, lhs, stage_bytes);
    ++*env.launches;
    if (*err == cudaSuccess) *err = cudaGetLastError();
    return true;
}

template <int CODE>
cudaError_t launch_k(const LaunchEnv& env, const MvArgmaxPlan& p, const uint8_t* lhs) {
    cudaError_t k2_err = cudaSuccess;
    if (launch_k2<CODE>(env, p, lhs, &k2_err)) return k2_err;
    const uint64_t groups = (p.rows + kKWarps * 32 - 1) / (kKWarps * 32);
    const size_t table = (size_t)kKWarps * 2 * 32 * KWindow<CODE>::SWM * 4 + 16;  // staging windows + alignment
    const size_t smem = (size_t)(p.k / 256) * (64 * 4 + 4 + 16 * 4) + table;
    static DeviceFlags configured;
    if (!configured.done(env.device)) {
        const cudaError_t e = cudaFuncSetAttribute(mv_argmax_k<CODE>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                   (int)(128 * (64 * 4 + 4 + 16 * 4) + table));
        if (e != cudaSuccess) return e;
        configured.mark(env.device);
    }
    // one wave of resident CTAs (registers or shared memory decide how many),
    // cached per device for the last shared-memory size seen there
    static DeviceKeyedValue resident;
    uint32_t ctas = 0;
    if (!resident.get(env.device, (uint32_t)smem, &ctas)) {
        int n = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, mv_argmax_k<CODE>, kKThreads, smem) != cudaSuccess || n < 1)
            n = 1;
        ctas = (uint32_t)n;
        resident.put(env.device, (uint32_t)smem, ctas);
    }
    const uint64_t cap = (uint64_t)env.sm_count * ctas;
    const cudaError_t err = launch_dependent(mv_argmax_k<CODE>, dim3((unsigned)(groups < cap ? groups : cap)),
                                             dim3(kKThreads), smem, env.stream, p, lhs);
    ++*env.launches;
    return err != cudaSuccess ? err : cudaGetLastError();
}

cudaError_t launch_mul_mat_argmax_k(const LaunchEnv& env, const MvArgmaxPlan& p, const uint8_t* lhs, int code) {
    switch (code) {
    case kDtypeQ2_K: return launch_k<kDtypeQ2_K>(env, p, lhs);
    case kDtypeQ3_K: return launch_k<kDtypeQ3_K>(env, p, lhs);
    case kDtypeQ4_K: return launch_k<kDtypeQ4_K>(env, p, lhs);
    default: return launch_k<kDtypeQ6_K>(env, p, lhs);
    }
}

cudaError_t launch_mul_mat_argmax_packed(const LaunchEnv& env, const MvArgmaxPlan& p, const uint8_t* lhs, int code) {
    cudaError_t err;
    switch (code) {
    case kDtypeQ4_0: err = launch_packed<kDtypeQ4_0>(env, p, lhs); break;
    case kDtypeQ4_1: err = launch_packed<kDtypeQ4_1>(env, p, lhs); break;
    case kDtypeQ5_0: err = launch_packed<kDtypeQ5_0>(env, p, lhs); break;
    default: err = launch_packed<kDtypeQ8_0>(env, p, lhs); break;
    }
    ++*env.launches;
    return err != cudaSuccess ? err : cudaGetLastError();
}

}  // namespace emel
