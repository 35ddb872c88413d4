// Peer exchange of small per-rank payloads (the whole-tensor sum and argmax
// partials of a sharded tensor) over NVLink, without a collective library.
//
// Each rank owns one buffer that every peer maps (CUDA IPC).  Publishing
// epoch e (a device-side counter, so a replayed CUDA graph advances it) is
// one tiny kernel: thread r stores this rank's payload into rank r's buffer,
// slot [e & 1][rank], with plain stores over NVLink, then stores e into that
// buffer's flag word for this rank with release semantics at system scope.
// Waiting is a second tiny kernel: thread r polls its own buffer's flag word
// for rank r with acquire loads until it reaches e, then copies slot
// [e & 1][r] into the caller's gathered array (rank order).
//
// Two slot banks make reuse safe: a rank publishes epoch e + 2 into bank
// e & 1 only after its wait for epoch e + 1 saw every peer's flag, and each
// peer published e + 1 after its own wait for e had copied bank e & 1.
//
// Every poll is bounded by the global timer (the limit given at creation)
// and by an iteration count; on expiry the wait sets the context's fault word
// (emel_cuda_stream_synchronize then returns EMEL_CUDA_TIMEOUT) and returns.
#include <cstdint>

#include "common.cuh"
#include "launch.hpp"
#include "pdl.cuh"

namespace emel {

namespace {

__device__ __forceinline__ void store_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t load_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint64_t now_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ char* slot(char* buffer, uint32_t epoch, int rank, uint32_t slot_bytes) {
    return buffer + kExchangeHeaderBytes + ((uint64_t)(epoch & 1u) * kExchangeMaxRanks + (uint64_t)rank) * slot_bytes;
}

// Both kernels are launched as programmatic dependents (pdl.cuh): they wait
// for the previous kernel of the stream (the payload's producer, or the
// work the gathered values follow) before touching memory, while their own
// launch overlaps its tail, and they let the next kernel be scheduled.
__global__ void __launch_bounds__(kExchangeMaxRanks) exchange_publish(ExchangeArgs a) {
    pdl_enter();
    __shared__ uint32_t epoch;
    if (threadIdx.x == 0) epoch = ++*a.epoch;
    __syncthreads();
    const int r = threadIdx.x;
    if (r >= a.world) return;
    const uint4* src = static_cast<const uint4*>(a.payload);
    uint4* dst = reinterpret_cast<uint4*>(slot(a.peers[r], epoch, a.rank, a.slot_bytes));
    for (uint32_t i = 0; i < a.bytes / 16; ++i) dst[i] = src[i];
    // release: the payload stores above are visible to rank r before the flag
    store_release_sys(reinterpret_cast<uint32_t*>(a.peers[r]) + a.rank, epoch);
}

// COMBINE: the payload is a shard's f64 sum then its argmax partial (32
// bytes); after the gather, thread 0 adds the sums in rank order and rounds
// once to f32 (reductions.rs:671-681 accumulates the whole tensor in f64),
// and picks the argmax with the reference's rules (reductions.rs:715-730:
// a later shard wins only with a strictly greater value; no comparable value,
// or a NaN at element 0 of the whole tensor, leaves index 0).
template <bool COMBINE>
__global__ void __launch_bounds__(kExchangeMaxRanks) exchange_wait(ExchangeArgs a, void* gathered, CombineOut c) {
    pdl_enter();
    __shared__ uint32_t failed;
    if (threadIdx.x == 0) failed = 0u;
    if constexpr (COMBINE) __syncthreads();
    const int r = threadIdx.x;
    if (r < a.world) {
        const uint32_t epoch = *a.epoch;  // set by this rank's publish, earlier on the stream
        char* own = a.peers[a.rank];
        const uint32_t* flag = reinterpret_cast<const uint32_t*>(own) + r;
        const uint64_t t0 = now_ns();
        bool ok = false;
        for (uint32_t i = 0; i < (1u << 28); ++i) {
            if ((int32_t)(load_acquire_sys(flag) - epoch) >= 0) {
                ok = true;
                break;
            }
            if ((i & 255u) == 255u) {
                if (now_ns() - t0 > a.timeout_ns) break;
                __nanosleep(200);
            }
        }
        if (!ok) {
            atomicExch(a.fault, 1u);
            atomicOr(&failed, 1u);
        } else {
            const uint4* src = reinterpret_cast<const uint4*>(slot(own, epoch, r, a.slot_bytes));
            uint4* dst = reinterpret_cast<uint4*>(static_cast<char*>(gathered) + (uint64_t)r * a.bytes);
            for (uint32_t i = 0; i < a.bytes / 16; ++i) dst[i] = src[i];
        }
    }
    if constexpr (COMBINE) {
        __syncthreads();  // the gathered payloads of every rank are written
        if (threadIdx.x != 0 || failed) return;
        const char* g = static_cast<const char*>(gathered);
        double total = 0.0;
        bool has = false;
        float best = 0.0f;
        int64_t idx = 0;
        for (int k = 0; k < a.world; ++k) {
            const char* q = g + (uint64_t)k * a.bytes;
            total += *reinterpret_cast<const double*>(q);
            const float v = *reinterpret_cast<const float*>(q + 8);
            const uint32_t h = *reinterpret_cast<const uint32_t*>(q + 12);
            const int64_t i = *reinterpret_cast<const int64_t*>(q + 16);
            if (!h) continue;
            if (!has || v > best || (v == best && i < idx)) {
                has = true;
                best = v;
                idx = i;
            }
        }
        const uint32_t first_nan = *reinterpret_cast<const uint32_t*>(g + 24);
        if (first_nan || !has) idx = 0;
        *static_cast<float*>(c.sum) = __double2float_rn(total);
        if (c.index_dtype == (int)DType::I64) *static_cast<int64_t*>(c.index) = idx;
        else if (c.index_dtype == (int)DType::I32) *static_cast<int32_t*>(c.index) = (int32_t)idx;
        else *static_cast<float*>(c.index) = (float)idx;
    }
}

}  // namespace

uint64_t exchange_buffer_bytes(uint32_t slot_bytes) {
    return kExchangeHeaderBytes + 2ull * kExchangeMaxRanks * slot_bytes;
}

cudaError_t launch_exchange_publish(cudaStream_t stream, const ExchangeArgs& args) {
    const cudaError_t err = launch_dependent(exchange_publish, dim3(1), dim3(kExchangeMaxRanks), 0, stream, args);
    return err != cudaSuccess ? err : cudaGetLastError();
}

cudaError_t launch_exchange_wait(cudaStream_t stream, const ExchangeArgs& args, void* gathered) {
    const cudaError_t err =
        launch_dependent(exchange_wait<false>, dim3(1), dim3(kExchangeMaxRanks), 0, stream, args, gathered, CombineOut{});
    return err != cudaSuccess ? err : cudaGetLastError();
}

cudaError_t launch_exchange_wait_combine(cudaStream_t stream, const ExchangeArgs& args, void* gathered,
                                         const CombineOut& out) {
    const cudaError_t err =
        launch_dependent(exchange_wait<true>, dim3(1), dim3(kExchangeMaxRanks), 0, stream, args, gathered, out);
    return err != cudaSuccess ? err : cudaGetLastError();
}

}  // namespace emel
