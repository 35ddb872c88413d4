// Kernel launchers called by the host API after validation.  Each returns the
// CUDA error of its launch(es); none allocates memory.
#pragma once

#include <atomic>
#include <cstdint>

#include "plan.hpp"

namespace emel {

// Per-device, thread-safe records of one-time launch set-up (a kernel's
// shared-memory limit raised, its occupancy found).  Devices 0..63 each have
// their own slot; a device beyond that redoes the set-up on every call.
constexpr int kSetupDevices = 64;

// One bit per device: the set-up it guards has been done on that device.
struct DeviceFlags {
    std::atomic<uint64_t> bits{0};
    bool done(int dev) const {
        return dev >= 0 && dev < kSetupDevices && ((bits.load(std::memory_order_acquire) >> dev) & 1ull);
    }
    void mark(int dev) {
        if (dev >= 0 && dev < kSetupDevices) bits.fetch_or(1ull << dev, std::memory_order_acq_rel);
    }
};

// One cached value per device, valid for one key (e.g. the dynamic
// shared-memory size an occupancy figure was computed for).  A slot packs
// (key + 1) << 32 | value, so 0 means empty; two threads that race store the
// same value for the same key.
struct DeviceKeyedValue {
    std::atomic<uint64_t> slot[kSetupDevices] = {};
    bool get(int dev, uint32_t key, uint32_t* value) const {
        if (dev < 0 || dev >= kSetupDevices) return false;
        const uint64_t s = slot[dev].load(std::memory_order_acquire);
        if ((s >> 32) != (uint64_t)key + 1) return false;
        *value = (uint32_t)s;
        return true;
    }
    void put(int dev, uint32_t key, uint32_t value) {
        if (dev >= 0 && dev < kSetupDevices)
            slot[dev].store((((uint64_t)key + 1) << 32) | value, std::memory_order_release);
    }
};

struct UnaryParams;

cudaError_t launch_unary(const LaunchEnv& env, const EwPlan& plan, int op, float pa, float pb);
cudaError_t launch_binary(const LaunchEnv& env, const EwPlan& plan, int op);

// op: 0 norm, 1 rms_norm, 2 rms_norm * weight (aux)
cudaError_t launch_norm(const LaunchEnv& env, const RowPlan& plan, int op, float eps);
// soft_max (scale applied when apply_scale; aux = optional mask)
cudaError_t launch_soft_max(const LaunchEnv& env, const RowPlan& plan, bool apply_scale, float scale);
cudaError_t launch_sum_rows(const LaunchEnv& env, const RowPlan& plan);
// dst dtype: F32 / I32 / I64, index written as the column
cudaError_t launch_argmax_rows(const LaunchEnv& env, const RowPlan& plan, int dst_dtype);

// Whole-tensor reductions over a RowPlan (rows of ne0), using the context
// workspace for per-block partials.
// mode: 0 -> write f32 sum to out (dst element), 1 -> f32 mean, 2 -> f64 sum
cudaError_t launch_sum(const LaunchEnv& env, const RowPlan& plan, int mode, void* out);
// out_kind: 0 -> index as dtype of dst (F32/I32/I64) into out; 1 -> argmax
// partial struct (value, has_value, index + index_base) into out
cudaError_t launch_argmax(const LaunchEnv& env, const RowPlan& plan, int out_kind, int dst_dtype, int64_t index_base,
                          void* out);

// Ring-staged norm / rms_norm / rms_norm * weight / soft_max (rowring.cu).
// Returns false, launching nothing, when the view does not qualify.
// op: 0 norm, 1 rms_norm, 2 rms_norm * weight, 3 soft_max, 4 / 5 the
// generic envelope's norm / rms_norm.
bool launch_row_ring(const LaunchEnv& env, const RowPlan& plan, int op, float param, bool apply_scale,
                     cudaError_t* err);

// The generic operation envelope (generic.rs): its norm (3) / rms_norm (4)
// numerics, its soft_max, and repeat as a modulo-broadcast copy.
cudaError_t launch_norm_generic(const LaunchEnv& env, const RowPlan& plan, int op, float eps);
cudaError_t launch_soft_max_generic(const LaunchEnv& env, const RowPlan& plan);
cudaError_t launch_repeat(const LaunchEnv& env, const EwPlan& plan);

// Few long rows (rowsplit.cu): one 8-CTA cluster per row.
bool split_rows_wanted(const LaunchEnv& env, const RowPlan& plan);
cudaError_t launch_argmax_rows_split(const LaunchEnv& env, const RowPlan& plan, int dst_dtype);
cudaError_t launch_sum_rows_split(const LaunchEnv& env, const RowPlan& plan);
cudaError_t launch_soft_max_split(const LaunchEnv& env, const RowPlan& plan, bool apply_scale, float scale);

// Byte offset, inside the workspace's 256-byte header, of the fault word a
// kernel sets when one of its bounded waits expires.
constexpr uint64_t kFaultWordOffset = 64;

// binary16 domain tables of a context (elementwise.cu): one table of 65,536
// halves for each of the 8 unary ops that stream large binary16 tensors
// through a lookup; built once by build_domain_tables.
constexpr int kDomainTableSlots = 8;
constexpr uint64_t kDomainTableBytes = (uint64_t)kDomainTableSlots * 65536ull * 2ull;
cudaError_t build_domain_tables(void* tables, cudaStream_t stream);

// Bytes of context workspace: the whole-tensor reductions' partials and, at
// split_rows_workspace_offset, one 16-byte partial per chunk of each of up to
// sm_count long rows plus one ticket per row (the few-long-rows kernels).
constexpr int kSplitRowChunks = 8;
uint64_t reduction_workspace_bytes(int sm_count);
uint64_t split_rows_workspace_offset(int sm_count);

// Row gather (getrows.cu).
enum GatherKind : int { kGatherF32 = 0, kGatherF16 = 1, kGatherBF16 = 2, kGatherQ4_0 = 3, kGatherQ8_0 = 4, kGatherQ4_K = 5,
                        kGatherF32Bytes = 6 };

// Workspace header words of the index guard: the context's sticky rejected
// status (reported by emel_cuda_stream_synchronize) and one call's flag.
constexpr uint64_t kRejectWordOffset = 72;
constexpr uint64_t kCallFlagOffset = 80;

struct GatherPlan {
    int kind;
    bool vec;               // F32 / F16 / BF16: rows may move as 16-byte vectors
    const char* src;
    float* dst;             // dense [cols, dst_rows]
    const int32_t* idx;
    uint64_t idx_ne[3];
    int64_t idx_st[3];      // elements
    uint64_t cols, rows, batches;
    int64_t src_st[4];      // bytes (F32: dims 1..3 used; F16 / BF16: all four)
    uint64_t row_bytes;     // quantized rows
    uint64_t dst_rows;      // number of indices
    uint32_t* flag;
    uint32_t* reject;
    uint32_t reject_code;
};

cudaError_t launch_get_rows(const LaunchEnv& env, const GatherPlan& plan);

// Rotary position embedding (rope.cu).
enum RopeMode : int { kRopeNorm = 0, kRopeNeox = 2, kRopeTimestep = 4 };

struct RopePlan {
    int mode;
    bool vec;               // norm / neox on 16-byte aligned unit-stride rows (see emel_cuda_rope)
    const char* src;
    char* dst;
    const char* positions;
    int64_t pos_stride;     // bytes
    int64_t src_st[4];      // bytes
    int64_t dst_st[4];
    uint64_t cols, rows, npos, batches;
    uint64_t n_dims;
    float theta_scale;      // powf(freq_base, -2 / n_dims), from the host
    float neg_log_period;   // -logf(freq_base), from the host
    float freq_scale, attn_factor;
};

cudaError_t launch_rope(const LaunchEnv& env, const RopePlan& plan);

// Vocabulary matvec + argmax (matvec.cu).
struct MvArgmaxPlan {
    const float* lhs;   // dense [k, rows]
    const float* rhs;   // dense [k]
    uint64_t k, rows;
    bool vec;           // k % 4 == 0 and 16-byte aligned operands: bulk-copy tiles
    float* dst_value;
    int32_t* dst_index;
    unsigned* ticket;   // workspace
    void* partials;     // workspace, 16 bytes per CTA
    uint32_t* fault;
};

cudaError_t launch_mul_mat_argmax(const LaunchEnv& env, const MvArgmaxPlan& plan);
// Packed rows (lhs: Q4_0 / Q4_1 / Q5_0 / Q8_0 blocks of 32 values, rows of
// k / 32 blocks, 4-byte aligned base); plan.lhs unused, plan.k a multiple of
// 32 up to 32768; code: the lhs dtype code.
constexpr int kDtypeQ4_0 = 2, kDtypeQ4_1 = 3, kDtypeQ5_0 = 6, kDtypeQ8_0 = 8;
cudaError_t launch_mul_mat_argmax_packed(const LaunchEnv& env, const MvArgmaxPlan& plan, const uint8_t* lhs, int code);
// K-quant rows: Q2_K (84-byte), Q3_K (110-byte), Q4_K (144-byte) or Q6_K
// (210-byte) blocks of 256 values, 4-byte aligned base; plan.k a multiple
// of 256 up to 32768.
constexpr int kDtypeQ2_K = 10, kDtypeQ3_K = 11, kDtypeQ4_K = 12, kDtypeQ6_K = 14;
cudaError_t launch_mul_mat_argmax_k(const LaunchEnv& env, const MvArgmaxPlan& plan, const uint8_t* lhs, int code);

// Single-query attention (attention.cu): one CTA per query head.
struct FlashAttnPlan {
    const float* q;     // dense [d, 1, heads]
    const char* k;      // binary16 [d, tokens, kv_heads], byte strides ks
    const char* v;      // binary16, byte strides vs
    float* dst;         // dense [d, 1, heads]
    uint64_t ks[3], vs[3];
    uint64_t d, tokens, heads, rep;  // rep = heads / kv_heads
    float scale;
    bool k_rows;        // key rows unit-stride, 16-byte aligned, d % 8 == 0: vector loads
    bool v_bulk;        // value rows unit-stride, 16-byte aligned, d % 8 == 0: TMA bulk copies
    bool v_dense;       // ... and consecutive tokens adjacent: one copy per tile
    uint32_t* fault;    // set when a bounded wait expires
};

cudaError_t launch_flash_attn(const LaunchEnv& env, const FlashAttnPlan& plan);

// Diagonal family (diag.cu): side x side row-major F32 matrices.
enum DiagMode : int { kDiag = 0, kDiagMaskInf = 1, kDiagMaskZero = 2, kDiagSoftMaxCausal = 3 };
struct DiagPlan {
    const float* in;    // diag: [side]; masks: [side * side] (may equal out)
    float* out;         // [side * side]
    uint64_t side;
    uint64_t n_past;    // masks: columns <= row + n_past keep the input
    bool vec;           // side % 4 == 0 and 16-byte aligned pointers
};

cudaError_t launch_diag(const LaunchEnv& env, const DiagPlan& plan, int mode);

// Peer exchange over NVLink (exchange.cu).  Every rank owns one buffer of
// kExchangeHeaderBytes flag words (flag r = the last epoch rank r published
// into this buffer) followed by two banks (epoch parity) of kExchangeMaxRanks
// slots; peers[r] is rank r's buffer as mapped in this process.
constexpr int kExchangeMaxRanks = 64;
constexpr uint32_t kExchangeHeaderBytes = 256;
constexpr uint32_t kExchangeMaxBytes = 1024;

struct ExchangeArgs {
    char* peers[kExchangeMaxRanks];
    const void* payload;  // this rank's payload (device, 16-byte aligned)
    uint32_t* epoch;      // this rank's epoch counter (device)
    uint32_t* fault;      // the context's fault word
    int world;
    int rank;
    uint32_t bytes;       // payload bytes, a multiple of 16
    uint32_t slot_bytes;  // slot stride
    uint64_t timeout_ns;
};

uint64_t exchange_buffer_bytes(uint32_t slot_bytes);
cudaError_t launch_exchange_publish(cudaStream_t stream, const ExchangeArgs& args);
cudaError_t launch_exchange_wait(cudaStream_t stream, const ExchangeArgs& args, void* gathered);

// Destinations of the combined whole-tensor answers: the f32 sum and the
// argmax index in dtype index_dtype (F32, I32 or I64).
struct CombineOut {
    void* sum;
    void* index;
    int index_dtype;
};
cudaError_t launch_exchange_wait_combine(cudaStream_t stream, const ExchangeArgs& args, void* gathered,
                                         const CombineOut& out);

}  // namespace emel
