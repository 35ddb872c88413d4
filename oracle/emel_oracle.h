/*
 * emel_oracle.h -- CPU restatement of the emel-kernels elementwise, broadcast
 * and reduction loops (stateforward/emel.rs, crates/emel-kernels/src/any/).
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker and the timed
 * CPU baseline.  Only tests/, __graft_entry__.smoke() and bench.py's CPU legs
 * may load it; the device library never links or calls it.
 *
 * Parity pinning: the restatement is checked against the reference's golden
 * parity manifests (snapshots/parity/kernel-{binary,broadcast,elementwise,
 * power,unary,softmax,normalization,activation,...}/manifest.txt) and the
 * known-answer unit tests (crates/emel-kernels/tests/any/) through
 * tests/golden/.  Operators the reference does not have (sub/div row
 * broadcast, modulo broadcast, f16 elementwise, softmax scale+mask, per-row
 * argmax, exact i64 argmax) are defined here as the cited loop extended with
 * the new operand; their parity is "unpinned" by any reference vector.
 *
 * Every entry point validates exactly as the reference guards do and never
 * writes the destination of a rejected request.
 */
#ifndef EMEL_ORACLE_H
#define EMEL_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same field layout as emel_tensor_view in include/emel_cuda.h so one host
 * struct can describe a buffer to both libraries. `data` is a HOST pointer. */
typedef struct oracle_view {
    void* data;
    uint64_t storage_bytes;
    uint64_t ne[4];
    uint64_t nb[4];
    uint32_t dtype;
    uint32_t reserved;
} oracle_view;

/* Status codes (numerically equal to emel_cuda_status). */
enum {
    ORACLE_OK = 0,
    ORACLE_INVALID_VIEW = 1,
    ORACLE_SHAPE_MISMATCH = 2,
    ORACLE_INVALID_PARAMETERS = 3,
    ORACLE_UNEXPECTED_EVENT = 4,
    ORACLE_INVALID_SHAPE = 6,
    ORACLE_UNSUPPORTED_OPERATION = 7,
    ORACLE_INVALID_LAYOUT = 8,
    ORACLE_INDEX_OUT_OF_BOUNDS = 9,
    ORACLE_UNSUPPORTED_SOURCE_STRIDE = 10,
    ORACLE_INVALID_MODE = 11,
    ORACLE_INVALID_REQUEST = 12,
    ORACLE_INVALID_ARGUMENT = 18
};

/* Shared op codes (numerically equal to the device library's enums). */
enum { ORACLE_ADD = 0, ORACLE_SUB = 1, ORACLE_MUL = 2, ORACLE_DIV = 3 };

int oracle_binary(int op, const oracle_view* lhs, const oracle_view* rhs, const oracle_view* dst);
int oracle_broadcast_row(int op, const oracle_view* src0, const oracle_view* src1, const oracle_view* dst);
int oracle_binary_repeat(int op, const oracle_view* src0, const oracle_view* src1, const oracle_view* dst);

int oracle_unary(int op, const oracle_view* src, const oracle_view* dst);
int oracle_op_unary(int subop, const oracle_view* src, const oracle_view* dst);
int oracle_scale(const oracle_view* src, const oracle_view* dst, float scale);
int oracle_clamp(const oracle_view* src, const oracle_view* dst, float lo, float hi);
int oracle_leaky_relu(const oracle_view* src, const oracle_view* dst, float slope);
int oracle_silu_back(const oracle_view* src, const oracle_view* grad, const oracle_view* dst);
/* matmul.rs OpMulMatArgmax: lhs [k, m] dense, rhs [1, k] dense, dst [1]. */
int oracle_mul_mat_argmax(const oracle_view* lhs, const oracle_view* rhs, const oracle_view* dst, int32_t* index_out);
/* matmul.rs OpMulMatArgmaxQ8_0: lhs Q8_0 packed rows [k, m] (k % 32 == 0,
 * k / 32 <= 1024), rhs [1, k] dense F32, dst [1]. */
int oracle_mul_mat_argmax_q8_0(const oracle_view* lhs, const oracle_view* rhs, const oracle_view* dst,
                               int32_t* index_out);
/* The same with Q4_0 (18-byte), Q4_1 (20-byte) and Q5_0 (22-byte) blocks
 * (matmul.rs OpMulMatArgmaxQ4_0 / Q4_1 / Q5_0). */
int oracle_mul_mat_argmax_q4_0(const oracle_view* lhs, const oracle_view* rhs, const oracle_view* dst,
                               int32_t* index_out);
int oracle_mul_mat_argmax_q4_1(const oracle_view* lhs, const oracle_view* rhs, const oracle_view* dst,
                               int32_t* index_out);
int oracle_mul_mat_argmax_q5_0(const oracle_view* lhs, const oracle_view* rhs, const oracle_view* dst,
                               int32_t* index_out);
/* K-quant rows (matmul.rs OpMulMatArgmaxQ4K / Q6K): 256-value blocks of 144 /
 * 210 bytes, k / 256 <= 128 blocks; the rhs is quantized to Q8_K. */
int oracle_mul_mat_argmax_q4_k(const oracle_view* lhs, const oracle_view* rhs, const oracle_view* dst,
                               int32_t* index_out);
int oracle_mul_mat_argmax_q6_k(const oracle_view* lhs, const oracle_view* rhs, const oracle_view* dst,
                               int32_t* index_out);
/* Q2_K (84-byte) and Q3_K (110-byte) blocks (OpMulMatArgmaxQ2K / Q3K). */
int oracle_mul_mat_argmax_q2_k(const oracle_view* lhs, const oracle_view* rhs, const oracle_view* dst,
                               int32_t* index_out);
int oracle_mul_mat_argmax_q3_k(const oracle_view* lhs, const oracle_view* rhs, const oracle_view* dst,
                               int32_t* index_out);
/* diag.rs OpDiag / OpDiagMaskInf (mode 0) / OpDiagMaskZero (mode 1) over flat
 * f32 slices. */
int oracle_diag(const float* input, uint64_t input_len, float* output, uint64_t output_len);
int oracle_diag_mask(int mode, const float* input, uint64_t input_len, float* output, uint64_t output_len,
                     int32_t n_past);
/* OpDiagMaskInf then OpSoftMax over the dense [side, side] result; scratch
 * holds side^2 floats. */
int oracle_soft_max_diag_mask_inf(const float* input, uint64_t input_len, float* output, uint64_t output_len,
                                  int32_t n_past, float* scratch);
/* flash_attn.rs FlashAttnOptions (flash_attn.rs:24-31): an absent scale is
 * 1 / sqrt(head_dim), an absent token count is the key's ne[1]. */
typedef struct oracle_flash_attn_options {
    float scale;
    uint32_t has_scale;
    uint32_t masked_total_tokens;
    uint32_t has_masked_total_tokens;
} oracle_flash_attn_options;
/* flash_attn.rs OpFlashAttnExt: query / dst dense F32 [d, 1, h, 1], key /
 * value F16 [d, t, hkv, 1] (any even strides); options nullable. */
uint16_t oracle_fa_f32_to_f16(float value); /* flash_attn.rs:528-557 */
int oracle_flash_attn_ext(const oracle_view* query, const oracle_view* key, const oracle_view* value,
                          const oracle_view* dst, const oracle_flash_attn_options* options);
/* rope.rs RopeParams (rope.rs:33-48) and OpRope. */
typedef struct oracle_rope_params {
    int32_t n_dims;
    int32_t mode;
    float freq_base;
    float freq_scale;
    float ext_factor;
    float attn_factor;
} oracle_rope_params;
int oracle_rope(const oracle_view* src, const oracle_view* positions, const oracle_view* dst,
                const oracle_rope_params* params);
/* get_rows.rs: every source type through one entry point (src dtype F32,
 * F16, BF16 30, Q4_0 2, Q8_0 8, Q4_K 12; indices I32 with ne[3] == 1; dst
 * dense F32). */
int oracle_get_rows(const oracle_view* src, const oracle_view* indices, const oracle_view* dst);
/* get_rows.rs OpGetRowsF32Bytes: byte-backed F32 source rows at any byte offset. */
int oracle_get_rows_f32_bytes(const oracle_view* src, const oracle_view* indices, const oracle_view* dst);
/* shape.rs OpCpy / OpCont. */
int oracle_cpy(const oracle_view* src, const oracle_view* dst);
int oracle_cont(const oracle_view* src, const oracle_view* dst);
/* glu.rs OpGlu: output[i] = input[i] * gate(input[n + i]), n = output_len. */
int oracle_glu(int subop, const float* input, uint64_t input_len, float* output, uint64_t output_len);
int oracle_add1(const oracle_view* src, const oracle_view* dst, float scalar);
int oracle_copy(const oracle_view* src, const oracle_view* dst);

int oracle_norm(const oracle_view* src, const oracle_view* dst, float eps);
int oracle_rms_norm(const oracle_view* src, const oracle_view* dst, float eps);
int oracle_rms_norm_mul(const oracle_view* src, const oracle_view* weight, const oracle_view* dst, float eps);

int oracle_soft_max(const oracle_view* src, const oracle_view* dst);
int oracle_soft_max_ext(const oracle_view* src, const oracle_view* mask, const oracle_view* dst, float scale);

int oracle_sum(const oracle_view* src, const oracle_view* dst);
int oracle_sum_f64(const oracle_view* src, double* out);
int oracle_mean(const oracle_view* src, const oracle_view* dst);
int oracle_sum_rows(const oracle_view* src, const oracle_view* dst);
int oracle_argmax(const oracle_view* src, const oracle_view* dst);
int oracle_argmax_index(const oracle_view* src, int64_t* index, float* value);
int oracle_argmax_rows(const oracle_view* src, const oracle_view* dst);

/* The generic operation envelope (generic.rs:580-766 GenericRequest, the
 * maintained routes of sm.rs:324-425 restricted to the device table's
 * elementwise / broadcast / reduction set; same layout as
 * emel_cuda_generic_request).  Other operation codes return
 * ORACLE_UNSUPPORTED_OPERATION, as the device table does. */
typedef struct oracle_generic_request {
    uint32_t op;
    uint32_t unary_subop;
    const oracle_view* src0;
    const oracle_view* src1;
    const oracle_view* src2;
    const oracle_view* dst;
    uint8_t params[64];
    uint32_t params_len;
    uint32_t reserved;
} oracle_generic_request;
int oracle_generic(const oracle_generic_request* request);

/* Row-range variants used by the multi-threaded CPU baseline: identical
 * arithmetic, restricted to rows [row_begin, row_end) of a validated request
 * (no validation; the caller validated the whole request first). */
void oracle_unary_range(int op, const oracle_view* src, const oracle_view* dst, uint64_t begin, uint64_t end);
void oracle_rms_norm_rows(const oracle_view* src, const oracle_view* dst, float eps, uint64_t row_begin, uint64_t row_end);

/* The reference's own binary16 conversions (crates/emel-kernels/src/any/unary.rs:546-586). */
uint16_t oracle_fp32_to_fp16(float value);
float oracle_fp16_to_fp32(uint16_t bits);

#ifdef __cplusplus
}
#endif
#endif
