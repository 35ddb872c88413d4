/*
 * emel_cuda.h -- C ABI of the B200 (sm_100a) device op table for the
 * emel-kernels elementwise, broadcast and reduction operators.
 *
 * Every entry point replaces one typed event of the reference operator
 * contract, `emel_kernels::Kernel::process_event<E: Event>` (stateforward/
 * emel.rs, crates/emel-kernels/src/any/actor.rs:936-943), and keeps its
 * argument meaning and error behaviour:
 *
 *   - views are the reference's 4-D `Layout { dtype, ne[4], nb[4] }`
 *     (crates/emel-kernels/src/any/tensor_view.rs:215-219) bound to device
 *     storage instead of a Rust slice; `nb` are byte strides and nb[0] == 0
 *     means implicit row-major (tensor_view.rs:262-277);
 *   - validation runs synchronously on the host before anything is launched,
 *     in the reference's guard order (view -> shape -> parameters), and a
 *     rejected request never writes its destination;
 *   - accepted requests are enqueued on `stream` (a cudaStream_t; NULL is the
 *     legacy default stream) and return EMEL_CUDA_OK without synchronising.
 *
 * Plain C: pointers and sizes only.  No entry point allocates device memory
 * except emel_cuda_context_create and emel_cuda_malloc.
 */
#ifndef EMEL_CUDA_H
#define EMEL_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define EMEL_CUDA_ABI_VERSION 1

#if defined(__GNUC__)
#define EMEL_CUDA_API __attribute__((visibility("default")))
#else
#define EMEL_CUDA_API
#endif

/* DType::code() wire values (tensor_view.rs:160-209). */
enum emel_cuda_dtype {
    EMEL_DTYPE_F32 = 0,
    EMEL_DTYPE_F16 = 1,
    EMEL_DTYPE_Q4_0 = 2,  /* packed blocks: ne[0] values, nb[0] == 1 (byte rows) */
    EMEL_DTYPE_Q4_1 = 3,
    EMEL_DTYPE_Q5_0 = 6,
    EMEL_DTYPE_Q8_0 = 8,
    EMEL_DTYPE_Q2_K = 10,
    EMEL_DTYPE_Q3_K = 11,
    EMEL_DTYPE_Q4_K = 12,
    EMEL_DTYPE_Q6_K = 14,
    EMEL_DTYPE_I32 = 26,
    EMEL_DTYPE_I64 = 27,
    EMEL_DTYPE_F64 = 28,
    EMEL_DTYPE_BF16 = 30
};

/* One status per reference error variant: BinaryError (binary.rs:20-29),
 * BroadcastError (broadcast.rs:29-38), UnaryError (unary.rs:22-31),
 * NormalizationError (normalization.rs:31-42), ReductionError
 * (reductions.rs:21-30); plus the device-side outcomes. */
typedef enum emel_cuda_status {
    EMEL_CUDA_OK = 0,
    EMEL_CUDA_INVALID_VIEW = 1,       /* *Error::InvalidView */
    EMEL_CUDA_SHAPE_MISMATCH = 2,     /* *Error::ShapeMismatch */
    EMEL_CUDA_INVALID_PARAMETERS = 3, /* NormalizationError::InvalidParameters */
    EMEL_CUDA_UNEXPECTED_EVENT = 4,   /* *Error::UnexpectedEvent */
    EMEL_CUDA_INTERNAL = 5,           /* *Error::Internal */
    EMEL_CUDA_INVALID_SHAPE = 6,      /* Error::InvalidShape (generic envelope, actor.rs:88-90) */
    EMEL_CUDA_UNSUPPORTED_OPERATION = 7, /* Error::UnsupportedOperation (actor.rs:92) */
    EMEL_CUDA_INVALID_LAYOUT = 8,     /* ShapeError::InvalidLayout (shape.rs:30-31) */
    EMEL_CUDA_INDEX_OUT_OF_BOUNDS = 9, /* GetRowsError::IndexOutOfBounds (get_rows.rs:522-535) */
    EMEL_CUDA_UNSUPPORTED_SOURCE_STRIDE = 10, /* GetRowsError::UnsupportedSourceStride */
    EMEL_CUDA_INVALID_MODE = 11,      /* RopeError::InvalidMode (rope.rs:104-117) */
    EMEL_CUDA_INVALID_REQUEST = 12,   /* FlashAttnError::InvalidRequest (flash_attn.rs:35-44); gguf Error::InvalidRequest */
    EMEL_CUDA_MODEL_INVALID = 13,     /* emel-gguf Error::ModelInvalid (loader/mod.rs:103-118) */
    EMEL_CUDA_CAPACITY = 14,          /* emel-gguf Error::Capacity */
    EMEL_CUDA_PARSE_FAILED = 15,      /* emel-gguf Error::ParseFailed */
    EMEL_CUDA_DEVICE_ERROR = 16,      /* a CUDA runtime call failed */
    EMEL_CUDA_TIMEOUT = 17,           /* a bounded device wait expired */
    EMEL_CUDA_INVALID_ARGUMENT = 18,  /* null context / output pointer */
    EMEL_CUDA_OUT_OF_MEMORY = 19
} emel_cuda_status;

/* A tensor view over device memory.  `data` is the device address of the
 * first byte of the backing storage; `storage_bytes` is how many bytes of it
 * the view may reach (the Rust slice length times the element size).  The
 * same struct describes inputs and outputs. */
typedef struct emel_tensor_view {
    void* data;
    uint64_t storage_bytes;
    uint64_t ne[4];
    uint64_t nb[4];
    uint32_t dtype;
    uint32_t reserved; /* must be 0 */
} emel_tensor_view;

typedef struct emel_cuda_context emel_cuda_context;

/* Binary formulas (binary.rs:386-409); codes match the generic envelope's
 * binary selector (generic.rs:1280-1305). */
typedef enum emel_cuda_binary_op {
    EMEL_BINARY_ADD = 0,
    EMEL_BINARY_SUB = 1,
    EMEL_BINARY_MUL = 2,
    EMEL_BINARY_DIV = 3
} emel_cuda_binary_op;

/* Unary formulas.  Codes 0..21 are the UnarySubOp wire codes
 * (unary.rs:101-146); 64.. are the other single-input reference events. */
typedef enum emel_cuda_unary_op {
    EMEL_UNARY_ABS = 0,
    EMEL_UNARY_SGN = 1,
    EMEL_UNARY_NEG = 2,
    EMEL_UNARY_STEP = 3,
    EMEL_UNARY_TANH = 4,
    EMEL_UNARY_ELU = 5,
    EMEL_UNARY_RELU = 6,
    EMEL_UNARY_SIGMOID = 7,
    EMEL_UNARY_GELU = 8,
    EMEL_UNARY_GELU_QUICK = 9,
    EMEL_UNARY_SILU = 10,
    EMEL_UNARY_HARDSWISH = 11,
    EMEL_UNARY_HARDSIGMOID = 12,
    EMEL_UNARY_EXP = 13,
    EMEL_UNARY_EXPM1 = 14,
    EMEL_UNARY_SOFTPLUS = 15,
    EMEL_UNARY_GELU_ERF = 16,
    EMEL_UNARY_XIELU = 17, /* no typed event in the reference: UNEXPECTED_EVENT */
    EMEL_UNARY_FLOOR = 18,
    EMEL_UNARY_CEIL = 19,
    EMEL_UNARY_ROUND = 20,
    EMEL_UNARY_TRUNC = 21,
    EMEL_UNARY_SQR = 64,  /* power.rs OpSqr (pow(x, 2.0)) */
    EMEL_UNARY_SQRT = 65, /* power.rs OpSqrt */
    EMEL_UNARY_LOG = 66,  /* reductions.rs OpLog */
    EMEL_UNARY_SIN = 67,  /* reductions.rs OpSin */
    EMEL_UNARY_COS = 68   /* reductions.rs OpCos */
} emel_cuda_unary_op;

/* ---- context, memory and streams (the Rust host side owns these) ------ */

/* Creates a context on `device`: selects the device, queries its SM count
 * and allocates the context's reduction workspace. */
EMEL_CUDA_API emel_cuda_status emel_cuda_context_create(int device, emel_cuda_context** out);
EMEL_CUDA_API emel_cuda_status emel_cuda_context_destroy(emel_cuda_context* ctx);
/* Human-readable text of the last CUDA error seen by this context. */
EMEL_CUDA_API const char* emel_cuda_context_last_error(const emel_cuda_context* ctx);

EMEL_CUDA_API emel_cuda_status emel_cuda_malloc(emel_cuda_context* ctx, uint64_t bytes, void** out);
EMEL_CUDA_API emel_cuda_status emel_cuda_free(emel_cuda_context* ctx, void* ptr);
EMEL_CUDA_API emel_cuda_status emel_cuda_memcpy_h2d(emel_cuda_context* ctx, void* stream, void* dst, const void* src, uint64_t bytes);
EMEL_CUDA_API emel_cuda_status emel_cuda_memcpy_d2h(emel_cuda_context* ctx, void* stream, void* dst, const void* src, uint64_t bytes);
EMEL_CUDA_API emel_cuda_status emel_cuda_memset(emel_cuda_context* ctx, void* stream, void* dst, int value, uint64_t bytes);
EMEL_CUDA_API emel_cuda_status emel_cuda_stream_create(emel_cuda_context* ctx, void** out);
EMEL_CUDA_API emel_cuda_status emel_cuda_stream_destroy(emel_cuda_context* ctx, void* stream);
/* Waits for the stream.  Returns EMEL_CUDA_TIMEOUT (once) when a kernel of
 * this context gave up a bounded device wait since the last call; the
 * outputs of the work enqueued since then are unspecified.  Otherwise
 * returns (once) the status of a request the device rejected since the last
 * call (emel_cuda_get_rows: EMEL_CUDA_INDEX_OUT_OF_BOUNDS; that request wrote
 * nothing). */
EMEL_CUDA_API emel_cuda_status emel_cuda_stream_synchronize(emel_cuda_context* ctx, void* stream);
/* Number of kernels this context has launched (all entry points; a graph
 * replay counts the kernels it contains). */
EMEL_CUDA_API uint64_t emel_cuda_launch_count(const emel_cuda_context* ctx);

/* Events.  emel_cuda_event_record on a stream being captured records a
 * dependency (fork / join of graph branches); emel_cuda_event_record_timed
 * there becomes an event-record node of the graph instead, so kernels
 * inside a replayed graph can be timed.  Outside a capture both record
 * normally.  No counterpart in the reference (it has no device). */
EMEL_CUDA_API emel_cuda_status emel_cuda_event_create(emel_cuda_context* ctx, void** out);
EMEL_CUDA_API emel_cuda_status emel_cuda_event_record(emel_cuda_context* ctx, void* event, void* stream);
EMEL_CUDA_API emel_cuda_status emel_cuda_event_record_timed(emel_cuda_context* ctx, void* event, void* stream);
EMEL_CUDA_API emel_cuda_status emel_cuda_event_elapsed_ms(emel_cuda_context* ctx, void* start, void* end, float* ms);
EMEL_CUDA_API emel_cuda_status emel_cuda_event_destroy(emel_cuda_context* ctx, void* event);
/* Makes `stream` wait for `event` (captured as a graph dependency: fork and
 * join of independent branches).  No counterpart in the reference. */
EMEL_CUDA_API emel_cuda_status emel_cuda_stream_wait_event(emel_cuda_context* ctx, void* stream, void* event);

/* Launch capture: every entry point called on `stream` between begin and
 * end is recorded (validated immediately, launched only on replay) into a
 * CUDA graph that emel_cuda_graph_launch replays with one host call.  This
 * is the device-side form of a fixed operator schedule such as an
 * emel-graph processor step (crates/emel-graph/src/processor/sm.rs:159-199).
 * `stream` must be a stream from emel_cuda_stream_create (not the legacy
 * default stream).  No counterpart in the reference. */
typedef struct emel_cuda_graph emel_cuda_graph;
EMEL_CUDA_API emel_cuda_status emel_cuda_graph_begin(emel_cuda_context* ctx, void* stream);
EMEL_CUDA_API emel_cuda_status emel_cuda_graph_end(emel_cuda_context* ctx, void* stream, emel_cuda_graph** out);
EMEL_CUDA_API emel_cuda_status emel_cuda_graph_launch(emel_cuda_context* ctx, emel_cuda_graph* graph, void* stream);
EMEL_CUDA_API emel_cuda_status emel_cuda_graph_destroy(emel_cuda_context* ctx, emel_cuda_graph* graph);

/* ---- binary family --------------------------------------------------- */

/* binary::OpAdd/OpSub/OpMul/OpDiv (binary.rs:47-81, guards 336-354, loop
 * 411-424): equal element counts, each operand read by logical ordinal
 * through its own layout.  F32, or F16 for all three views. */
EMEL_CUDA_API emel_cuda_status emel_cuda_binary(emel_cuda_context* ctx, void* stream, int op, const emel_tensor_view* lhs,
                                  const emel_tensor_view* rhs, const emel_tensor_view* dst);

/* broadcast::OpAddBroadcastRow / OpMulBroadcastRow (broadcast.rs:53-84,
 * guards 323-350, loops 352-390); SUB and DIV use the same contract. */
EMEL_CUDA_API emel_cuda_status emel_cuda_broadcast_row(emel_cuda_context* ctx, void* stream, int op, const emel_tensor_view* src0,
                                         const emel_tensor_view* src1, const emel_tensor_view* dst);

/* Fused ggml-style repeat + binary: generic repeat (generic.rs:1641-1665)
 * of src1 to dst's extents followed by the binary.rs formula.  src0.ne ==
 * dst.ne and every src1.ne[d] divides dst.ne[d]. */
EMEL_CUDA_API emel_cuda_status emel_cuda_binary_repeat(emel_cuda_context* ctx, void* stream, int op, const emel_tensor_view* src0,
                                         const emel_tensor_view* src1, const emel_tensor_view* dst);

/* ---- unary family ---------------------------------------------------- */

/* Typed unary events OpAbs..OpTrunc (unary.rs:72-92, guards 455-461),
 * power::OpSqr/OpSqrt (power.rs:48-63, 266-272) and reductions::OpLog/
 * OpSin/OpCos (reductions.rs:45-88, 448-466): valid views, equal element
 * counts.  F32, or F16 for both views. */
EMEL_CUDA_API emel_cuda_status emel_cuda_unary(emel_cuda_context* ctx, void* stream, int op, const emel_tensor_view* src,
                                 const emel_tensor_view* dst);

/* Generic unary::OpUnary (unary.rs:148-172, rows 276-292): only abs, neg,
 * tanh, elu, relu, gelu, silu and exp; every other subop, invalid view or
 * count mismatch reports EMEL_CUDA_UNEXPECTED_EVENT.  F32 only. */
EMEL_CUDA_API emel_cuda_status emel_cuda_op_unary(emel_cuda_context* ctx, void* stream, int subop, const emel_tensor_view* src,
                                    const emel_tensor_view* dst);

/* activation::OpScale (activation.rs:58, 366-377): dst = src * scale. */
EMEL_CUDA_API emel_cuda_status emel_cuda_scale(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                 const emel_tensor_view* dst, float scale);
/* activation::OpClamp (activation.rs:78, 403-423). */
EMEL_CUDA_API emel_cuda_status emel_cuda_clamp(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                 const emel_tensor_view* dst, float min, float max);
/* activation::OpLeakyRelu (activation.rs:507-521). */
EMEL_CUDA_API emel_cuda_status emel_cuda_leaky_relu(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                      const emel_tensor_view* dst, float negative_slope);
/* activation::OpSiluBack (activation.rs:467-481): dst = grad * silu'(src). */
EMEL_CUDA_API emel_cuda_status emel_cuda_silu_back(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                     const emel_tensor_view* grad, const emel_tensor_view* dst);
/* elementwise::OpAdd1 (elementwise.rs:280-291): dst = src + scalar. */
EMEL_CUDA_API emel_cuda_status emel_cuda_add1(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                const emel_tensor_view* dst, float scalar);
/* tensor_view::CopyTensor (tensor_view.rs:954-967, 1096-1122). */
EMEL_CUDA_API emel_cuda_status emel_cuda_copy(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                const emel_tensor_view* dst);

/* ---- row normalisation ----------------------------------------------- */

/* normalization::OpNorm (normalization.rs:58-76, guards 364-382, loop
 * 316-341): per ne0-row mean/variance normalisation, f64 accumulation. */
EMEL_CUDA_API emel_cuda_status emel_cuda_norm(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                const emel_tensor_view* dst, float eps);
/* normalization::OpRmsNorm (normalization.rs:78-96, loop 343-362). */
EMEL_CUDA_API emel_cuda_status emel_cuda_rms_norm(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                    const emel_tensor_view* dst, float eps);
/* OpRmsNorm followed by OpMulBroadcastRow with `weight` ne == [ne0,1,1,1],
 * in one pass; bit-identical to the two events run back to back. */
EMEL_CUDA_API emel_cuda_status emel_cuda_rms_norm_mul(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                        const emel_tensor_view* weight, const emel_tensor_view* dst, float eps);

/* ---- softmax --------------------------------------------------------- */

/* reductions::OpSoftMax (reductions.rs:150-163, guards 473-495, loops
 * 565-638): per ne0-row max, exp, sum (f64 for dense views, f32 otherwise),
 * divide. */
EMEL_CUDA_API emel_cuda_status emel_cuda_soft_max(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                    const emel_tensor_view* dst);
/* OpSoftMax over v = src * scale + mask (ggml soft_max_ext contract).  mask
 * may be NULL; when present it is F16 or F32 with ne0 == src ne0, ne1 >=
 * src ne1, and ne2/ne3 dividing the source extents. */
EMEL_CUDA_API emel_cuda_status emel_cuda_soft_max_ext(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                        const emel_tensor_view* mask, const emel_tensor_view* dst, float scale);

/* ---- reductions ------------------------------------------------------ */

/* reductions::OpSum (reductions.rs:90-103, 671-681): dst ne == [1,1,1,1]. */
EMEL_CUDA_API emel_cuda_status emel_cuda_sum(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                               const emel_tensor_view* dst);
/* emel_cuda_sum for callers that cannot allocate device memory.  No
 * counterpart in the reference (its kernels never touch a device).
 *
 * Who needs it: a host application that owns all device memory and hands a
 * plugin only the buffers to work on (its allocator has reserved the whole
 * device, or its contract forbids the plugin from allocating), and
 * latency-critical code that must not call cudaMalloc/cudaFree because they
 * can synchronise the device.  Such callers cannot create a context (that
 * allocates the reduction workspace), so this call takes no context: it
 * runs on the current device and enqueues on `stream` (NULL = the legacy
 * default stream).  It calls no allocating routine.
 *
 * Same validation and result as emel_cuda_sum (dst ne == [1,1,1,1], F32).
 * Its scratch is one fixed static device array -- a ticket plus 2048
 * per-block partial sums, 16.25 KiB -- that every GPU which loads this
 * library keeps until the process exits.  A device that would need more
 * than 2048 blocks (more than 512 SMs) gets EMEL_CUDA_OUT_OF_MEMORY and
 * nothing is launched.  The first call on each device looks up the array's
 * device address (cudaGetSymbolAddress with that device current); make that
 * first call before any stream capture on the device.  All calls share the
 * one array and each starts by clearing its ticket: calls whose work
 * overlaps on the GPU (other streams, other threads) race on it and can
 * return wrong sums, so issue them one after another. */
EMEL_CUDA_API emel_cuda_status emel_cuda_sum_noalloc(void* stream, const emel_tensor_view* src,
                                                     const emel_tensor_view* dst);
/* The f64 accumulator of OpSum, written to device memory `out` (one double):
 * the per-shard partial of a multi-GPU whole-tensor sum. */
EMEL_CUDA_API emel_cuda_status emel_cuda_sum_f64(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src, double* out);
/* reductions::OpMean (reductions.rs:120-133, 703-713). */
EMEL_CUDA_API emel_cuda_status emel_cuda_mean(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                const emel_tensor_view* dst);
/* reductions::OpSumRows (reductions.rs:105-118, 684-700): dst ne ==
 * [1, ne1, ne2, ne3]. */
EMEL_CUDA_API emel_cuda_status emel_cuda_sum_rows(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                    const emel_tensor_view* dst);
/* reductions::OpArgmax (reductions.rs:135-148, 715-730): first index of the
 * maximum over the whole tensor.  dst ne == [1,1,1,1]; dtype F32 (the
 * reference's index-as-f32, exact below 2^24), I32 or I64 (exact). */
EMEL_CUDA_API emel_cuda_status emel_cuda_argmax(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                  const emel_tensor_view* dst);
/* Per-shard argmax partial for multi-GPU combination, written to device
 * memory: the shard's winning value and its ordinal plus `index_base`
 * (has_value == 0 when the shard holds no comparable, non-NaN value), and
 * whether the shard's element 0 is NaN. */
typedef struct emel_cuda_argmax_partial {
    float value;
    uint32_t has_value;
    int64_t index;
    uint32_t first_is_nan;
    uint32_t reserved;
} emel_cuda_argmax_partial;
EMEL_CUDA_API emel_cuda_status emel_cuda_argmax_partial_compute(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                                  int64_t index_base, emel_cuda_argmax_partial* out);
/* Host-side combination of per-shard partials given in shard order: the
 * reference's tie rule (earliest index wins) and its NaN rule (a NaN at
 * element 0 of the whole tensor, i.e. of shard 0, pins the answer to 0). */
EMEL_CUDA_API emel_cuda_status emel_cuda_argmax_combine(const emel_cuda_argmax_partial* partials, int count, int64_t* index_out,
                                          float* value_out);
/* Per-row argmax (the reductions.rs:715-730 scan per ne0-row): dst ne ==
 * [1, ne1, ne2, ne3], dtype F32, I32 or I64; the index is the column. */
EMEL_CUDA_API emel_cuda_status emel_cuda_argmax_rows(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                       const emel_tensor_view* dst);

/* ---- row gather --------------------------------------------------------- */
/* get_rows::{OpGetRows, OpGetRowsF16, OpGetRowsBf16, OpGetRowsQ4_0,
 * OpGetRowsQ8_0, OpGetRowsQ4K} (get_rows.rs:219-512) in one entry point,
 * chosen by src->dtype (F32, F16, BF16, Q4_0, Q8_0, Q4_K): dst row r (dense
 * F32 [ne0, i0, i1, i2]) is source row indices[r] of source batch (i1, i2),
 * decoded to f32 (loops get_rows.rs:1453-1800; decoders quant.rs:106-205,
 * quant_more.rs:438-468; F16 bits as f16_matmul.rs:508-532).  indices: an I32
 * view with ne[3] == 1 (IndexView, get_rows.rs:44-215; nb[0] == 0 selects
 * contiguous strides).  Guards in the reference's order: INVALID_VIEW,
 * SHAPE_MISMATCH, UNSUPPORTED_SOURCE_STRIDE (F32 source nb[0] not 0 and
 * not a multiple of 4), then INDEX_OUT_OF_BOUNDS.  The index guard runs on
 * the device (the indices are device memory): when an index is outside
 * [0, ne1) the call still returns OK, nothing is written, and the next
 * emel_cuda_stream_synchronize on the context returns
 * EMEL_CUDA_INDEX_OUT_OF_BOUNDS (once).  No indices: a no-op after the
 * view and shape guards.  Device additions: element-aligned pointers
 * (4 bytes for F32 data and row strides, 2 for F16 / BF16 / packed),
 * else EMEL_CUDA_INVALID_ARGUMENT. */
EMEL_CUDA_API emel_cuda_status emel_cuda_get_rows(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                                  const emel_tensor_view* indices, const emel_tensor_view* dst);

/* get_rows.rs OpGetRowsF32Bytes (lines 233-255; guards 942-1003; loop
 * 1943-1979): the F32 gather over a byte-backed source (ByteTensorView,
 * tensor_view.rs:560-680) whose row, batch and outer strides may be any byte
 * count, so a row may start at any byte offset.  Guards: the byte view
 * (F32; nb[0] zero or a multiple of 4; every row's ne[0] * 4 bytes inside
 * storage_bytes; with no indices only the metadata rules) and a dense F32
 * destination -> EMEL_CUDA_INVALID_VIEW; shapes -> EMEL_CUDA_SHAPE_MISMATCH;
 * indices on the device as for emel_cuda_get_rows.  Device additions:
 * 4-byte aligned index and destination pointers (the source may have any
 * alignment), else EMEL_CUDA_INVALID_ARGUMENT. */
EMEL_CUDA_API emel_cuda_status emel_cuda_get_rows_f32_bytes(emel_cuda_context* ctx, void* stream,
                                                            const emel_tensor_view* src,
                                                            const emel_tensor_view* indices,
                                                            const emel_tensor_view* dst);

/* ---- rotary position embedding ---------------------------------------- */
/* rope::RopeParams (rope.rs:33-48). */
typedef struct emel_rope_params {
    int32_t n_dims;      /* rotated dimensions, even, <= src->ne[0] */
    int32_t mode;        /* 0 norm, 2 neox, 4 timestep (rope.rs:25-30) */
    float freq_base;
    float freq_scale;
    float ext_factor;    /* must be 0 */
    float attn_factor;
} emel_rope_params;
/* rope::OpRope (rope.rs:135-160) dispatched by RopeKernel::process_event:
 * src / dst F32 views of equal extents [cols, rows, positions, batches],
 * positions an I32 view [positions, 1, 1, 1] with explicit strides.
 * norm / neox rotate pairs (2k, 2k + 1) / (k, k + n_dims / 2) of every row
 * by theta_k = position * theta_scale^k (a binary32 product chain, theta_scale
 * = powf(freq_base, -2 / n_dims)) times freq_scale, with cos / sin scaled by
 * attn_factor and a' = fma(a, c, -(b s)), b' = fma(a, s, b c), and copy
 * columns n_dims .. cols - 1 (rope.rs:523-583); timestep (n_dims == cols,
 * dense views) writes the rotated real / imaginary halves (rope.rs:585-646).
 * Statuses in the reference's transition order: INVALID_VIEW,
 * INVALID_PARAMETERS, INVALID_MODE (shape valid, unknown mode), SHAPE_MISMATCH
 * (also timestep without its dense layout); nothing is written then.
 * Device addition: pointers must be 4-byte aligned (INVALID_ARGUMENT). */
EMEL_CUDA_API emel_cuda_status emel_cuda_rope(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                              const emel_tensor_view* positions, const emel_tensor_view* dst,
                                              const emel_rope_params* params);

/* ---- vocabulary matvec + argmax ---------------------------------------- */
/* matmul::OpMulMatArgmax (matmul.rs:167-192) dispatched by
 * MatmulArgmaxKernel::process_event (matmul.rs:969-987): lhs [k, m, 1, 1],
 * rhs [1, k, 1, 1], dst [1, 1, 1, 1], all dense F32 (matmul.rs:1416-1423,
 * 1504-1520).  The score of row r is one sequential binary32 sum of
 * lhs[r, i] * rhs[i] (separate products, the reference's order,
 * matmul.rs:3018-3052); the answer is the first row with the largest score
 * (row 0 starts the scan, a later row needs a strictly larger score).
 * Writes the best score to dst[0] and the row to *index_out (a device
 * int32; the reference returns it as the event's Ok value).  Statuses:
 * INVALID_VIEW, SHAPE_MISMATCH (nothing written).  Device additions: m <
 * 2^31, 4-byte aligned pointers, non-null index_out, else
 * INVALID_ARGUMENT.  Uses the context's reduction workspace (one call at a
 * time per context). */
EMEL_CUDA_API emel_cuda_status emel_cuda_mul_mat_argmax(emel_cuda_context* ctx, void* stream,
                                                        const emel_tensor_view* lhs, const emel_tensor_view* rhs,
                                                        const emel_tensor_view* dst, int32_t* index_out);

/* ---- diagonal family ---------------------------------------------------- */
/* diag::OpDiag::new(input, output) (diag.rs:44-66) dispatched by
 * DiagKernel::process_event: output (input_len^2 floats, row-major) becomes
 * the diagonal matrix of input, +0 off the diagonal (diag.rs:332-343).
 * input_len == 0 or output_len != input_len^2 is EMEL_CUDA_INVALID_SHAPE
 * (DiagError::InvalidShape) and writes nothing.  Device additions: a null
 * context, null or not 4-byte aligned pointers, or overlapping input and
 * output are EMEL_CUDA_INVALID_ARGUMENT.  Lengths count floats. */
EMEL_CUDA_API emel_cuda_status emel_cuda_diag(emel_cuda_context* ctx, void* stream, const float* input,
                                              uint64_t input_len, float* output, uint64_t output_len);
enum emel_diag_mask_mode { EMEL_DIAG_MASK_INF = 0, EMEL_DIAG_MASK_ZERO = 1 };
/* diag::OpDiagMaskInf / OpDiagMaskZero::new(input, output, n_past)
 * (diag.rs:68-108): for a side x side row-major matrix, output[row, col] =
 * -inf (EMEL_DIAG_MASK_INF) or +0 (EMEL_DIAG_MASK_ZERO) where col > row +
 * n_past, else input[row, col] with its bits (diag.rs:144-161).  n_past <
 * 0, input_len != output_len, or a length that is not a non-zero perfect
 * square is EMEL_CUDA_INVALID_SHAPE (mask_valid, diag.rs:122-124) and
 * writes nothing.  Device additions: an unknown mode, a null context, null
 * or not 4-byte aligned pointers, or partially overlapping slices are
 * EMEL_CUDA_INVALID_ARGUMENT; output == input (in place) is allowed. */
EMEL_CUDA_API emel_cuda_status emel_cuda_diag_mask(emel_cuda_context* ctx, void* stream, int mode,
                                                   const float* input, uint64_t input_len, float* output,
                                                   uint64_t output_len, int32_t n_past);

/* diag::OpDiagMaskInf::new(input, tmp, n_past) followed by
 * reductions::OpSoftMax over tmp as a dense [side, side] view (diag.rs:
 * 144-161, reductions.rs:565-638), in one call that reads each row's kept
 * part only: output row r is the soft_max of input[r, 0 .. r + n_past] with
 * +0 above it (the exact results of the two events; sums in binary64, so
 * within the soft_max tolerance of the sequential reference sum).  Guards
 * and device additions as emel_cuda_diag_mask; in place is allowed. */
EMEL_CUDA_API emel_cuda_status emel_cuda_soft_max_diag_mask_inf(emel_cuda_context* ctx, void* stream,
                                                                const float* input, uint64_t input_len,
                                                                float* output, uint64_t output_len, int32_t n_past);

/* ---- single-query attention ------------------------------------------- */
/* flash_attn.rs FlashAttnOptions (flash_attn.rs:24-31): has_scale == 0
 * selects 1 / sqrt(head_dim); has_masked_total_tokens == 0 selects the
 * key's token count.  A null options pointer is both defaults. */
typedef struct emel_flash_attn_options {
    float scale;
    uint32_t has_scale;
    uint32_t masked_total_tokens;
    uint32_t has_masked_total_tokens;
} emel_flash_attn_options;
/* flash_attn::OpFlashAttnExt::new(query, key, value, destination, options)
 * (flash_attn.rs:78-99) dispatched by FlashAttnKernel::process_event
 * (flash_attn.rs:198-203): query and dst F32 [head_dim, 1, heads, 1], dense
 * (flash_attn.rs:305-325); key and value F16 [head_dim, tokens, kv_heads, 1]
 * (F16View, f16_matmul.rs:45-85: any even strides on multi-element
 * dimensions); heads a multiple of kv_heads, head h reading kv head
 * h / (heads / kv_heads); head_dim <= 4096; masked_total_tokens >= tokens;
 * scale finite and > 0.  Any failed rule is EMEL_CUDA_INVALID_REQUEST and
 * nothing is written.  Per head, the reference's sequential recurrence
 * (flash_attn.rs:329-404) bit for bit: query rounded to binary16, score =
 * binary32(binary64 sum over the row of q * k) * scale, a running maximum,
 * a binary16 accumulator row rescaled when the maximum moves and updated
 * with v * round16(exp(score - max)), a binary32 score sum; out = acc /
 * sum, or 0 where the sum is 0.  Device additions: 4-byte aligned query /
 * dst and 2-byte aligned key / value pointers, heads < 2^31, else
 * EMEL_CUDA_INVALID_ARGUMENT.  One CTA per query head; allocates nothing. */
EMEL_CUDA_API emel_cuda_status emel_cuda_flash_attn_ext(emel_cuda_context* ctx, void* stream,
                                                        const emel_tensor_view* query, const emel_tensor_view* key,
                                                        const emel_tensor_view* value, const emel_tensor_view* dst,
                                                        const emel_flash_attn_options* options);
/* FlashAttnKernel::prepared_tokens / reuse_count (flash_attn.rs:205-215):
 * the token count of the context's last accepted attention call, and how
 * many accepted calls in a row repeated the token count before them. */
EMEL_CUDA_API emel_cuda_status emel_cuda_flash_attn_workspace(const emel_cuda_context* ctx,
                                                              uint64_t* prepared_tokens, uint64_t* reuse_count);

/* matmul::OpMulMatArgmaxQ8_0 (matmul.rs:500-520, routes 2958-2970): lhs
 * Q8_0 packed rows [k, m, 1, 1] (PackedRowView, tensor_view.rs:483-526:
 * nb[0] == 1, nb[1] == k / 32 * 34 bytes; k / 32 <= 1024 blocks), rhs dense
 * F32 [1, k, 1, 1], dst dense F32 [1, 1, 1, 1].  The rhs is quantized to
 * Q8_0 (quantize_q8_0, matmul.rs:1629-1653: scale = amax / 127 stored as
 * binary16, q = clamp(round(x / scale), -127, 127)); the score of row r is
 * the block-ordered binary32 sum of float(integer block dot) * (d_lhs *
 * d_rhs) (dot_q8_0, matmul.rs:1893-1910); the answer is the first row with
 * the largest score.  Writes the score to dst[0] and the row to *index_out
 * (device int32).  Statuses: INVALID_VIEW, SHAPE_MISMATCH (nothing
 * written).  Device additions: 4-byte aligned pointers, m < 2^31, non-null
 * index_out, else INVALID_ARGUMENT.  Uses the context's reduction workspace
 * (one call at a time per context). */
EMEL_CUDA_API emel_cuda_status emel_cuda_mul_mat_argmax_q8_0(emel_cuda_context* ctx, void* stream,
                                                             const emel_tensor_view* lhs, const emel_tensor_view* rhs,
                                                             const emel_tensor_view* dst, int32_t* index_out);
/* matmul::OpMulMatArgmaxQ4_0 / Q4_1 / Q5_0 (matmul.rs:490-520, routes
 * 2904-2956): the same contract with Q4_0 (18-byte blocks: binary16 scale,
 * 16 bytes of nibbles, value = nibble - 8), Q4_1 (20-byte: scale, min, 16
 * bytes, value = nibble) and Q5_0 (22-byte: scale, 32 high bits, 16 bytes,
 * value = (nibble | high << 4) - 16) rows; position i < 16 is byte i's low
 * nibble, 16 + i its high nibble.  Block terms follow dot_q4_0 / dot_q4_1 /
 * dot_q5_0 (matmul.rs:1804-1890): float(integer dot) * (d_lhs * d_rhs), and
 * for Q4_1 d_rhs * (d_lhs * float(dot) + m_lhs * float(rhs quant sum)). */
EMEL_CUDA_API emel_cuda_status emel_cuda_mul_mat_argmax_q4_0(emel_cuda_context* ctx, void* stream,
                                                             const emel_tensor_view* lhs, const emel_tensor_view* rhs,
                                                             const emel_tensor_view* dst, int32_t* index_out);
EMEL_CUDA_API emel_cuda_status emel_cuda_mul_mat_argmax_q4_1(emel_cuda_context* ctx, void* stream,
                                                             const emel_tensor_view* lhs, const emel_tensor_view* rhs,
                                                             const emel_tensor_view* dst, int32_t* index_out);
EMEL_CUDA_API emel_cuda_status emel_cuda_mul_mat_argmax_q5_0(emel_cuda_context* ctx, void* stream,
                                                             const emel_tensor_view* lhs, const emel_tensor_view* rhs,
                                                             const emel_tensor_view* dst, int32_t* index_out);
/* matmul::OpMulMatArgmaxQ4K (matmul.rs:530-535, route via
 * define_k_argmax_runner 2502-2534): Q4_K rows (144-byte blocks of 256
 * values: binary16 scale and minimum scale, 12 bytes of 6-bit group scales
 * and minimums, 128 bytes of nibbles), k / 256 <= 128 blocks.  The rhs is
 * quantized to Q8_K (quantize_q8_k, matmul.rs:1703-1745); each row keeps
 * eight lane sums (lane = position % 8) of d * float(scaled integer dots)
 * and a running total of -dmin * float(minimum sums), adding the lane sums
 * to the total after its last block (dot_q4_k, matmul.rs:2040-2114).
 * Statuses and device additions as emel_cuda_mul_mat_argmax_q8_0. */
EMEL_CUDA_API emel_cuda_status emel_cuda_mul_mat_argmax_q4_k(emel_cuda_context* ctx, void* stream,
                                                             const emel_tensor_view* lhs, const emel_tensor_view* rhs,
                                                             const emel_tensor_view* dst, int32_t* index_out);
/* matmul::OpMulMatArgmaxQ6K (matmul.rs:536-540): the same with Q6_K rows
 * (210-byte blocks: 128 bytes of low nibbles, 64 bytes of 2-bit highs, 16
 * signed group scales, binary16 scale; value = (nibble | high << 4) - 32)
 * and dot_q6_k's terms (matmul.rs:2117-2190): eight lane sums of
 * (d_rhs * d) * float(scaled integer dots), no minimum term. */
EMEL_CUDA_API emel_cuda_status emel_cuda_mul_mat_argmax_q6_k(emel_cuda_context* ctx, void* stream,
                                                             const emel_tensor_view* lhs, const emel_tensor_view* rhs,
                                                             const emel_tensor_view* dst, int32_t* index_out);
/* matmul::OpMulMatArgmaxQ2K / Q3K (matmul.rs:520-530): the same with Q2_K
 * rows (84-byte blocks: 16 bytes of 4-bit scale / minimum pairs, 64 bytes of
 * 2-bit values, binary16 scale and minimum scale; one term per block,
 * dot_q2_k, matmul.rs:1918-1962) and Q3_K rows (110-byte blocks: 32 bytes of
 * high-bit masks, 64 bytes of 2-bit values, 12 bytes of packed 6-bit
 * scales, binary16 scale; eight lane sums, dot_q3_k, matmul.rs:1994-2036). */
EMEL_CUDA_API emel_cuda_status emel_cuda_mul_mat_argmax_q2_k(emel_cuda_context* ctx, void* stream,
                                                             const emel_tensor_view* lhs, const emel_tensor_view* rhs,
                                                             const emel_tensor_view* dst, int32_t* index_out);
EMEL_CUDA_API emel_cuda_status emel_cuda_mul_mat_argmax_q3_k(emel_cuda_context* ctx, void* stream,
                                                             const emel_tensor_view* lhs, const emel_tensor_view* rhs,
                                                             const emel_tensor_view* dst, int32_t* index_out);

/* ---- shape copies ----------------------------------------------------- */
/* shape::OpCpy (shape.rs:55-69; guards 453-466, loop copy_view 438-444):
 * dst.write(i, src.read(i)) for every ordinal i of two F32 views with equal
 * element counts (extents may differ).  Invalid view -> INVALID_VIEW,
 * counts differ -> SHAPE_MISMATCH; nothing is written then.  Bits are
 * copied unchanged (NaN payloads included). */
EMEL_CUDA_API emel_cuda_status emel_cuda_cpy(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                             const emel_tensor_view* dst);
/* shape::OpCont (shape.rs:71-84; guards 492-512): OpCpy into a destination
 * whose byte strides are exactly dense row-major (Layout::is_dense_contiguous,
 * tensor_view.rs:281-314; nb[0] == 0 does not qualify), else
 * EMEL_CUDA_INVALID_LAYOUT (checked after the view and count guards). */
EMEL_CUDA_API emel_cuda_status emel_cuda_cont(emel_cuda_context* ctx, void* stream, const emel_tensor_view* src,
                                              const emel_tensor_view* dst);

/* ---- gated linear units ---------------------------------------------- */
/* glu::OpGlu::new(input, output, subop) (glu.rs:66-92) dispatched by
 * GluKernel::process_event (glu.rs:199-212): output[i] = value[i] *
 * gate(g[i]) with value = input[0, n), g = input[n, 2n), n = output_len
 * (glu.rs:114-123, 264-277).  subop: the GluSubOp wire codes (glu.rs:22-38)
 * ReGlu 0 (relu), GeGlu 1 (tanh GELU), SwiGlu 2 (silu), SwiGluOai 3
 * (silu(1.702 min(g, 7)) / 1.702 * (min(v, 7) + 1)), GeGluErf 4, GeGluQuick 5
 * (sigmoid(1.702 g)).  input_len == 0, odd, or output_len != input_len / 2
 * is EMEL_CUDA_INVALID_SHAPE (GluError::InvalidShape, glu.rs:84-91) and
 * writes nothing.  Device additions: a null context, an unknown subop, a
 * null or not 4-byte aligned pointer is EMEL_CUDA_INVALID_ARGUMENT.  input
 * and output are device arrays of f32 (elements, not bytes); output may be
 * exactly either half of input, no other overlap. */
EMEL_CUDA_API emel_cuda_status emel_cuda_glu(emel_cuda_context* ctx, void* stream, int subop, const float* input,
                                             uint64_t input_len, float* output, uint64_t output_len);

/* ---- generic operation envelope -------------------------------------- */
/* The op-coded boundary for graph-driven dispatch: GenericRequest with
 * KernelOperation wire codes (generic.rs:24-316), up to three sources, a
 * destination and the 64-byte op_params buffer (generic.rs:580-735),
 * dispatched as Kernel::process_event(GenericEvent) (actor.rs:951-960,
 * sm.rs:320-425).  Executed with the generic loops' own numerics
 * (generic.rs:1263-2050, which differ from the typed events in places:
 * GELU without binary16 rounding and with a fused cubic term, soft_max with
 * a sequential binary32 sum and no NaN pin, norms squaring in binary32):
 *   Dup 0, Add 1, Add1 3, Sub 5, Mul 6, Div 7, Sqr 8, Sqrt 9, Log 10, Sin 11,
 *   Cos 12, Sum 13, Mean 16, Argmax 17, Repeat 19, SiluBack 22, Norm 23,
 *   RmsNorm 24, Scale 32, SoftMax 46, Clamp 50, LeakyRelu 70, and Unary 85
 *   with subops Abs 0, Neg 2, Tanh 4, Elu 5, Relu 6, Gelu 8, Silu 10, Exp 13.
 * Scalars are op_params slots of 4 bytes (f32 at slot 0, clamp max at slot
 * 1, norm eps at slot 0).  Statuses follow the reference state machine: a
 * view that fails GenericRequest::validate, or a maintained operation whose
 * operands do not fit it, is EMEL_CUDA_INVALID_SHAPE; any other operation
 * code (including the reference's CPU-only routes such as Cumsum, Concat,
 * MulMat) is EMEL_CUDA_UNSUPPORTED_OPERATION.  Device addition: F32 views
 * whose data pointer or byte strides are not multiples of 4 are
 * EMEL_CUDA_INVALID_ARGUMENT (the reference reads them byte by byte). */
typedef struct emel_cuda_generic_request {
    uint32_t op;          /* KernelOperation wire code, 0..94 */
    uint32_t unary_subop; /* UnarySubOp wire code (unary.rs:101-160) when op == 85 */
    const emel_tensor_view* src0; /* nullable */
    const emel_tensor_view* src1; /* nullable */
    const emel_tensor_view* src2; /* nullable */
    const emel_tensor_view* dst;  /* nullable */
    uint8_t params[64];   /* op_params */
    uint32_t params_len;  /* initialised prefix, <= 64 (OpParams::new) */
    uint32_t reserved;
} emel_cuda_generic_request;
EMEL_CUDA_API emel_cuda_status emel_cuda_generic(emel_cuda_context* ctx, void* stream,
                                                 const emel_cuda_generic_request* request);

/* ---- graph seam: a device kernel step ---------------------------------- */
/* emel-graph's processor runs a step through RunKernelFn = fn(&ExecuteRequest,
 * &mut i32) -> bool (crates/emel-graph/src/processor/kernel_step/sm.rs:125-126).
 * The data fields of its ExecuteRequest (processor/sm.rs:170-199), in the same
 * order; handles are integers as in the reference: step_plan is an
 * emel_cuda_step and compute_ctx the emel_cuda_context it was built on. */
typedef struct emel_cuda_execute_request {
    uint64_t step_plan;
    uint64_t output_out;
    uint64_t lifecycle;
    uint64_t tensor_machine;
    int32_t step_index;
    int32_t step_size;
    int32_t kv_tokens;
    int32_t expected_outputs;
    uint64_t memory_sm;
    uint64_t memory_view;
    uint64_t compute_ctx;
} emel_cuda_execute_request;

typedef struct emel_cuda_step emel_cuda_step;
#define EMEL_CUDA_STEP_MAX_REQUESTS 4096u
/* flags: CAPTURE records the requests into one CUDA graph on the first run
 * and replays it on every later run (the views and op_params are fixed at
 * creation, as a processor step's bound tensors are); ASYNC returns from
 * emel_cuda_run_kernel without synchronising the stream (device-side
 * failures then surface at the caller's next emel_cuda_stream_synchronize). */
#define EMEL_CUDA_STEP_CAPTURE 1u
#define EMEL_CUDA_STEP_ASYNC 2u
/* A step plan: `count` generic requests (emel_cuda_generic's envelope) and
 * the views they point to, copied, to run in order on `stream`.  Requests
 * are validated when they run, one by one, exactly as emel_cuda_generic
 * validates them.  Invalid arguments (null pointers, count 0 or above
 * EMEL_CUDA_STEP_MAX_REQUESTS, unknown flags, CAPTURE on the legacy stream,
 * params_len > 64) are EMEL_CUDA_INVALID_ARGUMENT. */
EMEL_CUDA_API emel_cuda_status emel_cuda_step_create(emel_cuda_context* ctx, void* stream,
                                                     const emel_cuda_generic_request* requests, uint32_t count,
                                                     uint32_t flags, emel_cuda_step** out);
EMEL_CUDA_API emel_cuda_status emel_cuda_step_destroy(emel_cuda_context* ctx, emel_cuda_step* step);
/* Completed runs of a step (a run counts when every request succeeded). */
EMEL_CUDA_API uint64_t emel_cuda_step_runs(const emel_cuda_step* step);
/* The RunKernelFn callback (kernel_step/sm.rs:126): runs the step named by
 * request->step_plan on request->compute_ctx, synchronises its stream unless
 * the step is ASYNC, writes the emel_cuda_status to *error_out and returns
 * nonzero on success.  The first failing request stops the step; its status
 * is the one reported (nothing after it runs). */
EMEL_CUDA_API int emel_cuda_run_kernel(const emel_cuda_execute_request* request, int32_t* error_out);

/* emel-tensor's TensorLayout (crates/emel-tensor/src/lib.rs:24-50):
 * dimensions in row-major order and an ElementType.  Builds the dense view of
 * such a tensor stored at device address `data`: ne[0] is the innermost
 * (last) dimension, byte strides dense, unused dimensions 1.  Quantized
 * elements have no fixed size (the model format names the block type: build
 * those views from the GGUF tensor type) and are EMEL_CUDA_INVALID_ARGUMENT,
 * as are rank > 4 and a storage smaller than the dense span. */
#define EMEL_ELEMENT_F32 0u
#define EMEL_ELEMENT_F16 1u
#define EMEL_ELEMENT_BF16 2u
#define EMEL_ELEMENT_QUANTIZED 3u
EMEL_CUDA_API emel_cuda_status emel_cuda_layout_view(const uint64_t* dimensions, uint32_t rank, uint32_t element_type,
                                                     void* data, uint64_t storage_bytes, emel_tensor_view* out);

/* ---- GGUF tensor tables into device buffers ----------------------------- */
/* emel-gguf's loader (crates/emel-gguf/src/loader/mod.rs:137-232; scanner
 * loader/detail.rs:294-530), restated for the tensor records.  probe
 * validates a GGUF v3 image held in host memory (magic, version, every
 * metadata entry's type and bounds, general.alignment a u32 power of two,
 * unique non-empty keys and tensor names, at most 4 dimensions, known tensor
 * types, whole column groups, each tensor's offset the padded running total,
 * the data section inside the image) and returns the Requirements
 * (loader/mod.rs:15-27); parse fills one record per tensor (TensorInfo,
 * loader/mod.rs:58-84) into caller storage of at least tensor_count records.
 * Errors, with the reference's classes: EMEL_CUDA_PARSE_FAILED (truncated or
 * inconsistent offsets), EMEL_CUDA_MODEL_INVALID (unsupported or invalid
 * constructs), EMEL_CUDA_CAPACITY (counts, sizes or caller capacity),
 * EMEL_CUDA_INVALID_REQUEST (null image or requirements, or a parse whose
 * counts differ from the probe's).  Metadata values are validated and
 * skipped (the tensor table is what feeds the device). */
typedef struct emel_gguf_requirements {
    uint32_t tensor_count;
    uint32_t kv_count;
    uint32_t max_key_bytes;
    uint32_t max_value_bytes;
    uint64_t tensor_data_bytes;
} emel_gguf_requirements;
typedef struct emel_gguf_tensor_info {
    uint32_t name_offset;     /* byte offset of the name in the image */
    uint32_t name_length;
    uint32_t tensor_type;     /* GGML wire code (SerializedType) */
    uint32_t dimension_count;
    uint64_t dimensions[4];   /* ne order, unused entries 1 */
    uint64_t data_offset;     /* relative to the tensor-data section */
    uint64_t file_offset;     /* absolute in the image */
    uint64_t data_section_offset;
    uint32_t alignment;
    uint32_t reserved;
    uint64_t data_size;       /* unpadded payload bytes */
} emel_gguf_tensor_info;
EMEL_CUDA_API emel_cuda_status emel_gguf_probe(const uint8_t* image, uint64_t image_bytes,
                                               emel_gguf_requirements* out);
EMEL_CUDA_API emel_cuda_status emel_gguf_parse(const uint8_t* image, uint64_t image_bytes,
                                               const emel_gguf_requirements* probed, emel_gguf_tensor_info* tensors,
                                               uint32_t tensor_capacity);
/* The device view of a parsed tensor stored at `data`: F32, F16 and BF16 as
 * dense views; Q4_0, Q4_1, Q5_0, Q8_0, Q2_K, Q3_K, Q4_K and Q6_K as the block
 * views the row gather and the vocabulary argmax consume (ne[0] values per
 * row, nb[0] == 1, nb[1] the row's bytes).  Other GGUF types have no device
 * kernel: EMEL_CUDA_UNSUPPORTED_OPERATION.  storage_bytes below data_size is
 * EMEL_CUDA_INVALID_ARGUMENT. */
EMEL_CUDA_API emel_cuda_status emel_gguf_tensor_view(const emel_gguf_tensor_info* tensor, void* data,
                                                     uint64_t storage_bytes, emel_tensor_view* out);
/* Copies one parsed tensor's serialized bytes from the host image into
 * device memory `device_dst` (stream-ordered, like emel_cuda_memcpy_h2d)
 * and writes its view (emel_gguf_tensor_view). */
EMEL_CUDA_API emel_cuda_status emel_gguf_upload(emel_cuda_context* ctx, void* stream, const uint8_t* image,
                                                uint64_t image_bytes, const emel_gguf_tensor_info* tensor,
                                                void* device_dst, uint64_t device_bytes, emel_tensor_view* view_out);

/* ---- peer exchange over NVLink (multi-GPU partials) -------------------- */
/* One process per GPU shards a tensor; each rank's small partial (the f64
 * sum and the emel_cuda_argmax_partial of its shard) must reach every rank.
 * No counterpart in the reference (a single-process CPU library): this
 * replaces the collective of the sharded plan.  Every rank creates an
 * exchange with the same world size and payload size, shares the 64-byte
 * handle of its buffer with the others (any host channel), and connects
 * with all handles in rank order.  Then, per step and on a stream:
 *   emel_cuda_exchange_publish stores this rank's payload into every rank's
 *     buffer over NVLink (peer stores, release flag at system scope);
 *   emel_cuda_exchange_wait waits (bounded by timeout_ms) until every rank
 *     published the same step, then writes all payloads, rank order, to
 *     `gathered`.  A wait that expires sets the context's fault word:
 *     emel_cuda_stream_synchronize returns EMEL_CUDA_TIMEOUT.
 * Publish/wait calls alternate, one pair per step on every rank (a device
 * counter numbers the steps, so a captured graph may replay them).
 * payload and gathered are device pointers, 16-byte aligned; bytes_per_rank
 * is a multiple of 16, at most 1024; world is 1..64.  Destroy only after
 * every rank's last wait has completed (a host barrier). */
typedef struct emel_cuda_exchange emel_cuda_exchange;
#define EMEL_CUDA_EXCHANGE_HANDLE_BYTES 64
EMEL_CUDA_API emel_cuda_status emel_cuda_exchange_create(emel_cuda_context* ctx, int world, int rank,
                                                         uint32_t bytes_per_rank, uint32_t timeout_ms,
                                                         emel_cuda_exchange** out);
EMEL_CUDA_API emel_cuda_status emel_cuda_exchange_handle(const emel_cuda_exchange* ex, void* handle_out);
EMEL_CUDA_API emel_cuda_status emel_cuda_exchange_connect(emel_cuda_context* ctx, emel_cuda_exchange* ex,
                                                          const void* handles);
EMEL_CUDA_API emel_cuda_status emel_cuda_exchange_publish(emel_cuda_context* ctx, void* stream, emel_cuda_exchange* ex,
                                                          const void* payload);
EMEL_CUDA_API emel_cuda_status emel_cuda_exchange_wait(emel_cuda_context* ctx, void* stream, emel_cuda_exchange* ex,
                                                       void* gathered);
/* The wait above for the sharded whole-tensor reductions, with the combine
 * done on the device in the same kernel: the payload of every rank is its
 * emel_cuda_sum_f64 result followed by its emel_cuda_argmax_partial
 * (bytes_per_rank == 32).  After the gather, the f64 sums are added in rank
 * order and rounded once to f32 into sum_dst (OpSum, reductions.rs:671-681,
 * one f64 accumulator over the whole tensor), and the argmax index is
 * written to argmax_dst (OpArgmax, reductions.rs:715-730: a later shard wins
 * only with a strictly greater value; a NaN at element 0 of the whole
 * tensor, or no comparable value, gives index 0).  sum_dst is an F32 view and
 * argmax_dst an F32 / I32 / I64 view, both of ne [1,1,1,1]; views are
 * checked like emel_cuda_sum's and emel_cuda_argmax's destinations. */
EMEL_CUDA_API emel_cuda_status emel_cuda_exchange_wait_sum_argmax(emel_cuda_context* ctx, void* stream,
                                                                  emel_cuda_exchange* ex, void* gathered,
                                                                  const emel_tensor_view* sum_dst,
                                                                  const emel_tensor_view* argmax_dst);
EMEL_CUDA_API emel_cuda_status emel_cuda_exchange_destroy(emel_cuda_context* ctx, emel_cuda_exchange* ex);

#ifdef __cplusplus
}
#endif

#endif /* EMEL_CUDA_H */
