/*
 * emel_oracle.c -- CPU restatement of the emel-kernels elementwise, broadcast
 * and reduction hot path.  TEST INFRASTRUCTURE ONLY (parity checker and timed
 * CPU baseline); see emel_oracle.h.
 *
 * Citations are paths inside stateforward/emel.rs.  Build flags matter:
 * -O2 -ffp-contract=off -fno-fast-math -fno-math-errno, x86-64 SSE scalar
 * arithmetic, glibc libm for expf/tanhf/expm1f/log1pf/logf/sinf/cosf (the
 * functions Rust's f32::{exp,tanh,exp_m1,ln_1p,ln,sin,cos} call on Linux).
 */
#include "emel_oracle.h"

#include <math.h>
#include <stdint.h>
#include <string.h>

typedef unsigned __int128 u128;

/* The reference's f32 libm calls.  By default they are the host's glibc
 * float functions (what Rust's f32::exp etc. call on Linux).  Built with
 * -DORACLE_CR_LIBM they are evaluated in binary64 and rounded once, i.e. the
 * reference loops running on a platform whose float libm is correctly
 * rounded (as glibc's newer float functions are): the device kernels, which
 * evaluate the same way, must match that build bit for bit. */
#ifdef ORACLE_CR_LIBM
#define expf(x) ((float)exp((double)(x)))
#define expm1f(x) ((float)expm1((double)(x)))
#define tanhf(x) ((float)tanh((double)(x)))
#define log1pf(x) ((float)log1p((double)(x)))
#define logf(x) ((float)log((double)(x)))
#define sinf(x) ((float)sin((double)(x)))
#define cosf(x) ((float)cos((double)(x)))
#endif

enum { DT_F32 = 0, DT_F16 = 1, DT_I32 = 26, DT_I64 = 27 };

/* ---------------------------------------------------------------------- */
/* Layout rules: crates/emel-kernels/src/any/tensor_view.rs                */
/* ---------------------------------------------------------------------- */

static uint64_t dtype_size(uint32_t dtype) {
    switch (dtype) {
    case DT_F32: return 4;
    case DT_F16: return 2;
    case DT_I32: return 4;
    case DT_I64: return 8;
    default: return 0;
    }
}

/* Layout::element_count (tensor_view.rs:346-358): zero extent or overflow -> none. */
static int element_count(const oracle_view* v, uint64_t* out) {
    uint64_t count = 1;
    for (int d = 0; d < 4; ++d) {
        if (v->ne[d] == 0) return 0;
        if (__builtin_mul_overflow(count, v->ne[d], &count)) return 0;
    }
    *out = count;
    return 1;
}

/* Layout::effective_f32_strides (tensor_view.rs:262-277), generalised to the
 * element size of the view's dtype: nb[0]==0 means implicit row-major. */
static int effective_strides(const oracle_view* v, uint64_t elem, uint64_t s[4]) {
    if (v->nb[0] != 0) {
        memcpy(s, v->nb, sizeof(uint64_t) * 4);
        return 1;
    }
    s[0] = elem;
    for (int d = 1; d < 4; ++d)
        if (__builtin_mul_overflow(s[d - 1], v->ne[d - 1], &s[d])) return 0;
    return 1;
}

/* Layout::validate_element_storage (tensor_view.rs:392-447).  Returns 1 when
 * the view is valid for `dtype`; strides must be >= and a multiple of the
 * element size (an explicit zero stride on a singleton dimension is allowed
 * only under the binary contract), and the whole byte span must fit. */
static int validate_as(const oracle_view* v, uint32_t dtype, int allow_singleton_zero, uint64_t* count_out) {
    if (v == NULL || v->dtype != dtype) return 0;
    uint64_t elem = dtype_size(dtype);
    uint64_t count;
    if (!element_count(v, &count)) return 0;
    uint64_t s[4];
    if (!effective_strides(v, elem, s)) return 0;
    for (int d = 0; d < 4; ++d) {
        int singleton_zero = allow_singleton_zero && v->ne[d] == 1 && s[d] == 0;
        if (!singleton_zero && (s[d] < elem || s[d] % elem != 0)) return 0;
    }
    u128 max_offset = 0;
    for (int d = 0; d < 4; ++d) max_offset += (u128)(v->ne[d] - 1) * (u128)s[d];
    u128 end = max_offset + elem;
    if (end > (u128)v->storage_bytes) return 0;
    if (count_out) *count_out = count;
    return 1;
}

/* Float views: F32 always; F16 as this build's extension of the same rule. */
static int validate_float(const oracle_view* v, int allow_singleton_zero, uint64_t* count) {
    if (v == NULL) return 0;
    if (v->dtype != DT_F32 && v->dtype != DT_F16) return 0;
    return validate_as(v, v->dtype, allow_singleton_zero, count);
}

/* normalization_view_valid (normalization.rs:237-287). */
static int normalization_view_valid(const oracle_view* v) {
    if (v == NULL || v->dtype != DT_F32 || v->ne[0] == 0) return 0;
    if (v->nb[0] != 0) {
        if (v->nb[0] < 4 || v->nb[0] % 4 != 0) return 0;
        for (int d = 0; d < 4; ++d)
            if (v->ne[d] > 1 && v->nb[d] == 0) return 0;
    }
    for (int d = 0; d < 4; ++d)
        if (v->ne[d] == 0) return 0;
    uint64_t s[4];
    if (!effective_strides(v, 4, s)) return 0;
    for (int d = 0; d < 4; ++d)
        if (s[d] < 4 || s[d] % 4 != 0) return 0;
    u128 max_offset = 0;
    for (int d = 0; d < 4; ++d) max_offset += (u128)(v->ne[d] - 1) * (u128)s[d];
    return max_offset + 4 <= (u128)v->storage_bytes;
}

static int same_ne(const oracle_view* a, const oracle_view* b) {
    return memcmp(a->ne, b->ne, sizeof(uint64_t) * 4) == 0;
}

/* Layout::is_dense_contiguous_for (tensor_view.rs:297-314). */
static int is_dense(const oracle_view* v, uint64_t elem) {
    uint64_t expected = elem;
    for (int d = 0; d < 4; ++d) {
        if (v->nb[d] != expected) return 0;
        if (__builtin_mul_overflow(expected, v->ne[d], &expected)) return 0;
    }
    return 1;
}

/* TensorView::element_index (tensor_view.rs:778-789): logical ordinal ->
 * byte offset through each dimension's extent and effective stride. */
static uint64_t ordinal_offset(const oracle_view* v, const uint64_t s[4], uint64_t ordinal) {
    uint64_t off = 0;
    for (int d = 0; d < 4; ++d) {
        off += (ordinal % v->ne[d]) * s[d];
        ordinal /= v->ne[d];
    }
    return off;
}

/* Incremental form of ordinal_offset for consecutive ordinals: the same
 * ordinal -> offset map walked in ordinal order without per-element
 * division (dimension 0 fastest, carries into 1, 2, 3). */
typedef struct walker {
    uint64_t ne[4], s[4], c[4], off;
} walker;

static void walker_init(walker* w, const oracle_view* v, const uint64_t s[4], uint64_t ordinal) {
    w->off = 0;
    for (int d = 0; d < 4; ++d) {
        w->ne[d] = v->ne[d];
        w->s[d] = s[d];
        w->c[d] = ordinal % v->ne[d];
        ordinal /= v->ne[d];
        w->off += w->c[d] * s[d];
    }
}

static inline void walker_next(walker* w) {
    for (int d = 0; d < 4; ++d) {
        w->off += w->s[d];
        if (++w->c[d] < w->ne[d]) return;
        w->off -= w->ne[d] * w->s[d];
        w->c[d] = 0;
    }
}

/* Reference binary16 helpers (unary.rs:546-586), kept step for step because
 * the GELU path rounds through them and their results are part of parity. */
static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

uint16_t oracle_fp32_to_fp16(float value) {
    const float scale_to_inf = u2f(0x77800000u);
    const float scale_to_zero = u2f(0x08800000u);
    float base = (fabsf(value) * scale_to_inf) * scale_to_zero;
    uint32_t word = f2u(value);
    uint32_t doubled = word + word;
    uint32_t sign = word & 0x80000000u;
    uint32_t bias = doubled & 0xff000000u;
    if (bias < 0x71000000u) bias = 0x71000000u;
    base += u2f((bias >> 1) + 0x07800000u);
    uint32_t base_bits = f2u(base);
    uint32_t exponent = (base_bits >> 13) & 0x00007c00u;
    uint32_t mantissa = base_bits & 0x00000fffu;
    uint32_t nonsign = exponent + mantissa;
    return (uint16_t)((sign >> 16) | (doubled > 0xff000000u ? 0x7e00u : nonsign));
}

float oracle_fp16_to_fp32(uint16_t bits16) {
    uint32_t word = (uint32_t)bits16 << 16;
    uint32_t sign = word & 0x80000000u;
    uint32_t doubled = word + word;
    uint32_t exp_offset = 0xe0u << 23;
    float normalized = u2f((doubled >> 4) + exp_offset) * u2f(0x07800000u);
    float denormalized = u2f((doubled >> 17) | (126u << 23)) - 0.5f;
    uint32_t result = doubled < (1u << 27) ? (sign | f2u(denormalized)) : (sign | f2u(normalized));
    return u2f(result);
}

/* Element accessors for F32/F16 storage. */
static inline float load_f(const oracle_view* v, uint64_t off) {
    const unsigned char* p = (const unsigned char*)v->data + off;
    if (v->dtype == DT_F16) {
        uint16_t h;
        memcpy(&h, p, 2);
        return oracle_fp16_to_fp32(h);
    }
    float f;
    memcpy(&f, p, 4);
    return f;
}

static inline void store_f(const oracle_view* v, uint64_t off, float value) {
    unsigned char* p = (unsigned char*)v->data + off;
    if (v->dtype == DT_F16) {
        uint16_t h = oracle_fp32_to_fp16(value);
        memcpy(p, &h, 2);
        return;
    }
    memcpy(p, &value, 4);
}

/* ---------------------------------------------------------------------- */
/* Binary family                                                          */
/* ---------------------------------------------------------------------- */

/* Formulas: binary.rs:386-409. */
static inline float binary_apply(int op, float a, float b) {
    switch (op) {
    case ORACLE_ADD: return a + b;
    case ORACLE_SUB: return a - b;
    case ORACLE_MUL: return a * b;
    default: return a / b;
    }
}

static int all_same_float_dtype(const oracle_view* a, const oracle_view* b, const oracle_view* c) {
    return a->dtype == b->dtype && a->dtype == c->dtype;
}

/* binary.rs:336-354 guards, 411-424 loop: every output ordinal reads the
 * same ordinal of each operand through its own layout. */
int oracle_binary(int op, const oracle_view* lhs, const oracle_view* rhs, const oracle_view* dst) {
    if (op < ORACLE_ADD || op > ORACLE_DIV) return ORACLE_UNEXPECTED_EVENT;
    uint64_t nl, nr, nd;
    if (!validate_float(lhs, 1, &nl) || !validate_float(rhs, 1, &nr) || !validate_float(dst, 1, &nd) ||
        !all_same_float_dtype(lhs, rhs, dst))
        return ORACLE_INVALID_VIEW;
    if (nl != nr || nl != nd) return ORACLE_SHAPE_MISMATCH;
    uint64_t sl[4], sr[4], sd[4];
    effective_strides(lhs, dtype_size(lhs->dtype), sl);
    effective_strides(rhs, dtype_size(rhs->dtype), sr);
    effective_strides(dst, dtype_size(dst->dtype), sd);
    walker wl, wr, wd;
    walker_init(&wl, lhs, sl, 0);
    walker_init(&wr, rhs, sr, 0);
    walker_init(&wd, dst, sd, 0);
    for (uint64_t i = 0; i < nd; ++i) {
        float a = load_f(lhs, wl.off);
        float b = load_f(rhs, wr.off);
        store_f(dst, wd.off, binary_apply(op, a, b));
        walker_next(&wl);
        walker_next(&wr);
        walker_next(&wd);
    }
    return ORACLE_OK;
}

/* broadcast.rs:323-350 guards, 352-390 loops (add/mul; sub/div use the
 * same loop with the binary.rs formula). */
int oracle_broadcast_row(int op, const oracle_view* src0, const oracle_view* src1, const oracle_view* dst) {
    if (op < ORACLE_ADD || op > ORACLE_DIV) return ORACLE_UNEXPECTED_EVENT;
    uint64_t n0, n1, nd;
    if (!validate_float(src0, 1, &n0) || !validate_float(src1, 1, &n1) || !validate_float(dst, 1, &nd) ||
        !all_same_float_dtype(src0, src1, dst))
        return ORACLE_INVALID_VIEW;
    if (!(same_ne(src0, dst) && dst->ne[0] > 0 && src1->ne[0] == dst->ne[0] && src1->ne[1] == 1 &&
          src1->ne[2] == 1 && src1->ne[3] == 1 && dst->ne[1] > 0 && nd > n1))
        return ORACLE_SHAPE_MISMATCH;
    uint64_t s0[4], s1[4], sd[4];
    effective_strides(src0, dtype_size(src0->dtype), s0);
    effective_strides(src1, dtype_size(src1->dtype), s1);
    effective_strides(dst, dtype_size(dst->dtype), sd);
    uint64_t columns = n1, rows = nd / columns;
    walker w0, wd, w1;
    walker_init(&w0, src0, s0, 0);
    walker_init(&wd, dst, sd, 0);
    for (uint64_t r = 0; r < rows; ++r) {
        walker_init(&w1, src1, s1, 0);
        for (uint64_t c = 0; c < columns; ++c) {
            float a = load_f(src0, w0.off);
            float b = load_f(src1, w1.off);
            store_f(dst, wd.off, binary_apply(op, a, b));
            walker_next(&w0);
            walker_next(&w1);
            walker_next(&wd);
        }
    }
    return ORACLE_OK;
}

/* generic.rs:1641-1665 (repeat: dst coordinate % source extent) composed
 * with binary.rs:386-424.  src0 and dst share extents; every src1 extent
 * divides the dst extent (the ggml repeat contract). */
int oracle_binary_repeat(int op, const oracle_view* src0, const oracle_view* src1, const oracle_view* dst) {
    if (op < ORACLE_ADD || op > ORACLE_DIV) return ORACLE_UNEXPECTED_EVENT;
    uint64_t n0, n1, nd;
    if (!validate_float(src0, 1, &n0) || !validate_float(src1, 1, &n1) || !validate_float(dst, 1, &nd) ||
        !all_same_float_dtype(src0, src1, dst))
        return ORACLE_INVALID_VIEW;
    if (!same_ne(src0, dst)) return ORACLE_SHAPE_MISMATCH;
    for (int d = 0; d < 4; ++d)
        if (dst->ne[d] % src1->ne[d] != 0) return ORACLE_SHAPE_MISMATCH;
    uint64_t s0[4], s1[4], sd[4];
    effective_strides(src0, dtype_size(src0->dtype), s0);
    effective_strides(src1, dtype_size(src1->dtype), s1);
    effective_strides(dst, dtype_size(dst->dtype), sd);
    walker w0, wd;
    walker_init(&w0, src0, s0, 0);
    walker_init(&wd, dst, sd, 0);
    for (uint64_t i = 0; i < nd; ++i) {
        /* wd.c holds dst's coordinates of ordinal i */
        uint64_t off1 = 0;
        for (int d = 0; d < 4; ++d) off1 += (wd.c[d] % src1->ne[d]) * s1[d];
        float a = load_f(src0, w0.off);
        float b = load_f(src1, off1);
        store_f(dst, wd.off, binary_apply(op, a, b));
        walker_next(&w0);
        walker_next(&wd);
    }
    return ORACLE_OK;
}

/* ---------------------------------------------------------------------- */
/* Unary family                                                            */
/* ---------------------------------------------------------------------- */

enum {
    U_ABS = 0, U_SGN = 1, U_NEG = 2, U_STEP = 3, U_TANH = 4, U_ELU = 5, U_RELU = 6, U_SIGMOID = 7,
    U_GELU = 8, U_GELU_QUICK = 9, U_SILU = 10, U_HARDSWISH = 11, U_HARDSIGMOID = 12, U_EXP = 13,
    U_EXPM1 = 14, U_SOFTPLUS = 15, U_GELU_ERF = 16, U_XIELU = 17, U_FLOOR = 18, U_CEIL = 19,
    U_ROUND = 20, U_TRUNC = 21,
    U_SQR = 64, U_SQRT = 65, U_LOG = 66, U_SIN = 67, U_COS = 68
};

/* Rust's f32::clamp keeps NaN; both comparisons are false for it. */
static inline float clampf_rs(float v, float lo, float hi) {
    if (v < lo) return lo;
    if (v > hi) return hi;
    return v;
}

/* Formulas: unary.rs:474-672, power.rs:315 and 397-412, reductions.rs:640-668. */
static inline float unary_apply(int op, float v) {
    switch (op) {
    case U_ABS: return fabsf(v);
    case U_SGN: return isnan(v) ? NAN : copysignf(1.0f, v); /* f32::signum: NaN -> f32::NAN */
    case U_NEG: return -v;
    case U_STEP: return v > 0.0f ? 1.0f : 0.0f;
    case U_TANH: return tanhf(v);
    case U_ELU: return v >= 0.0f ? v : expm1f(v);
    case U_RELU: return isnan(v) ? 0.0f : (v > 0.0f ? v : 0.0f); /* f32::max(0.0) */
    case U_SIGMOID: return 1.0f / (1.0f + expf(-v));
    case U_GELU: {
        if (v <= -10.0f) return 0.0f;
        if (v >= 10.0f) return v;
        float q = oracle_fp16_to_fp32(oracle_fp32_to_fp16(v));
        float inner = 0.7978846f * (q + 0.044715f * q * q * q);
        float approximation = 0.5f * q * (1.0f + tanhf(inner));
        return oracle_fp16_to_fp32(oracle_fp32_to_fp16(approximation));
    }
    case U_GELU_QUICK: return 0.5f * v * (1.0f + tanhf(0.7978846f * v * (1.0f + 0.044715f * v * v)));
    case U_SILU: return v / (1.0f + expf(-v));
    case U_HARDSWISH: return v * clampf_rs(v + 3.0f, 0.0f, 6.0f) / 6.0f;
    case U_HARDSIGMOID: return clampf_rs(v + 3.0f, 0.0f, 6.0f) / 6.0f;
    case U_EXP: return expf(v);
    case U_EXPM1: return expm1f(v);
    case U_SOFTPLUS: return log1pf(expf(v));
    case U_GELU_ERF: {
        float sign = v < 0.0f ? -1.0f : 1.0f;
        float x = fabsf(v) / 1.41421356237309504880f;
        float t = 1.0f / (1.0f + 0.3275911f * x);
        float polynomial = (((((1.0614054f * t - 1.4531521f) * t) + 1.4214138f) * t - 0.28449672f) * t + 0.2548296f) * t;
        float erf = sign * (1.0f - polynomial * expf(-x * x));
        return 0.5f * v * (1.0f + erf);
    }
    case U_FLOOR: return floorf(v);
    case U_CEIL: return ceilf(v);
    case U_ROUND: return roundf(v);
    case U_TRUNC: return truncf(v);
    case U_SQR: return v * v;
    case U_SQRT: return sqrtf(v);
    case U_LOG: return logf(v);
    case U_SIN: return sinf(v);
    case U_COS: return cosf(v);
    default: return v;
    }
}

static int unary_op_known(int op) {
    return (op >= U_ABS && op <= U_TRUNC && op != U_XIELU) || (op >= U_SQR && op <= U_COS);
}

/* unary.rs:455-461 guards (both views valid, equal element counts) and the
 * ordinal loop of unary.rs:674-685.  The same guard shape is used by
 * power.rs:266-272 and reductions.rs:448-466. */
static int unary_views(const oracle_view* src, const oracle_view* dst, uint64_t* count) {
    uint64_t ns, nd;
    if (!validate_float(src, 0, &ns) || !validate_float(dst, 0, &nd) || src->dtype != dst->dtype)
        return ORACLE_INVALID_VIEW;
    if (ns != nd) return ORACLE_SHAPE_MISMATCH;
    *count = ns;
    return ORACLE_OK;
}

void oracle_unary_range(int op, const oracle_view* src, const oracle_view* dst, uint64_t begin, uint64_t end) {
    uint64_t ss[4], sd[4];
    effective_strides(src, dtype_size(src->dtype), ss);
    effective_strides(dst, dtype_size(dst->dtype), sd);
    walker ws, wd;
    walker_init(&ws, src, ss, begin);
    walker_init(&wd, dst, sd, begin);
    for (uint64_t i = begin; i < end; ++i) {
        store_f(dst, wd.off, unary_apply(op, load_f(src, ws.off)));
        walker_next(&ws);
        walker_next(&wd);
    }
}

int oracle_unary(int op, const oracle_view* src, const oracle_view* dst) {
    if (!unary_op_known(op)) return ORACLE_UNEXPECTED_EVENT;
    uint64_t count;
    int st = unary_views(src, dst, &count);
    if (st != ORACLE_OK) return st;
    oracle_unary_range(op, src, dst, 0, count);
    return ORACLE_OK;
}

/* Generic OpUnary (unary.rs:276-292, 942-1027): eight accepted subops; any
 * other subop, invalid view or count mismatch reports UnexpectedEvent. */
int oracle_op_unary(int subop, const oracle_view* src, const oracle_view* dst) {
    int accepted = subop == U_ABS || subop == U_NEG || subop == U_TANH || subop == U_ELU ||
                   subop == U_RELU || subop == U_GELU || subop == U_SILU || subop == U_EXP;
    uint64_t ns, nd;
    if (!accepted || !validate_as(src, DT_F32, 0, &ns) || !validate_as(dst, DT_F32, 0, &nd) || ns != nd)
        return ORACLE_UNEXPECTED_EVENT;
    oracle_unary_range(subop, src, dst, 0, ns);
    return ORACLE_OK;
}

/* activation.rs:327-333 guards (valid views, identical extents). */
static int same_shape_views(const oracle_view* src, const oracle_view* dst, uint64_t* count) {
    uint64_t ns, nd;
    if (!validate_as(src, DT_F32, 0, &ns) || !validate_as(dst, DT_F32, 0, &nd)) return ORACLE_INVALID_VIEW;
    if (!same_ne(src, dst)) return ORACLE_SHAPE_MISMATCH;
    *count = ns;
    return ORACLE_OK;
}

#define ORACLE_MAP(src, dst, count, expr)                                                  \
    do {                                                                                   \
        uint64_t ss_[4], sd_[4];                                                           \
        walker ws_, wd_;                                                                   \
        effective_strides(src, 4, ss_);                                                    \
        effective_strides(dst, 4, sd_);                                                    \
        walker_init(&ws_, src, ss_, 0);                                                    \
        walker_init(&wd_, dst, sd_, 0);                                                    \
        for (uint64_t i_ = 0; i_ < (count); ++i_) {                                        \
            float v = load_f(src, ws_.off);                                                \
            store_f(dst, wd_.off, (expr));                                                 \
            walker_next(&ws_);                                                             \
            walker_next(&wd_);                                                             \
        }                                                                                  \
    } while (0)

/* activation.rs:366-377 */
int oracle_scale(const oracle_view* src, const oracle_view* dst, float scale) {
    uint64_t n;
    int st = same_shape_views(src, dst, &n);
    if (st != ORACLE_OK) return st;
    ORACLE_MAP(src, dst, n, v * scale);
    return ORACLE_OK;
}

/* activation.rs:403-423 (std::clamp comparison contract; NaN passes). */
int oracle_clamp(const oracle_view* src, const oracle_view* dst, float lo, float hi) {
    uint64_t n;
    int st = same_shape_views(src, dst, &n);
    if (st != ORACLE_OK) return st;
    ORACLE_MAP(src, dst, n, (v < lo ? lo : (v > hi ? hi : v)));
    return ORACLE_OK;
}

/* activation.rs:507-521 */
int oracle_leaky_relu(const oracle_view* src, const oracle_view* dst, float slope) {
    uint64_t n;
    int st = same_shape_views(src, dst, &n);
    if (st != ORACLE_OK) return st;
    ORACLE_MAP(src, dst, n, (v < 0.0f ? v * slope : v));
    return ORACLE_OK;
}

/* activation.rs:335-349 guards (three valid views, identical extents),
 * 467-481 loop. */
int oracle_silu_back(const oracle_view* src, const oracle_view* grad, const oracle_view* dst) {
    uint64_t n, ng;
    if (!validate_as(src, DT_F32, 0, &n) || !validate_as(grad, DT_F32, 0, &ng) || !validate_as(dst, DT_F32, 0, NULL))
        return ORACLE_INVALID_VIEW;
    if (!same_ne(src, grad) || !same_ne(src, dst)) return ORACLE_SHAPE_MISMATCH;
    uint64_t ss[4], sg[4], sd[4];
    effective_strides(src, 4, ss);
    effective_strides(grad, 4, sg);
    effective_strides(dst, 4, sd);
    walker ws, wg, wd;
    walker_init(&ws, src, ss, 0);
    walker_init(&wg, grad, sg, 0);
    walker_init(&wd, dst, sd, 0);
    for (uint64_t i = 0; i < n; ++i) {
        float v = load_f(src, ws.off);
        float sigmoid = 1.0f / (1.0f + expf(-v));
        float derivative = sigmoid * (1.0f + v * (1.0f - sigmoid));
        store_f(dst, wd.off, load_f(grad, wg.off) * derivative);
        walker_next(&ws);
        walker_next(&wg);
        walker_next(&wd);
    }
    return ORACLE_OK;
}

/* Gated linear units: glu.rs:84-91 (split_len), 99-127 (gates), 114-123
 * (apply_split), 264-277 (SwiGluOai).  f32::max(0.0) / f32::min(7.0) are
 * written as the comparisons x86's maxss / minss perform with the constant
 * as second operand (a NaN or tied input yields the constant). */
static float glu_one(int subop, float value, float g) {
    switch (subop) {
    case 0: return value * (g > 0.0f ? g : 0.0f);
    case 1: return value * unary_apply(U_GELU_QUICK, g);
    case 2: return value * unary_apply(U_SILU, g);
    case 3: {
        float gate = g < 7.0f ? g : 7.0f;
        float v = value < 7.0f ? value : 7.0f;
        return unary_apply(U_SILU, 1.702f * gate) / 1.702f * (v + 1.0f);
    }
    case 4: return value * unary_apply(U_GELU_ERF, g);
    default: return value * (1.0f / (1.0f + expf(-1.702f * g)));
    }
}

int oracle_glu(int subop, const float* input, uint64_t input_len, float* output, uint64_t output_len) {
    if (subop < 0 || subop > 5) return ORACLE_UNEXPECTED_EVENT; /* not expressible in the reference */
    if (input_len == 0 || input_len % 2 != 0 || output_len != input_len / 2) return ORACLE_INVALID_SHAPE;
    const uint64_t n = output_len;
    for (uint64_t i = 0; i < n; ++i) output[i] = glu_one(subop, input[i], input[n + i]);
    return ORACLE_OK;
}

/* ---------------------------------------------------------------------- */
/* Diagonal family: diag.rs OpDiag / OpDiagMaskInf / OpDiagMaskZero        */
/* ---------------------------------------------------------------------- */

/* square_side (diag.rs:107-120): the side of a non-empty perfect square. */
static int diag_square_side(uint64_t len, uint64_t* side) {
    if (len == 0) return 0;
    uint64_t s = (uint64_t)sqrt((double)len);
    while (s > 0 && s * s > len) --s;
    while ((s + 1) * (s + 1) <= len) ++s;
    if (s * s != len) return 0;
    *side = s;
    return 1;
}

/* OpDiag::side (diag.rs:56-65) and effect_diag (diag.rs:332-343): output
 * filled with +0, then output[i * n + i] = input[i]. */
int oracle_diag(const float* input, uint64_t input_len, float* output, uint64_t output_len) {
    const uint64_t n = input_len;
    uint64_t nn;
    if (n == 0 || __builtin_mul_overflow(n, n, &nn) || output_len != nn) return ORACLE_INVALID_SHAPE;
    for (uint64_t i = 0; i < nn; ++i) output[i] = 0.0f;
    for (uint64_t i = 0; i < n; ++i) output[i * n + i] = input[i];
    return ORACLE_OK;
}

/* mask_valid (diag.rs:122-124) and apply_mask (diag.rs:144-161): mode 0
 * writes -inf, mode 1 writes +0 where col > row + n_past; elsewhere the
 * input element (bits unchanged). */
int oracle_diag_mask(int mode, const float* input, uint64_t input_len, float* output, uint64_t output_len,
                     int32_t n_past) {
    uint64_t side;
    if (mode != 0 && mode != 1) return ORACLE_UNEXPECTED_EVENT;
    if (n_past < 0 || input_len != output_len || !diag_square_side(input_len, &side)) return ORACLE_INVALID_SHAPE;
    const float masked = mode == 0 ? -INFINITY : 0.0f;
    for (uint64_t row = 0; row < side; ++row)
        for (uint64_t col = 0; col < side; ++col) {
            const uint64_t i = row * side + col;
            if (col > row + (uint64_t)n_past)
                output[i] = masked;
            else
                memcpy(&output[i], &input[i], 4);
        }
    return ORACLE_OK;
}

/* elementwise.rs:219-225 guards, 280-291 loop. */
int oracle_add1(const oracle_view* src, const oracle_view* dst, float scalar) {
    uint64_t n;
    int st = same_shape_views(src, dst, &n);
    if (st != ORACLE_OK) return st;
    ORACLE_MAP(src, dst, n, v + scalar);
    return ORACLE_OK;
}

/* tensor_view.rs:1096-1122 (CopyTensor: valid views, identical extents). */
int oracle_copy(const oracle_view* src, const oracle_view* dst) {
    uint64_t n;
    int st = same_shape_views(src, dst, &n);
    if (st != ORACLE_OK) return st;
    ORACLE_MAP(src, dst, n, v);
    return ORACLE_OK;
}

/* shape.rs: OpCpy (guards 453-466, copy_view 438-444) copies by ordinal
 * between count-equal views of any extents; OpCont (guards 492-512)
 * additionally requires a destination whose byte strides are exactly the
 * dense row-major ones (Layout::is_dense_contiguous, tensor_view.rs:281-314:
 * the implicit nb[0] == 0 form does not qualify). */
static int dense_contiguous_f32(const oracle_view* v) {
    if (v->dtype != DT_F32) return 0;
    uint64_t expected = 4;
    for (int d = 0; d < 4; ++d) {
        if (v->nb[d] != expected) return 0;
        if (__builtin_mul_overflow(expected, v->ne[d], &expected)) return 0;
    }
    return 1;
}

static int shape_copy(const oracle_view* src, const oracle_view* dst, int cont) {
    uint64_t ns, nd;
    if (!validate_as(src, DT_F32, 0, &ns) || !validate_as(dst, DT_F32, 0, &nd)) return ORACLE_INVALID_VIEW;
    if (ns != nd) return ORACLE_SHAPE_MISMATCH;
    if (cont && !dense_contiguous_f32(dst)) return ORACLE_INVALID_LAYOUT;
    ORACLE_MAP(src, dst, ns, v);
    return ORACLE_OK;
}

int oracle_cpy(const oracle_view* src, const oracle_view* dst) { return shape_copy(src, dst, 0); }

int oracle_cont(const oracle_view* src, const oracle_view* dst) { return shape_copy(src, dst, 1); }

/* ---------------------------------------------------------------------- */
/* Row gather: get_rows.rs (F32, F16, BF16, Q4_0, Q8_0, Q4_K sources)      */
/* ---------------------------------------------------------------------- */

enum { DT_Q4_0 = 2, DT_Q8_0 = 8, DT_Q4_K = 12, DT_BF16 = 30 };

typedef struct {
    const int32_t* data;
    uint64_t ne[3];
    uint64_t st[3]; /* element strides */
    uint64_t count;
    int valid;
} gr_index;

/* IndexView::with_strides (get_rows.rs:44-139, 180-215): an I32 view with
 * ne[3] == 1; nb[0] == 0 selects the implicit contiguous strides. */
static gr_index gr_index_view(const oracle_view* v) {
    gr_index x;
    memset(&x, 0, sizeof x);
    if (v == NULL || v->dtype != DT_I32 || v->ne[3] != 1) return x;
    x.data = (const int32_t*)v->data;
    const uint64_t len = v->storage_bytes / 4;
    uint64_t bs[3];
    int strides_valid = 1, shape_valid = 1, zero = 0;
    const int implicit = v->nb[0] == 0;
    if (implicit) {
        bs[0] = 4;
        for (int d = 1; d < 3; ++d)
            if (__builtin_mul_overflow(bs[d - 1], v->ne[d - 1], &bs[d])) {
                strides_valid = 0;
                bs[d] = 0;
            }
    } else {
        for (int d = 0; d < 3; ++d) bs[d] = v->nb[d];
    }
    uint64_t count = 1;
    for (int d = 0; d < 3; ++d) {
        x.ne[d] = v->ne[d];
        if (v->ne[d] > 1 && bs[d] == 0 && !implicit) strides_valid = 0;
        if (bs[d] != 0 && (bs[d] < 4 || bs[d] % 4 != 0)) strides_valid = 0;
        x.st[d] = bs[d] / 4;
        if (v->ne[d] == 0) zero = 1;
        else if (!zero && __builtin_mul_overflow(count, v->ne[d], &count)) {
            shape_valid = 0;
            count = 0;
        }
    }
    if (zero) count = 0;
    int span = 1;
    if (!zero) {
        u128 max_offset = 0;
        for (int d = 0; d < 3; ++d) max_offset += (u128)(v->ne[d] - 1) * (u128)bs[d];
        span = max_offset + 4 <= (u128)len * 4;
    }
    x.count = count;
    x.valid = strides_valid && shape_valid && span;
    return x;
}

static int32_t gr_index_read(const gr_index* x, uint64_t ordinal) {
    const uint64_t i0 = ordinal % x->ne[0], rem = ordinal / x->ne[0];
    const uint64_t i1 = rem % x->ne[1], i2 = rem / x->ne[1];
    return x->data[i0 * x->st[0] + i1 * x->st[1] + i2 * x->st[2]];
}

/* shape_valid (get_rows.rs:1045-1054) and its per-dtype copies */
static int gr_shape_valid(const oracle_view* src, const gr_index* x, const oracle_view* dst) {
    return src->ne[0] > 0 && src->ne[1] > 0 && dst->ne[0] == src->ne[0] && dst->ne[1] == x->ne[0] &&
           dst->ne[2] == x->ne[1] && dst->ne[3] == x->ne[2] && src->ne[2] == x->ne[1] && src->ne[3] == x->ne[2];
}

/* indices_valid (get_rows.rs:1254-1265): 0 <= row < src.ne[1] */
static int gr_indices_valid(const gr_index* x, uint64_t rows) {
    for (uint64_t o = 0; o < x->count; ++o) {
        const int32_t r = gr_index_read(x, o);
        if (r < 0 || (uint64_t)r >= rows) return 0;
    }
    return 1;
}

/* empty_index_source_valid (get_rows.rs:1000-1022) */
static int gr_empty_f32_source_valid(const oracle_view* v) {
    if (v->dtype != DT_F32 || v->ne[0] == 0 || v->ne[1] == 0 || (v->nb[0] != 0 && v->nb[0] != 4)) return 0;
    if (v->nb[0] != 0)
        for (int d = 0; d < 4; ++d)
            if (v->ne[d] > 1 && v->nb[d] == 0) return 0;
    return 1;
}

/* destination_valid (get_rows.rs:1024-1031) */
static int gr_destination_valid(const oracle_view* dst, uint64_t count) {
    if (count == 0) return dst->dtype == DT_F32 && dense_contiguous_f32(dst);
    return validate_as(dst, DT_F32, 0, NULL) && dense_contiguous_f32(dst);
}

/* F16View::validate (f16_matmul.rs:45-85) / Bf16View::validate (get_rows.rs:300-340) */
static int gr_half_view_valid(const oracle_view* v, uint32_t dtype) {
    if (v->dtype != dtype) return 0;
    uint64_t count;
    if (!element_count(v, &count)) return 0;
    uint64_t s[4];
    if (v->nb[0] != 0) {
        for (int d = 0; d < 4; ++d) s[d] = v->nb[d];
    } else {
        s[0] = 2;
        for (int d = 1; d < 4; ++d)
            if (__builtin_mul_overflow(s[d - 1], v->ne[d - 1], &s[d])) return 0;
    }
    for (int d = 0; d < 4; ++d) {
        if (dtype == DT_F16) {
            if (v->ne[d] > 1 && (s[d] < 2 || s[d] % 2 != 0)) return 0;
        } else if (v->nb[0] != 0) {
            if ((v->ne[d] > 1 && v->nb[d] == 0) || (v->nb[d] != 0 && (v->nb[d] < 2 || v->nb[d] % 2 != 0))) return 0;
        }
    }
    u128 max_offset = 0;
    for (int d = 0; d < 4; ++d) max_offset += (u128)(v->ne[d] - 1) * (u128)s[d];
    return max_offset + 2 <= (u128)(v->storage_bytes / 2) * 2;
}

/* PackedRowView::validate (tensor_view.rs:483-526) */
static int gr_packed_view_valid(const oracle_view* v, uint32_t code, uint64_t block_values, uint64_t block_bytes) {
    if (v->dtype != code) return 0;
    for (int d = 0; d < 4; ++d)
        if (v->ne[d] == 0) return 0;
    if (v->ne[0] % block_values != 0 || v->nb[0] != 1) return 0;
    uint64_t row_bytes, s2, s3;
    if (__builtin_mul_overflow(v->ne[0] / block_values, block_bytes, &row_bytes)) return 0;
    if (__builtin_mul_overflow(row_bytes, v->ne[1], &s2)) return 0;
    if (__builtin_mul_overflow(s2, v->ne[2], &s3)) return 0;
    if (row_bytes == 0 || v->nb[1] != row_bytes || v->nb[2] != s2 || v->nb[3] != s3) return 0;
    u128 max_offset = 0;
    for (int d = 1; d < 4; ++d) max_offset += (u128)(v->ne[d] - 1) * (u128)v->nb[d];
    return max_offset + row_bytes <= (u128)v->storage_bytes;
}

/* f16_to_f32 (f16_matmul.rs:508-532): exact, NaN payload kept as is */
static float gr_f16_bits_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1fu, f = h & 0x3ffu;
    uint32_t bits;
    if (e == 0) {
        if (f == 0) {
            bits = sign;
        } else {
            uint32_t n = f, shift = 0;
            while ((n & 0x400u) == 0) {
                n <<= 1;
                ++shift;
            }
            bits = sign | ((127u - (14u + shift)) << 23) | ((n & 0x3ffu) << 13);
        }
    } else if (e == 0x1f) {
        bits = sign | 0x7f800000u | (f << 13);
    } else {
        bits = sign | ((e + 112u) << 23) | (f << 13);
    }
    float r;
    memcpy(&r, &bits, 4);
    return r;
}

/* fp16_to_f32 (quant.rs:287-302), the magic-number conversion, in binary32
 * arithmetic as written (a NaN comes out of the multiply quietened). */
static float gr_quant_fp16_to_f32(uint16_t h) {
    const uint32_t word = (uint32_t)h << 16;
    const uint32_t sign = word & 0x80000000u;
    const uint32_t doubled = word + word;
    uint32_t a = (doubled >> 4) + (0xe0u << 23), b = 0x07800000u, c = (doubled >> 17) | (126u << 23);
    float fa, fb, fc;
    memcpy(&fa, &a, 4);
    memcpy(&fb, &b, 4);
    memcpy(&fc, &c, 4);
    const float normalized = fa * fb;
    const float denormalized = fc - 0.5f;
    uint32_t nbits, dbits;
    memcpy(&nbits, &normalized, 4);
    memcpy(&dbits, &denormalized, 4);
    const uint32_t bits = doubled < (1u << 27) ? (sign | dbits) : (sign | nbits);
    float r;
    memcpy(&r, &bits, 4);
    return r;
}

static uint16_t gr_le16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* Q4_0Row::decode_block (quant.rs:106-134) */
static void gr_q4_0_block(const uint8_t* b, float* out) {
    const float scale = gr_quant_fp16_to_f32(gr_le16(b));
    for (int i = 0; i < 16; ++i) {
        const uint8_t p = b[i + 2];
        out[i] = ((float)(p & 0x0f) - 8.0f) * scale;
        out[i + 16] = ((float)(p >> 4) - 8.0f) * scale;
    }
}

/* Q8_0Row::decode_block (quant.rs:178-205) */
static void gr_q8_0_block(const uint8_t* b, float* out) {
    const float scale = gr_quant_fp16_to_f32(gr_le16(b));
    for (int i = 0; i < 32; ++i) out[i] = (float)(int8_t)b[i + 2] * scale;
}

/* q4_k_scale_min (quant_more.rs:952-961) */
static void gr_q4_k_scale_min(int j, const uint8_t* q, uint8_t* sc, uint8_t* m) {
    if (j < 4) {
        *sc = q[j] & 0x3f;
        *m = q[j + 4] & 0x3f;
    } else {
        *sc = (uint8_t)((q[j + 4] & 0x0f) | ((q[j - 4] >> 6) << 4));
        *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

/* Q4KRow::decode_block (quant_more.rs:438-468) */
static void gr_q4_k_block(const uint8_t* b, float* out) {
    const float scale = gr_quant_fp16_to_f32(gr_le16(b));
    const float minimum = gr_quant_fp16_to_f32(gr_le16(b + 2));
    const uint8_t* scales = b + 4;
    for (int g = 0; g < 4; ++g) {
        uint8_t sa, ma, sb, mb;
        gr_q4_k_scale_min(2 * g, scales, &sa, &ma);
        gr_q4_k_scale_min(2 * g + 1, scales, &sb, &mb);
        const float d0 = scale * (float)sa, d1 = scale * (float)sb;
        const float m0 = minimum * (float)ma, m1 = minimum * (float)mb;
        const uint8_t* q = b + 16 + 32 * g;
        for (int l = 0; l < 32; ++l) {
            out[64 * g + l] = d0 * (float)(q[l] & 0x0f) - m0;
            out[64 * g + 32 + l] = d1 * (float)(q[l] >> 4) - m1;
        }
    }
}

/* One entry point for every source type (the reference has one event per
 * type: OpGetRows, OpGetRowsF16, OpGetRowsBf16, OpGetRowsQ4_0, OpGetRowsQ8_0,
 * OpGetRowsQ4K); guards in each event's order, then the gather loops of
 * get_rows.rs:1453-1800. */
/* ByteTensorView::validate (tensor_view.rs:588-643): F32 metadata, nb[0]
 * zero or a multiple of 4 that is at least 4, no zero stride on a
 * multi-element dimension when strides are explicit, and every row's bytes
 * (ne[0] * 4 from any outer byte offset) inside the byte storage. */
static int gr_byte_view_valid(const oracle_view* v) {
    if (v->dtype != DT_F32) return 0;
    uint64_t count;
    if (!element_count(v, &count)) return 0;
    if (v->nb[0] != 0 && (v->nb[0] < 4 || v->nb[0] % 4 != 0)) return 0;
    if (v->nb[0] != 0)
        for (int d = 0; d < 4; ++d)
            if (v->ne[d] > 1 && v->nb[d] == 0) return 0;
    uint64_t s[4];
    if (!effective_strides(v, 4, s)) return 0;
    u128 max_offset = 0;
    for (int d = 1; d < 4; ++d) max_offset += (u128)(v->ne[d] - 1) * (u128)s[d];
    return max_offset + (u128)v->ne[0] * 4 <= (u128)v->storage_bytes;
}

/* empty_f32_bytes_source_valid (get_rows.rs:951-971) */
static int gr_byte_empty_valid(const oracle_view* v) {
    if (v->dtype != DT_F32 || v->ne[0] == 0 || v->ne[1] == 0) return 0;
    if (v->nb[0] != 0 && (v->nb[0] < 4 || v->nb[0] % 4 != 0)) return 0;
    if (v->nb[0] != 0)
        for (int d = 0; d < 4; ++d)
            if (v->ne[d] > 1 && v->nb[d] == 0) return 0;
    return 1;
}

/* OpGetRowsF32Bytes (get_rows.rs:233-255; guards 942-1003 in the order view,
 * shape, indices; loop 1943-1979): dst row r is the ne[0] * 4 bytes at source
 * row indices[r] of batch (i1, i2), read from any byte offset. */
int oracle_get_rows_f32_bytes(const oracle_view* src, const oracle_view* indices, const oracle_view* dst) {
    if (src == NULL || indices == NULL || dst == NULL) return ORACLE_INVALID_VIEW;
    const gr_index ix = gr_index_view(indices);
    const int views = ix.valid && (ix.count == 0 ? gr_byte_empty_valid(src) : gr_byte_view_valid(src)) &&
                      gr_destination_valid(dst, ix.count);
    if (!views) return ORACLE_INVALID_VIEW;
    if (!gr_shape_valid(src, &ix, dst)) return ORACLE_SHAPE_MISMATCH;
    if (!gr_indices_valid(&ix, src->ne[1])) return ORACLE_INDEX_OUT_OF_BOUNDS;
    if (ix.count == 0) return ORACLE_OK;
    uint64_t s[4];
    effective_strides(src, 4, s);
    const uint64_t cols = src->ne[0];
    float* out = (float*)dst->data;
    uint64_t dst_row = 0;
    for (uint64_t i2 = 0; i2 < ix.ne[2]; ++i2)
        for (uint64_t i1 = 0; i1 < ix.ne[1]; ++i1)
            for (uint64_t i0 = 0; i0 < ix.ne[0]; ++i0, ++dst_row) {
                const uint64_t index = (uint64_t)gr_index_read(&ix, dst_row);
                memcpy(out + dst_row * cols, (const char*)src->data + index * s[1] + i1 * s[2] + i2 * s[3], cols * 4);
            }
    return ORACLE_OK;
}

int oracle_get_rows(const oracle_view* src, const oracle_view* indices, const oracle_view* dst) {
    if (src == NULL || indices == NULL || dst == NULL) return ORACLE_INVALID_VIEW;
    const gr_index ix = gr_index_view(indices);
    const uint32_t t = src->dtype;
    uint64_t bv = 0, bb = 0;
    int views;
    if (t == DT_F32) {
        views = ix.valid && (ix.count == 0 ? gr_empty_f32_source_valid(src) : validate_as(src, DT_F32, 1, NULL)) &&
                gr_destination_valid(dst, ix.count);
    } else if (t == DT_F16 || t == DT_BF16) {
        views = ix.valid && gr_half_view_valid(src, t) && validate_as(dst, DT_F32, 0, NULL) &&
                dense_contiguous_f32(dst);
    } else if (t == DT_Q4_0 || t == DT_Q8_0 || t == DT_Q4_K) {
        bv = t == DT_Q4_K ? 256 : 32;
        bb = t == DT_Q4_0 ? 18 : (t == DT_Q8_0 ? 34 : 144);
        views = ix.valid && gr_packed_view_valid(src, t, bv, bb) &&
                (ix.count == 0 ? dense_contiguous_f32(dst) : (validate_as(dst, DT_F32, 0, NULL) && dense_contiguous_f32(dst))) &&
                dst->dtype == DT_F32;
    } else {
        return ORACLE_INVALID_VIEW;
    }
    if (!views) return ORACLE_INVALID_VIEW;
    if (!gr_shape_valid(src, &ix, dst)) return ORACLE_SHAPE_MISMATCH;
    if (t == DT_F32 && !(src->nb[0] == 0 || (src->nb[0] >= 4 && src->nb[0] % 4 == 0)))
        return ORACLE_UNSUPPORTED_SOURCE_STRIDE;
    if (!gr_indices_valid(&ix, src->ne[1])) return ORACLE_INDEX_OUT_OF_BOUNDS;
    if (ix.count == 0) return ORACLE_OK;

    const uint64_t cols = src->ne[0], rows = src->ne[1], batches = src->ne[2];
    float* out = (float*)dst->data;
    uint64_t s[4] = {0, 0, 0, 0};
    if (t == DT_F32) effective_strides(src, 4, s);
    if (t == DT_F16 || t == DT_BF16) {
        if (src->nb[0] != 0) {
            for (int d = 0; d < 4; ++d) s[d] = src->nb[d];
        } else {
            s[0] = 2;
            for (int d = 1; d < 4; ++d) s[d] = s[d - 1] * src->ne[d - 1];
        }
    }
    float block[256];
    uint64_t dst_row = 0;
    for (uint64_t i2 = 0; i2 < ix.ne[2]; ++i2)
        for (uint64_t i1 = 0; i1 < ix.ne[1]; ++i1)
            for (uint64_t i0 = 0; i0 < ix.ne[0]; ++i0, ++dst_row) {
                const uint64_t index = (uint64_t)gr_index_read(&ix, dst_row);
                float* o = out + dst_row * cols;
                if (t == DT_F32) {
                    /* read_row_contiguous (tensor_view.rs:756-769): columns 4 bytes apart */
                    const char* base = (const char*)src->data + index * s[1] + i1 * s[2] + i2 * s[3];
                    memcpy(o, base, cols * 4);
                } else if (t == DT_F16 || t == DT_BF16) {
                    /* F16View / Bf16View read of ordinal ((i2 * ne2 + i1) * rows + index) * cols + c */
                    const uint64_t first = ((i2 * batches + i1) * rows + index) * cols;
                    for (uint64_t c = 0; c < cols; ++c) {
                        uint64_t rem = first + c, off = 0;
                        for (int d = 0; d < 4; ++d) {
                            off += (rem % src->ne[d]) * s[d];
                            rem /= src->ne[d];
                        }
                        const uint16_t h = *(const uint16_t*)((const char*)src->data + off);
                        if (t == DT_F16) {
                            o[c] = gr_f16_bits_to_f32(h);
                        } else {
                            const uint32_t bits = (uint32_t)h << 16;
                            memcpy(&o[c], &bits, 4);
                        }
                    }
                } else {
                    const uint64_t row_bytes = cols / bv * bb;
                    const uint8_t* r = (const uint8_t*)src->data + ((i2 * batches + i1) * rows + index) * row_bytes;
                    for (uint64_t blk = 0; blk < cols / bv; ++blk) {
                        if (t == DT_Q4_0) gr_q4_0_block(r + blk * bb, block);
                        else if (t == DT_Q8_0) gr_q8_0_block(r + blk * bb, block);
                        else gr_q4_k_block(r + blk * bb, block);
                        memcpy(o + blk * bv, block, bv * 4);
                    }
                }
            }
    return ORACLE_OK;
}

/* ---------------------------------------------------------------------- */
/* Rotary position embedding: rope.rs                                      */
/* ---------------------------------------------------------------------- */

enum { ROPE_NORM = 0, ROPE_NEOX = 2, ROPE_TIMESTEP = 4 };

/* Layout::validate_i32 (tensor_view.rs:388-390 -> 392-447): raw strides
 * (no implicit form for I32), each >= 4 and a multiple of 4. */
static int rope_positions_valid(const oracle_view* v) {
    if (v == NULL || v->dtype != DT_I32) return 0;
    uint64_t count;
    if (!element_count(v, &count)) return 0;
    for (int d = 0; d < 4; ++d)
        if (v->nb[d] < 4 || v->nb[d] % 4 != 0) return 0;
    u128 max_offset = 0;
    for (int d = 0; d < 4; ++d) max_offset += (u128)(v->ne[d] - 1) * (u128)v->nb[d];
    return max_offset + 4 <= (u128)(v->storage_bytes / 4) * 4;
}

static int dense_contiguous_i32(const oracle_view* v) {
    if (v->dtype != DT_I32) return 0;
    uint64_t expected = 4;
    for (int d = 0; d < 4; ++d) {
        if (v->nb[d] != expected) return 0;
        if (__builtin_mul_overflow(expected, v->ne[d], &expected)) return 0;
    }
    return 1;
}

/* Guards of rope.rs:338-440 in transition order (view, parameters, then
 * shape / mode / the timestep layout), then execute_rotation (rope.rs:523-
 * 583) or execute_timestep (rope.rs:585-646).  The dense variants
 * (rope.rs:477-521) compute the same values.  The per-operation scalars use
 * the host libm exactly as the reference does: theta_scale =
 * powf(freq_base, -2 / n_dims) and -logf(freq_base) ((logf) bypasses the
 * correctly-rounded build's macro: the device library computes these two on
 * the host with the same calls). */
int oracle_rope(const oracle_view* src, const oracle_view* positions, const oracle_view* dst,
                const oracle_rope_params* pr) {
    uint64_t n;
    if (!validate_as(src, DT_F32, 0, &n) || !rope_positions_valid(positions) || !validate_as(dst, DT_F32, 0, NULL))
        return ORACLE_INVALID_VIEW;
    const uint64_t cols = src->ne[0];
    const int params_ok = pr->n_dims > 0 && pr->n_dims % 2 == 0 && (uint64_t)pr->n_dims <= cols &&
                          pr->ext_factor == 0.0f && isfinite(pr->freq_base) && pr->freq_base > 0.0f &&
                          isfinite(pr->freq_scale) && pr->freq_scale > 0.0f && isfinite(pr->attn_factor);
    if (!params_ok) return ORACLE_INVALID_PARAMETERS;
    const int shape_ok = same_ne(src, dst) && cols > 0 && positions->ne[0] == src->ne[2] && positions->ne[1] == 1 &&
                         positions->ne[2] == 1 && positions->ne[3] == 1 && src->ne[2] > 0;
    const int mode = pr->mode;
    const int known = mode == ROPE_NORM || mode == ROPE_NEOX || mode == ROPE_TIMESTEP;
    const int layout_ok = mode != ROPE_TIMESTEP || ((uint64_t)pr->n_dims == cols && dense_contiguous_f32(src) &&
                                                    dense_contiguous_i32(positions) && dense_contiguous_f32(dst));
    if (shape_ok && !known) return ORACLE_INVALID_MODE;
    if (!shape_ok || !layout_ok) return ORACLE_SHAPE_MISMATCH;

    uint64_t ss[4], sd[4];
    effective_strides(src, 4, ss);
    effective_strides(dst, 4, sd);
    const uint64_t rows = src->ne[1], npos = src->ne[2], batches = src->ne[3];
    const char* sb = (const char*)src->data;
    char* db = (char*)dst->data;
#define ROPE_AT(base, st, c, r, p, b) ((float*)((base) + (c) * (st)[0] + (r) * (st)[1] + (p) * (st)[2] + (b) * (st)[3]))
    if (mode != ROPE_TIMESTEP) {
        const uint64_t half = (uint64_t)pr->n_dims / 2;
        const float theta_scale = powf(pr->freq_base, -2.0f / (float)pr->n_dims);
        for (uint64_t b = 0; b < batches; ++b)
            for (uint64_t p = 0; p < npos; ++p) {
                /* I32View::read_at (rope.rs:85-101): raw strides */
                const int32_t pos_i = *(const int32_t*)((const char*)positions->data + p * positions->nb[0]);
                const float position = (float)pos_i;
                for (uint64_t r = 0; r < rows; ++r) {
                    float theta = position;
                    for (uint64_t k = 0; k < half; ++k) {
                        const float rotated = theta * pr->freq_scale;
                        const float cosine = cosf(rotated) * pr->attn_factor;
                        const float sine = sinf(rotated) * pr->attn_factor;
                        const uint64_t ia = mode == ROPE_NEOX ? k : 2 * k, ib = mode == ROPE_NEOX ? k + half : 2 * k + 1;
                        const float first = *ROPE_AT(sb, ss, ia, r, p, b), second = *ROPE_AT(sb, ss, ib, r, p, b);
                        *ROPE_AT(db, sd, ia, r, p, b) = fmaf(first, cosine, -(second * sine));
                        *ROPE_AT(db, sd, ib, r, p, b) = fmaf(first, sine, second * cosine);
                        theta *= theta_scale;
                    }
                    for (uint64_t c = (uint64_t)pr->n_dims; c < cols; ++c)
                        *ROPE_AT(db, sd, c, r, p, b) = *ROPE_AT(sb, ss, c, r, p, b);
                }
            }
    } else {
        const uint64_t half = cols / 2;
        const float neg_log_period = -(logf)(pr->freq_base);
        for (uint64_t b = 0; b < batches; ++b)
            for (uint64_t p = 0; p < npos; ++p) {
                const float position = (float)((const int32_t*)positions->data)[p];
                for (uint64_t r = 0; r < rows; ++r)
                    for (uint64_t k = 0; k < half; ++k) {
                        const float real = *ROPE_AT(sb, ss, 2 * k, r, p, b), imag = *ROPE_AT(sb, ss, 2 * k + 1, r, p, b);
                        const float frequency = expf(neg_log_period * (float)k / (float)half);
                        const float argument = position * frequency * pr->freq_scale;
                        const float cosine = cosf(argument) * pr->attn_factor;
                        const float sine = sinf(argument) * pr->attn_factor;
                        const volatile float rc = real * cosine, is = imag * sine, rs = real * sine, ic = imag * cosine;
                        *ROPE_AT(db, sd, k, r, p, b) = rc - is;
                        *ROPE_AT(db, sd, half + k, r, p, b) = rs + ic;
                    }
            }
    }
#undef ROPE_AT
    return ORACLE_OK;
}

/* ---------------------------------------------------------------------- */
/* Vocabulary matvec + argmax: matmul.rs OpMulMatArgmax (F32)               */
/* ---------------------------------------------------------------------- */

/* argmax_views_valid / argmax_shape_valid (matmul.rs:1416-1423, 1504-1520)
 * and effect_mul_mat_argmax_execute (matmul.rs:3018-3052): each row's dot
 * product is one sequential binary32 sum of separate products; the first
 * row starts the scan, a later row wins only with a strictly larger score. */
int oracle_mul_mat_argmax(const oracle_view* lhs, const oracle_view* rhs, const oracle_view* dst, int32_t* index_out) {
    if (!validate_as(lhs, DT_F32, 0, NULL) || !validate_as(rhs, DT_F32, 0, NULL) || !validate_as(dst, DT_F32, 0, NULL) ||
        !dense_contiguous_f32(lhs) || !dense_contiguous_f32(rhs) || !dense_contiguous_f32(dst))
        return ORACLE_INVALID_VIEW;
    const uint64_t* l = lhs->ne;
    const uint64_t* r = rhs->ne;
    const uint64_t* d = dst->ne;
    if (!(l[0] > 0 && l[1] > 0 && l[2] == 1 && l[3] == 1 && r[0] == 1 && r[1] == l[0] && r[2] == 1 && r[3] == 1 &&
          d[0] == 1 && d[1] == 1 && d[2] == 1 && d[3] == 1))
        return ORACLE_SHAPE_MISMATCH;
    const uint64_t k = l[0], rows = l[1];
    const float* a = (const float*)lhs->data;
    const float* v = (const float*)rhs->data;
    int32_t best_index = 0;
    float best = -INFINITY;
    for (uint64_t row = 0; row < rows; ++row) {
        float acc = 0.0f;
        for (uint64_t i = 0; i < k; ++i) acc += a[row * k + i] * v[i];
        if (acc > best || row == 0) {
            best = acc;
            best_index = (int32_t)row;
        }
    }
    *(float*)dst->data = best;
    if (index_out) *index_out = best_index;
    return ORACLE_OK;
}

/* Packed vocabulary matvec + argmax: matmul.rs OpMulMatArgmaxQ4_0 / Q4_1 /
 * Q5_0 / Q8_0 (routes matmul.rs:2904-2970).  quantized_views_valid /
 * quantized_shape_valid (matmul.rs:1522-1564), quantize_q8_0 (1629-1653),
 * dot_q4_0 / dot_q4_1 / dot_q5_0 / dot_q8_0 (1804-1910), run_argmax_*
 * (2193-2498): the rhs is quantized per 32-value block (scale = amax / 127
 * stored as binary16, q = clamp(round(x / scale))); each lhs row is the sum
 * over blocks, in order, of that block's term; the first row with the
 * largest sum wins. */
static int oracle_argmax_packed(int code, const oracle_view* lhs, const oracle_view* rhs, const oracle_view* dst,
                                int32_t* index_out) {
    uint64_t bb;
    switch (code) {
    case 2: bb = 18; break;  /* Q4_0 */
    case 3: bb = 20; break;  /* Q4_1 */
    case 6: bb = 22; break;  /* Q5_0 */
    default: bb = 34; break; /* Q8_0 */
    }
    if (!gr_packed_view_valid(lhs, (uint32_t)code, 32, bb) || lhs->ne[0] / 32 > 1024 ||
        !validate_as(rhs, DT_F32, 0, NULL) || !validate_as(dst, DT_F32, 0, NULL) || !dense_contiguous_f32(rhs) ||
        !dense_contiguous_f32(dst))
        return ORACLE_INVALID_VIEW;
    const uint64_t* l = lhs->ne;
    const uint64_t* r = rhs->ne;
    const uint64_t* d = dst->ne;
    if (!(l[0] > 0 && l[1] > 0 && l[2] == 1 && l[3] == 1 && r[0] == 1 && r[1] == l[0] && r[2] == 1 && r[3] == 1 &&
          d[0] == 1 && d[1] == 1 && d[2] == 1 && d[3] == 1))
        return ORACLE_SHAPE_MISMATCH;
    const uint64_t blocks = l[0] / 32, rows = l[1], row_bytes = blocks * bb;
    const float* x = (const float*)rhs->data;
    static int8_t qs[1024 * 32];
    static uint16_t dr16[1024];
    for (uint64_t b = 0; b < blocks; ++b) {
        float amax = 0.0f;
        for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(x[b * 32 + i]));
        const float scale = amax / 127.0f;
        const float inverse = scale == 0.0f ? 0.0f : 1.0f / scale;
        dr16[b] = oracle_fp32_to_fp16(scale);
        for (int i = 0; i < 32; ++i) {
            float q = roundf(x[b * 32 + i] * inverse);
            if (isnan(q)) q = 0.0f; /* `as i8` of NaN */
            q = q < -127.0f ? -127.0f : (q > 127.0f ? 127.0f : q);
            qs[b * 32 + i] = (int8_t)q;
        }
    }
    const uint8_t* base = (const uint8_t*)lhs->data;
    float best = -INFINITY;
    int32_t best_index = 0;
    for (uint64_t row = 0; row < rows; ++row) {
        const uint8_t* rp = base + row * row_bytes;
        float sum = 0.0f;
        for (uint64_t b = 0; b < blocks; ++b) {
            const uint8_t* blk = rp + b * bb;
            const int8_t* q = qs + b * 32;
            const float dl = gr_quant_fp16_to_f32(gr_le16(blk)), drs = gr_quant_fp16_to_f32(dr16[b]);
            int32_t integer = 0;
            if (code == 8) {
                for (int i = 0; i < 32; ++i) integer += (int32_t)(int8_t)blk[2 + i] * (int32_t)q[i];
                sum += (float)integer * (dl * drs);
            } else if (code == 2) {
                for (int i = 0; i < 16; ++i) {
                    integer += ((int32_t)(blk[2 + i] & 0x0f) - 8) * (int32_t)q[i];
                    integer += ((int32_t)(blk[2 + i] >> 4) - 8) * (int32_t)q[i + 16];
                }
                sum += (float)integer * (dl * drs);
            } else if (code == 6) {
                const uint32_t high = (uint32_t)blk[2] | ((uint32_t)blk[3] << 8) | ((uint32_t)blk[4] << 16) |
                                      ((uint32_t)blk[5] << 24);
                for (int i = 0; i < 16; ++i) {
                    const int32_t lo = (int32_t)((blk[6 + i] & 0x0f) | (((high >> i) & 1u) << 4)) - 16;
                    const int32_t hi = (int32_t)((blk[6 + i] >> 4) | (((high >> (i + 16)) & 1u) << 4)) - 16;
                    integer += lo * (int32_t)q[i] + hi * (int32_t)q[i + 16];
                }
                sum += (float)integer * (dl * drs);
            } else { /* Q4_1: rhs_scale * (d * integer + m * rhs_sum) (matmul.rs:1832-1858) */
                int32_t rhs_sum = 0;
                for (int i = 0; i < 16; ++i) {
                    integer += (int32_t)(blk[4 + i] & 0x0f) * (int32_t)q[i];
                    integer += (int32_t)(blk[4 + i] >> 4) * (int32_t)q[i + 16];
                    rhs_sum += (int32_t)q[i] + (int32_t)q[i + 16];
                }
                const float ml = gr_quant_fp16_to_f32(gr_le16(blk + 2));
                sum += drs * (dl * (float)integer + ml * (float)rhs_sum);
            }
        }
        if (sum > best || row == 0) {
            best = sum;
            best_index = (int32_t)row;
        }
    }
    *(float*)dst->data = best;
    if (index_out) *index_out = best_index;
    return ORACLE_OK;
}

int oracle_mul_mat_argmax_q8_0(const oracle_view* lhs, const oracle_view* rhs, const oracle_view* dst,
                               int32_t* index_out) {
    return oracle_argmax_packed(8, lhs, rhs, dst, index_out);
}

int oracle_mul_mat_argmax_q4_0(const oracle_view* lhs, const oracle_view* rhs, const oracle_view* dst,
                               int32_t* index_out) {
    return oracle_argmax_packed(2, lhs, rhs, dst, index_out);
}

int oracle_mul_mat_argmax_q4_1(const oracle_view* lhs, const oracle_view* rhs, const oracle_view* dst,
                               int32_t* index_out) {
    return oracle_argmax_packed(3, lhs, rhs, dst, index_out);
}

int oracle_mul_mat_argmax_q5_0(const oracle_view* lhs, const oracle_view* rhs, const oracle_view* dst,
                               int32_t* index_out) {
    return oracle_argmax_packed(6, lhs, rhs, dst, index_out);
}

/* K-quant vocabulary matvec + argmax: matmul.rs OpMulMatArgmaxQ4K / Q6K
 * (routes through define_k_argmax_runner, matmul.rs:2502-2535).  The rhs is
 * quantized to Q8_K per 256-value block (quantize_q8_k, matmul.rs:1703-1745:
 * the first value of largest magnitude sets inverse = -127 / value, d =
 * 1 / inverse, q = min(nearest_int(inverse * x), 127), 16 group sums);
 * dot_q4_k (2040-2114), dot_q3_k (1994-2036) and dot_q6_k (2117-2190) keep
 * eight lane sums, lane = position % 8, added to the row total after the
 * last block; dot_q2_k (1918-1962) adds one term per block. */
typedef struct {
    float d;
    int8_t qs[256];
    int16_t bsums[16];
} q8k_block;

/* nearest_int (matmul.rs:1696-1700): round through the 1.5 * 2^23 bias. */
static int32_t q8k_nearest_int(float v) {
    const float biased = v + 12582912.0f;
    return (int32_t)(f2u(biased) & 0x007fffffu) - 0x00400000;
}

static void q8k_quantize(const float* x, uint64_t blocks, q8k_block* out) {
    for (uint64_t b = 0; b < blocks; ++b) {
        const float* v = x + b * 256;
        float maximum = 0.0f, absolute = 0.0f;
        for (int i = 0; i < 256; ++i)
            if (fabsf(v[i]) > absolute) {
                absolute = fabsf(v[i]);
                maximum = v[i];
            }
        memset(&out[b], 0, sizeof out[b]);
        if (absolute == 0.0f) continue;
        const float inverse = -127.0f / maximum;
        out[b].d = 1.0f / inverse;
        for (int i = 0; i < 256; ++i) {
            int32_t q = q8k_nearest_int(inverse * v[i]);
            out[b].qs[i] = (int8_t)(q < 127 ? q : 127);
        }
        for (int g = 0; g < 16; ++g) {
            int16_t sum = 0;
            for (int i = 0; i < 16; ++i) sum = (int16_t)(sum + out[b].qs[g * 16 + i]);
            out[b].bsums[g] = sum;
        }
    }
}

static float dot_q4_k_block(const uint8_t* blk, const q8k_block* r, float* lane_sums, float sum) {
    int8_t q4[256];
    for (int g = 0; g < 4; ++g)
        for (int l = 0; l < 32; ++l) {
            const uint8_t packed = blk[16 + g * 32 + l];
            q4[g * 64 + l] = (int8_t)(packed & 0x0f);
            q4[g * 64 + 32 + l] = (int8_t)(packed >> 4);
        }
    const uint8_t* sc = blk + 4;
    uint8_t scales[8], mins[8];
    for (int l = 0; l < 4; ++l) {
        scales[l] = sc[l] & 0x3f;
        scales[4 + l] = (uint8_t)((sc[8 + l] & 0x0f) | (((sc[l] >> 6) & 0x03) << 4));
        mins[l] = sc[4 + l] & 0x3f;
        mins[4 + l] = (uint8_t)(((sc[8 + l] >> 4) & 0x0f) | (((sc[4 + l] >> 6) & 0x03) << 4));
    }
    int32_t min_sum = 0;
    for (int g = 0; g < 16; ++g) min_sum += (int32_t)r->bsums[g] * (int32_t)mins[g / 2];
    int32_t acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int g = 0; g < 8; ++g)
        for (int l = 0; l < 32; ++l)
            acc[l % 8] += (int32_t)scales[g] * ((int32_t)q4[g * 32 + l] * (int32_t)r->qs[g * 32 + l]);
    const float d = gr_quant_fp16_to_f32(gr_le16(blk)) * r->d;
    for (int l = 0; l < 8; ++l) lane_sums[l] += d * (float)acc[l];
    const float dmin = gr_quant_fp16_to_f32(gr_le16(blk + 2)) * r->d;
    return sum - dmin * (float)min_sum;
}

static void dot_q6_k_block(const uint8_t* blk, const q8k_block* r, float* lane_sums) {
    const uint8_t* ql = blk;
    const uint8_t* qh = blk + 128;
    const int8_t* scales = (const int8_t*)(blk + 192);
    const float d = gr_quant_fp16_to_f32(gr_le16(blk + 208));
    int8_t dec[256];
    for (int c = 0; c < 2; ++c)
        for (int i = 0; i < 32; ++i) {
            const uint8_t high = qh[c * 32 + i];
            dec[c * 128 + i] = (int8_t)(((ql[c * 64 + i] & 0x0f) | ((high & 3) << 4)) - 32);
            dec[c * 128 + i + 32] = (int8_t)(((ql[c * 64 + i + 32] & 0x0f) | (((high >> 2) & 3) << 4)) - 32);
            dec[c * 128 + i + 64] = (int8_t)((((ql[c * 64 + i] >> 4) & 0x0f) | (((high >> 4) & 3) << 4)) - 32);
            dec[c * 128 + i + 96] = (int8_t)((((ql[c * 64 + i + 32] >> 4) & 0x0f) | (((high >> 6) & 3) << 4)) - 32);
        }
    int32_t sums[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int g = 0; g < 16; ++g) {
        const int32_t scale = scales[g];
        for (int l = 0; l < 16; ++l) sums[l % 8] += scale * (int32_t)dec[g * 16 + l] * (int32_t)r->qs[g * 16 + l];
    }
    const float sc = r->d * d;
    for (int l = 0; l < 8; ++l) lane_sums[l] += sc * (float)sums[l];
}

/* dot_q2_k (matmul.rs:1918-1962): one total per block. */
static float dot_q2_k_block(const uint8_t* blk, const q8k_block* r, float total) {
    const uint8_t* scales = blk;
    const uint8_t* q = blk + 16;
    const float d = gr_quant_fp16_to_f32(gr_le16(blk + 80));
    const float dmin = gr_quant_fp16_to_f32(gr_le16(blk + 82));
    int32_t sum_mins = 0;
    for (int g = 0; g < 16; ++g) sum_mins += (int32_t)r->bsums[g] * (int32_t)(scales[g] >> 4);
    int32_t sum = 0;
    int si = 0;
    for (int c = 0; c < 2; ++c)
        for (int shift = 0; shift < 8; shift += 2) {
            const int32_t s0 = scales[si] & 0x0f, s1 = scales[si + 1] & 0x0f;
            int32_t low = 0, high = 0;
            for (int i = 0; i < 16; ++i) {
                low += (int32_t)r->qs[c * 128 + (shift / 2) * 32 + i] * (int32_t)((q[c * 32 + i] >> shift) & 3);
                high += (int32_t)r->qs[c * 128 + (shift / 2) * 32 + 16 + i] * (int32_t)((q[c * 32 + 16 + i] >> shift) & 3);
            }
            sum += s0 * low + s1 * high;
            si += 2;
        }
    const float d_all = r->d * d, d_min = r->d * dmin;
    return total + (d_all * (float)sum - d_min * (float)sum_mins);
}

/* unpack_q3_scales (matmul.rs:1964-1990) and dot_q3_k (1994-2036). */
static void dot_q3_k_block(const uint8_t* blk, const q8k_block* r, float* lane_sums) {
    const uint8_t* hmask = blk;
    const uint8_t* q = blk + 32;
    const uint8_t* sb = blk + 96;
    uint32_t aux[4];
    aux[0] = (uint32_t)sb[0] | ((uint32_t)sb[1] << 8) | ((uint32_t)sb[2] << 16) | ((uint32_t)sb[3] << 24);
    aux[1] = (uint32_t)sb[4] | ((uint32_t)sb[5] << 8) | ((uint32_t)sb[6] << 16) | ((uint32_t)sb[7] << 24);
    const uint32_t tmp = (uint32_t)sb[8] | ((uint32_t)sb[9] << 8) | ((uint32_t)sb[10] << 16) | ((uint32_t)sb[11] << 24);
    aux[2] = ((aux[0] >> 4) & 0x0f0f0f0fu) | (((tmp >> 4) & 0x03030303u) << 4);
    aux[3] = ((aux[1] >> 4) & 0x0f0f0f0fu) | (((tmp >> 6) & 0x03030303u) << 4);
    aux[0] = (aux[0] & 0x0f0f0f0fu) | ((tmp & 0x03030303u) << 4);
    aux[1] = (aux[1] & 0x0f0f0f0fu) | (((tmp >> 2) & 0x03030303u) << 4);
    int8_t scales[16];
    for (int i = 0; i < 16; ++i) scales[i] = (int8_t)((uint8_t)(aux[i / 4] >> (8 * (i % 4))) - 32u);
    const float d = gr_quant_fp16_to_f32(gr_le16(blk + 108));
    int32_t acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int g = 0; g < 16; ++g) {
        const int32_t scale = scales[g];
        const int qbase = (g / 8) * 32, half = (g % 2) * 16;
        const uint8_t mask = (uint8_t)(1u << (g / 2));
        for (int i = 0; i < 16; ++i) {
            const uint8_t qbyte = q[qbase + half + i];
            const int32_t quantized = (int32_t)((qbyte >> (((g / 2) % 4) * 2)) & 3) - ((hmask[half + i] & mask) == 0 ? 4 : 0);
            acc[i & 7] += scale * quantized * (int32_t)r->qs[g * 16 + i];
        }
    }
    const float sc = r->d * d;
    for (int l = 0; l < 8; ++l) lane_sums[l] += sc * (float)acc[l];
}

static int oracle_argmax_k(int code, const oracle_view* lhs, const oracle_view* rhs, const oracle_view* dst,
                           int32_t* index_out) {
    const uint64_t bb = code == 10 ? 84 : code == 11 ? 110 : code == 12 ? 144 : 210;
    if (!gr_packed_view_valid(lhs, (uint32_t)code, 256, bb) || lhs->ne[0] / 256 > 128 ||
        !validate_as(rhs, DT_F32, 0, NULL) || !validate_as(dst, DT_F32, 0, NULL) || !dense_contiguous_f32(rhs) ||
        !dense_contiguous_f32(dst))
        return ORACLE_INVALID_VIEW;
    const uint64_t* l = lhs->ne;
    const uint64_t* r = rhs->ne;
    const uint64_t* d = dst->ne;
    if (!(l[0] > 0 && l[1] > 0 && l[2] == 1 && l[3] == 1 && r[0] == 1 && r[1] == l[0] && r[2] == 1 && r[3] == 1 &&
          d[0] == 1 && d[1] == 1 && d[2] == 1 && d[3] == 1))
        return ORACLE_SHAPE_MISMATCH;
    const uint64_t blocks = l[0] / 256, rows = l[1], row_bytes = blocks * bb;
    static q8k_block q8[128];
    q8k_quantize((const float*)rhs->data, blocks, q8);
    const uint8_t* base = (const uint8_t*)lhs->data;
    float best = -INFINITY;
    int32_t best_index = 0;
    for (uint64_t row = 0; row < rows; ++row) {
        const uint8_t* rp = base + row * row_bytes;
        float lane_sums[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        float sum = 0.0f;
        for (uint64_t b = 0; b < blocks; ++b) {
            if (code == 10)
                sum = dot_q2_k_block(rp + b * bb, &q8[b], sum);
            else if (code == 11)
                dot_q3_k_block(rp + b * bb, &q8[b], lane_sums);
            else if (code == 12)
                sum = dot_q4_k_block(rp + b * bb, &q8[b], lane_sums, sum);
            else
                dot_q6_k_block(rp + b * bb, &q8[b], lane_sums);
        }
        if (code != 10)
            for (int k = 0; k < 8; ++k) sum += lane_sums[k];
        if (sum > best || row == 0) {
            best = sum;
            best_index = (int32_t)row;
        }
    }
    *(float*)dst->data = best;
    if (index_out) *index_out = best_index;
    return ORACLE_OK;
}

int oracle_mul_mat_argmax_q4_k(const oracle_view* lhs, const oracle_view* rhs, const oracle_view* dst,
                               int32_t* index_out) {
    return oracle_argmax_k(12, lhs, rhs, dst, index_out);
}

int oracle_mul_mat_argmax_q6_k(const oracle_view* lhs, const oracle_view* rhs, const oracle_view* dst,
                               int32_t* index_out) {
    return oracle_argmax_k(14, lhs, rhs, dst, index_out);
}

int oracle_mul_mat_argmax_q2_k(const oracle_view* lhs, const oracle_view* rhs, const oracle_view* dst,
                               int32_t* index_out) {
    return oracle_argmax_k(10, lhs, rhs, dst, index_out);
}

int oracle_mul_mat_argmax_q3_k(const oracle_view* lhs, const oracle_view* rhs, const oracle_view* dst,
                               int32_t* index_out) {
    return oracle_argmax_k(11, lhs, rhs, dst, index_out);
}

/* ---------------------------------------------------------------------- */
/* Single-query attention: flash_attn.rs OpFlashAttnExt                    */
/* ---------------------------------------------------------------------- */

/* flash_attn.rs:528-557: binary32 -> binary16 bits.  Normal results round
 * to nearest even; results below 2^-24 flush to a signed zero and the
 * subnormal range rounds half up (not IEEE); any NaN is 0x7E00 with the
 * input's sign. */
uint16_t oracle_fa_f32_to_f16(float value) {
    const uint32_t w = f2u(value);
    const uint16_t sign = (uint16_t)((w >> 16) & 0x8000u);
    const uint32_t e = (w >> 23) & 0xffu, frac = w & 0x7fffffu;
    if (e == 0xffu) return (uint16_t)(sign | (frac == 0 ? 0x7c00u : 0x7e00u));
    if (e > 142u) return (uint16_t)(sign | 0x7c00u);
    if (e < 103u) return sign;
    if (e < 113u) {
        const uint32_t shift = 113u - e, m = 0x800000u | frac;
        return (uint16_t)(sign | ((m + (1u << (shift + 12u))) >> (shift + 13u)));
    }
    uint16_t h = (uint16_t)(sign | ((e - 112u) << 10) | (frac >> 13));
    const uint32_t rem = frac & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h = (uint16_t)(h + 1u);
    return h;
}

/* round_fp16_scalar (flash_attn.rs:420-422): through the helper above and
 * quant.rs's magic-number widening. */
static float fa_round16(float v) { return gr_quant_fp16_to_f32(oracle_fa_f32_to_f16(v)); }

/* dense_f32_layout (flash_attn.rs:305-325): effective strides exactly
 * row-major (nb[0] == 0 resolves to that). */
static int fa_dense_f32(const oracle_view* v) {
    uint64_t s[4], expected = 4;
    if (v->dtype != DT_F32 || !effective_strides(v, 4, s)) return 0;
    for (int d = 0; d < 4; ++d) {
        if (s[d] != expected) return 0;
        if (__builtin_mul_overflow(expected, v->ne[d], &expected)) return 0;
    }
    return 1;
}

/* OpFlashAttnExt::new (flash_attn.rs:78-99), valid_request (262-303) and
 * execute (329-404) with its helpers (406-470): per head, one sequential
 * pass over the key/value tokens with a running maximum, a binary16
 * accumulator row and a binary32 score sum. */
int oracle_flash_attn_ext(const oracle_view* q, const oracle_view* k, const oracle_view* v, const oracle_view* dst,
                          const oracle_flash_attn_options* options) {
    if (!q || !k || !v || !dst) return ORACLE_INVALID_ARGUMENT;
    const uint64_t head_dim = q->ne[0], query_count = q->ne[1], heads = q->ne[2];
    const uint64_t tokens = k->ne[1], kv_heads = k->ne[2];
    float scale = 1.0f / sqrtf((float)head_dim);
    uint64_t masked_total = tokens;
    if (options && options->has_scale) scale = options->scale;
    if (options && options->has_masked_total_tokens) masked_total = options->masked_total_tokens;
    uint64_t ks[4], vs[4];
    const int valid =
        validate_as(q, DT_F32, 0, NULL) && validate_as(dst, DT_F32, 0, NULL) && gr_half_view_valid(k, DT_F16) &&
        gr_half_view_valid(v, DT_F16) && fa_dense_f32(q) && fa_dense_f32(dst) && head_dim != 0 && query_count == 1 &&
        heads != 0 && tokens != 0 && kv_heads != 0 && k->ne[0] == head_dim && v->ne[0] == head_dim &&
        v->ne[1] == tokens && v->ne[2] == kv_heads && dst->ne[0] == head_dim && dst->ne[1] == query_count &&
        dst->ne[2] == heads && q->ne[3] == 1 && k->ne[3] == 1 && v->ne[3] == 1 && dst->ne[3] == 1 &&
        heads % kv_heads == 0 && head_dim <= 4096 && masked_total >= tokens && isfinite(scale) && scale > 0.0f;
    if (!valid) return ORACLE_INVALID_REQUEST;
    effective_strides(k, 2, ks);
    effective_strides(v, 2, vs);
    const float* qd = (const float*)q->data;
    float* out = (float*)dst->data;
    const unsigned char* kb = (const unsigned char*)k->data;
    const unsigned char* vb = (const unsigned char*)v->data;
    const uint64_t rep = heads / kv_heads;
    uint16_t qh[4096], acc[4096];
    for (uint64_t h = 0; h < heads; ++h) {
        const uint64_t kvh = h / rep;
        for (uint64_t d = 0; d < head_dim; ++d) {
            qh[d] = oracle_fa_f32_to_f16(qd[h * head_dim + d]);
            acc[d] = 0;
        }
        float score_sum = 0.0f, max_score = -INFINITY;
        for (uint64_t t = 0; t < tokens; ++t) {
            /* dot_product_f16_f16_scores (flash_attn.rs:424-441) */
            double dot = 0.0;
            for (uint64_t d = 0; d < head_dim; ++d) {
                uint16_t kh;
                memcpy(&kh, kb + d * ks[0] + t * ks[1] + kvh * ks[2], 2);
                dot += (double)gr_quant_fp16_to_f32(qh[d]) * (double)gr_f16_bits_to_f32(kh);
            }
            const float score = (float)dot * scale;
            const float old_max = max_score;
            float max_scale = 1.0f, value_scale = 1.0f;
            if (score > max_score) {
                max_score = score;
                max_scale = expf(old_max - max_score);
                /* scale_f16_buffer_scalar (flash_attn.rs:443-451) */
                const float rs = fa_round16(max_scale);
                for (uint64_t d = 0; d < head_dim; ++d)
                    acc[d] = oracle_fa_f32_to_f16(fa_round16(gr_quant_fp16_to_f32(acc[d]) * rs));
            } else {
                value_scale = expf(score - max_score);
            }
            /* axpy_f16_buffer_scalar (flash_attn.rs:453-470) */
            const float alpha = fa_round16(value_scale);
            for (uint64_t d = 0; d < head_dim; ++d) {
                uint16_t vh;
                memcpy(&vh, vb + d * vs[0] + t * vs[1] + kvh * vs[2], 2);
                const float prod = gr_f16_bits_to_f32(vh) * alpha;
                acc[d] = oracle_fa_f32_to_f16(fa_round16(gr_quant_fp16_to_f32(acc[d]) + prod));
            }
            score_sum = score_sum * max_scale + value_scale;
        }
        /* finalize_attention_output (flash_attn.rs:382-404) */
        if (score_sum == 0.0f) {
            for (uint64_t d = 0; d < head_dim; ++d) out[h * head_dim + d] = 0.0f;
        } else {
            const float inv = 1.0f / score_sum;
            for (uint64_t d = 0; d < head_dim; ++d) out[h * head_dim + d] = gr_quant_fp16_to_f32(acc[d]) * inv;
        }
    }
    return ORACLE_OK;
}

/* ---------------------------------------------------------------------- */
/* Row normalisation: normalization.rs                                     */
/* ---------------------------------------------------------------------- */

static int norm_guards(const oracle_view* src, const oracle_view* dst, float eps) {
    if (!normalization_view_valid(src) || !normalization_view_valid(dst)) return ORACLE_INVALID_VIEW;
    if (!same_ne(src, dst)) return ORACLE_SHAPE_MISMATCH;
    if (!(isfinite(eps) && eps >= 0.0f)) return ORACLE_INVALID_PARAMETERS;
    return ORACLE_OK;
}

/* normalization.rs:316-341 */
int oracle_norm(const oracle_view* src, const oracle_view* dst, float eps) {
    int st = norm_guards(src, dst, eps);
    if (st != ORACLE_OK) return st;
    uint64_t ss[4], sd[4], count = 0;
    effective_strides(src, 4, ss);
    effective_strides(dst, 4, sd);
    element_count(src, &count);
    uint64_t columns = src->ne[0], rows = count / columns;
    for (uint64_t r = 0; r < rows; ++r) {
        /* a row is dimension 0 at fixed (i1, i2, i3): base + column * stride */
        uint64_t xb = ordinal_offset(src, ss, r * columns), yb = ordinal_offset(dst, sd, r * columns);
        double sum = 0.0;
        for (uint64_t c = 0; c < columns; ++c) sum += (double)load_f(src, xb + c * ss[0]);
        float mean = (float)(sum / (double)columns);
        double variance_sum = 0.0;
        for (uint64_t c = 0; c < columns; ++c) {
            float centered = load_f(src, xb + c * ss[0]) - mean;
            variance_sum += (double)centered * (double)centered;
        }
        float variance = (float)(variance_sum / (double)columns);
        float scale = 1.0f / sqrtf(variance + eps);
        for (uint64_t c = 0; c < columns; ++c)
            store_f(dst, yb + c * sd[0], (load_f(src, xb + c * ss[0]) - mean) * scale);
    }
    return ORACLE_OK;
}

/* normalization.rs:343-362, optionally followed by the broadcast.rs:372-390
 * row multiply (weight ne == [ne0,1,1,1]). */
static void rms_rows(const oracle_view* src, const oracle_view* weight, const oracle_view* dst, float eps,
                     uint64_t row_begin, uint64_t row_end) {
    uint64_t ss[4], sd[4], sw[4] = {0, 0, 0, 0};
    effective_strides(src, 4, ss);
    effective_strides(dst, 4, sd);
    if (weight) effective_strides(weight, 4, sw);
    uint64_t columns = src->ne[0];
    for (uint64_t r = row_begin; r < row_end; ++r) {
        uint64_t xb = ordinal_offset(src, ss, r * columns), yb = ordinal_offset(dst, sd, r * columns);
        double sum = 0.0;
        for (uint64_t c = 0; c < columns; ++c) {
            float v = load_f(src, xb + c * ss[0]);
            sum += (double)(v * v);
        }
        float mean = (float)(sum / (double)columns);
        float scale = 1.0f / sqrtf(mean + eps);
        for (uint64_t c = 0; c < columns; ++c) {
            float y = load_f(src, xb + c * ss[0]) * scale;
            if (weight) y = y * load_f(weight, c * sw[0]);
            store_f(dst, yb + c * sd[0], y);
        }
    }
}

void oracle_rms_norm_rows(const oracle_view* src, const oracle_view* dst, float eps, uint64_t row_begin,
                          uint64_t row_end) {
    rms_rows(src, NULL, dst, eps, row_begin, row_end);
}

int oracle_rms_norm(const oracle_view* src, const oracle_view* dst, float eps) {
    int st = norm_guards(src, dst, eps);
    if (st != ORACLE_OK) return st;
    uint64_t count = 0;
    element_count(src, &count);
    rms_rows(src, NULL, dst, eps, 0, count / src->ne[0]);
    return ORACLE_OK;
}

int oracle_rms_norm_mul(const oracle_view* src, const oracle_view* weight, const oracle_view* dst, float eps) {
    uint64_t count = 0;
    if (!normalization_view_valid(src) || !normalization_view_valid(dst) || !validate_as(weight, DT_F32, 1, NULL))
        return ORACLE_INVALID_VIEW;
    if (!same_ne(src, dst) || weight->ne[0] != src->ne[0] || weight->ne[1] != 1 || weight->ne[2] != 1 ||
        weight->ne[3] != 1)
        return ORACLE_SHAPE_MISMATCH;
    if (!(isfinite(eps) && eps >= 0.0f)) return ORACLE_INVALID_PARAMETERS;
    element_count(src, &count);
    rms_rows(src, weight, dst, eps, 0, count / src->ne[0]);
    return ORACLE_OK;
}

/* ---------------------------------------------------------------------- */
/* Softmax: reductions.rs:473-495 guards, 565-638 loops                   */
/* ---------------------------------------------------------------------- */

static int soft_max_dense_layout(const oracle_view* v) {
    if (v->nb[0] == 0) {
        uint64_t s[4];
        return effective_strides(v, 4, s);
    }
    return is_dense(v, 4);
}

/* mask (optional): F16 or F32, ne0 == src ne0, ne1 >= src ne1, ne2/ne3
 * divide the source extents; row (i1,i2,i3) reads mask row (i1, i2 % m2, i3 % m3). */
static int soft_max_core(const oracle_view* src, const oracle_view* mask, const oracle_view* dst, float scale,
                         int apply_scale) {
    uint64_t ns, nd;
    if (!validate_as(src, DT_F32, 0, &ns) || !validate_as(dst, DT_F32, 0, &nd)) return ORACLE_INVALID_VIEW;
    if (mask && !validate_float(mask, 0, NULL)) return ORACLE_INVALID_VIEW;
    uint64_t width = src->ne[0];
    if (!(width > 0 && ns > 0 && ns % width == 0 && ns == nd)) return ORACLE_SHAPE_MISMATCH;
    if (mask && !(mask->ne[0] == width && mask->ne[1] >= src->ne[1] && src->ne[2] % mask->ne[2] == 0 &&
                  src->ne[3] % mask->ne[3] == 0))
        return ORACLE_SHAPE_MISMATCH;
    int dense = soft_max_dense_layout(src) && soft_max_dense_layout(dst);
    uint64_t ss[4], sd[4], sm[4] = {0, 0, 0, 0};
    effective_strides(src, 4, ss);
    effective_strides(dst, 4, sd);
    if (mask) effective_strides(mask, dtype_size(mask->dtype), sm);
    uint64_t rows = ns / width;
    int dst_rows = same_ne(src, dst);
    for (uint64_t r = 0; r < rows; ++r) {
        uint64_t offset = r * width;
        uint64_t xb = ordinal_offset(src, ss, offset);
        uint64_t yb = dst_rows ? ordinal_offset(dst, sd, offset) : 0;
        uint64_t mask_row = 0;
        if (mask) {
            uint64_t i1 = r % src->ne[1], i2 = (r / src->ne[1]) % src->ne[2], i3 = r / (src->ne[1] * src->ne[2]);
            mask_row = i1 * sm[1] + (i2 % mask->ne[2]) * sm[2] + (i3 % mask->ne[3]) * sm[3];
        }
#define SM_VALUE(c)                                                                                   \
    (!apply_scale ? load_f(src, xb + (c) * ss[0])                                                   \
     : mask ? load_f(src, xb + (c) * ss[0]) * scale + load_f(mask, mask_row + (c) * sm[0])          \
            : load_f(src, xb + (c) * ss[0]) * scale)
#define SM_DST(c) (dst_rows ? yb + (c) * sd[0] : ordinal_offset(dst, sd, offset + (c)))
        float max_value = SM_VALUE(0);
        for (uint64_t c = 1; c < width; ++c) {
            float v = SM_VALUE(c);
            if (v > max_value) max_value = v;
        }
        if (dense) {
            double sum = 0.0;
            for (uint64_t c = 0; c < width; ++c) {
                float e = expf(SM_VALUE(c) - max_value);
                store_f(dst, SM_DST(c), e);
                sum += (double)e;
            }
            float denominator = (float)sum;
            for (uint64_t c = 0; c < width; ++c) {
                uint64_t o = SM_DST(c);
                store_f(dst, o, load_f(dst, o) / denominator);
            }
        } else {
            float sum = 0.0f;
            for (uint64_t c = 0; c < width; ++c) {
                float e = expf(SM_VALUE(c) - max_value);
                store_f(dst, SM_DST(c), e);
                sum += e;
            }
            for (uint64_t c = 0; c < width; ++c) {
                uint64_t o = SM_DST(c);
                store_f(dst, o, load_f(dst, o) / sum);
            }
        }
#undef SM_VALUE
#undef SM_DST
    }
    return ORACLE_OK;
}

int oracle_soft_max(const oracle_view* src, const oracle_view* dst) { return soft_max_core(src, NULL, dst, 1.0f, 0); }

/* OpDiagMaskInf then OpSoftMax (diag.rs:144-161, reductions.rs:565-638):
 * the two events in sequence, the mask's result held in `scratch` (side^2
 * floats) and read by the soft_max as a dense [side, side] view. */
int oracle_soft_max_diag_mask_inf(const float* input, uint64_t input_len, float* output, uint64_t output_len,
                                  int32_t n_past, float* scratch) {
    int st = oracle_diag_mask(0, input, input_len, scratch, output_len, n_past);
    if (st != ORACLE_OK) return st;
    uint64_t side = 0;
    diag_square_side(input_len, &side);
    const uint64_t ne[4] = {side, side, 1, 1};
    const uint64_t nb[4] = {4, 4 * side, 4 * side * side, 4 * side * side};
    oracle_view src, dst;
    memset(&src, 0, sizeof src);
    memset(&dst, 0, sizeof dst);
    src.data = scratch;
    dst.data = output;
    src.storage_bytes = dst.storage_bytes = input_len * 4;
    for (int d = 0; d < 4; ++d) {
        src.ne[d] = dst.ne[d] = ne[d];
        src.nb[d] = dst.nb[d] = nb[d];
    }
    src.dtype = dst.dtype = DT_F32;
    return soft_max_core(&src, NULL, &dst, 1.0f, 0);
}

int oracle_soft_max_ext(const oracle_view* src, const oracle_view* mask, const oracle_view* dst, float scale) {
    return soft_max_core(src, mask, dst, scale, 1);
}

/* ---------------------------------------------------------------------- */
/* Reductions: reductions.rs:448-463 guards, 671-730 loops                */
/* ---------------------------------------------------------------------- */

static int scalar_output(const oracle_view* dst) {
    return dst->ne[0] == 1 && dst->ne[1] == 1 && dst->ne[2] == 1 && dst->ne[3] == 1;
}

static int rows_output(const oracle_view* src, const oracle_view* dst) {
    return dst->ne[0] == 1 && dst->ne[1] == src->ne[1] && dst->ne[2] == src->ne[2] && dst->ne[3] == src->ne[3];
}

int oracle_sum_f64(const oracle_view* src, double* out) {
    uint64_t n;
    if (!validate_as(src, DT_F32, 0, &n)) return ORACLE_INVALID_VIEW;
    uint64_t ss[4];
    effective_strides(src, 4, ss);
    double sum = 0.0;
    walker w;
    walker_init(&w, src, ss, 0);
    for (uint64_t i = 0; i < n; ++i) {
        sum += (double)load_f(src, w.off);
        walker_next(&w);
    }
    *out = sum;
    return ORACLE_OK;
}

int oracle_sum(const oracle_view* src, const oracle_view* dst) {
    if (!validate_as(src, DT_F32, 0, NULL) || !validate_as(dst, DT_F32, 0, NULL)) return ORACLE_INVALID_VIEW;
    if (!scalar_output(dst)) return ORACLE_SHAPE_MISMATCH;
    double sum;
    oracle_sum_f64(src, &sum);
    store_f(dst, 0, (float)sum);
    return ORACLE_OK;
}

int oracle_mean(const oracle_view* src, const oracle_view* dst) {
    uint64_t n;
    if (!validate_as(src, DT_F32, 0, &n) || !validate_as(dst, DT_F32, 0, NULL)) return ORACLE_INVALID_VIEW;
    if (!scalar_output(dst)) return ORACLE_SHAPE_MISMATCH;
    double sum;
    oracle_sum_f64(src, &sum);
    store_f(dst, 0, (float)(sum / (double)n));
    return ORACLE_OK;
}

int oracle_sum_rows(const oracle_view* src, const oracle_view* dst) {
    uint64_t n;
    if (!validate_as(src, DT_F32, 0, &n) || !validate_as(dst, DT_F32, 0, NULL)) return ORACLE_INVALID_VIEW;
    if (!rows_output(src, dst)) return ORACLE_SHAPE_MISMATCH;
    uint64_t ss[4], sd[4];
    effective_strides(src, 4, ss);
    effective_strides(dst, 4, sd);
    uint64_t width = src->ne[0], rows = n / width;
    for (uint64_t r = 0; r < rows; ++r) {
        double sum = 0.0;
        uint64_t xb = ordinal_offset(src, ss, r * width);
        for (uint64_t c = 0; c < width; ++c) sum += (double)load_f(src, xb + c * ss[0]);
        store_f(dst, ordinal_offset(dst, sd, r), (float)sum);
    }
    return ORACLE_OK;
}

/* reductions.rs:715-730: first index of the strict running maximum. */
static uint64_t argmax_scan(const oracle_view* src, const uint64_t ss[4], uint64_t begin, uint64_t end,
                            float* best_out) {
    uint64_t best_index = begin;
    walker w;
    walker_init(&w, src, ss, begin);
    float best_value = load_f(src, w.off);
    for (uint64_t i = begin + 1; i < end; ++i) {
        walker_next(&w);
        float v = load_f(src, w.off);
        if (v > best_value) {
            best_value = v;
            best_index = i;
        }
    }
    if (best_out) *best_out = best_value;
    return best_index;
}

int oracle_argmax_index(const oracle_view* src, int64_t* index, float* value) {
    uint64_t n;
    if (!validate_as(src, DT_F32, 0, &n)) return ORACLE_INVALID_VIEW;
    uint64_t ss[4];
    effective_strides(src, 4, ss);
    float best;
    uint64_t i = argmax_scan(src, ss, 0, n, &best);
    if (index) *index = (int64_t)i;
    if (value) *value = best;
    return ORACLE_OK;
}

/* Scalar destination: F32 (the reference's index-as-f32, exact below 2^24)
 * or I64 (exact index, this build's extension). */
static int index_output_valid(const oracle_view* dst) {
    return validate_as(dst, DT_F32, 0, NULL) || validate_as(dst, DT_I64, 0, NULL) ||
           validate_as(dst, DT_I32, 0, NULL);
}

static void store_index(const oracle_view* dst, uint64_t off, uint64_t index) {
    unsigned char* p = (unsigned char*)dst->data + off;
    if (dst->dtype == DT_F32) {
        float f = (float)index;
        memcpy(p, &f, 4);
    } else if (dst->dtype == DT_I64) {
        int64_t v = (int64_t)index;
        memcpy(p, &v, 8);
    } else {
        int32_t v = (int32_t)index;
        memcpy(p, &v, 4);
    }
}

int oracle_argmax(const oracle_view* src, const oracle_view* dst) {
    uint64_t n;
    if (!validate_as(src, DT_F32, 0, &n) || !index_output_valid(dst)) return ORACLE_INVALID_VIEW;
    if (!scalar_output(dst)) return ORACLE_SHAPE_MISMATCH;
    uint64_t ss[4];
    effective_strides(src, 4, ss);
    store_index(dst, 0, argmax_scan(src, ss, 0, n, NULL));
    return ORACLE_OK;
}

/* Per-row argmax: the reductions.rs:715-730 scan applied to each ne0 row;
 * index is the column within the row. */
int oracle_argmax_rows(const oracle_view* src, const oracle_view* dst) {
    uint64_t n;
    if (!validate_as(src, DT_F32, 0, &n) || !index_output_valid(dst)) return ORACLE_INVALID_VIEW;
    if (!rows_output(src, dst)) return ORACLE_SHAPE_MISMATCH;
    uint64_t ss[4], sd[4];
    effective_strides(src, 4, ss);
    effective_strides(dst, dtype_size(dst->dtype), sd);
    uint64_t width = src->ne[0], rows = n / width;
    for (uint64_t r = 0; r < rows; ++r) {
        uint64_t i = argmax_scan(src, ss, r * width, r * width + width, NULL);
        store_index(dst, ordinal_offset(dst, sd, r), i - r * width);
    }
    return ORACLE_OK;
}

/* ---------------------------------------------------------------------- */
/* Generic operation envelope: crates/emel-kernels/src/any/generic.rs      */
/* ---------------------------------------------------------------------- */

/* validate_span (generic.rs:822-862). */
static int generic_span(const oracle_view* v, uint64_t nb[4], uint64_t* count) {
    if (v->dtype == DT_F32) {
        if (!effective_strides(v, 4, nb)) return 0;
    } else {
        memcpy(nb, v->nb, sizeof(uint64_t) * 4);
    }
    uint64_t c = 1;
    for (int d = 0; d < 4; ++d) {
        if (v->ne[d] == 0 || __builtin_mul_overflow(c, v->ne[d], &c)) return 0;
        if (v->ne[d] > 1 && nb[d] == 0) return 0;
    }
    u128 max_offset = 0;
    for (int d = 0; d < 4; ++d) {
        u128 term = (u128)(v->ne[d] - 1) * (u128)nb[d];
        if (__builtin_add_overflow(max_offset, term, &max_offset)) return 0;
    }
    u128 end;
    if (__builtin_add_overflow(max_offset, (u128)1, &end)) return 0;
    if (end > (u128)v->storage_bytes) return 0;
    *count = c;
    return 1;
}

/* RawTensorView::f32_valid (generic.rs:467-473). */
static int generic_f32(const oracle_view* v, uint64_t nb[4], uint64_t* count) {
    if (v == NULL || v->dtype != DT_F32) return 0;
    if (!generic_span(v, nb, count)) return 0;
    for (int d = 0; d < 4; ++d)
        if (nb[d] < 4) return 0;
    return 1;
}

/* read_f32_index / write_f32_index (generic.rs:474-482, 553-578): ordinal ->
 * coordinates -> byte offset; unaligned bytes are fine on the host. */
static float generic_read(const oracle_view* v, const uint64_t nb[4], uint64_t index) {
    float f;
    memcpy(&f, (const unsigned char*)v->data + ordinal_offset(v, nb, index), 4);
    return f;
}

static void generic_write(const oracle_view* v, const uint64_t nb[4], uint64_t index, float value) {
    memcpy((unsigned char*)v->data + ordinal_offset(v, nb, index), &value, 4);
}

static int generic_param(const oracle_generic_request* r, int slot, float* out) {
    uint32_t end = (uint32_t)slot * 4u + 4u;
    if (end > r->params_len) return 0;
    memcpy(out, r->params + slot * 4, 4);
    return 1;
}

/* f32::max(a, b) with the first argument the running maximum: a NaN operand
 * is ignored (an equal pair keeps the running value). */
static inline float rs_max(float a, float b) {
    if (isnan(b)) return a;
    if (isnan(a)) return b;
    return b > a ? b : a;
}

/* execute_generic_unary formulas (generic.rs:1307-1350). */
static float generic_unary_apply(int code, float v) {
    switch (code) {
    case 0: return fabsf(v);
    case 1: return -v;
    case 2: return tanhf(v);
    case 3: return v > 0.0f ? v : expm1f(v);
    case 4: return rs_max(v, 0.0f) == 0.0f ? 0.0f : rs_max(v, 0.0f); /* f32::max(v, 0.0); zeros -> +0 */
    case 5: {
        float rounded = v; /* f32::from_ne_bytes(value.to_ne_bytes()) */
        return 0.5f * rounded * (1.0f + tanhf(0.7978846f * fmaf(0.044715f * rounded * rounded, rounded, rounded)));
    }
    case 6: return v / (1.0f + expf(-v));
    case 7: return expf(v);
    case 8: return v * v;
    case 9: return sqrtf(v);
    case 10: return logf(v);
    case 11: return sinf(v);
    case 12: return cosf(v);
    default: return v;
    }
}

int oracle_generic(const oracle_generic_request* r) {
    if (r == NULL || r->op >= 95 || r->params_len > 64) return ORACLE_INVALID_ARGUMENT;
    const oracle_view* all[4] = {r->src0, r->src1, r->src2, r->dst};
    for (int k = 0; k < 4; ++k) {
        uint64_t nb[4], count;
        if (all[k] != NULL && !generic_span(all[k], nb, &count)) return ORACLE_INVALID_SHAPE;
    }
    uint64_t n0[4], n1[4], nd[4], c0 = 0, c1 = 0, cd = 0;
    const int v0 = generic_f32(r->src0, n0, &c0);
    const int v1 = generic_f32(r->src1, n1, &c1);
    const int vd = generic_f32(r->dst, nd, &cd);
    float pa = 0.0f, pb = 0.0f;
    int unary_code = -1;
    switch (r->op) {
    case 85:
        switch (r->unary_subop) { /* UnarySubOp -> execute_generic_unary selector */
        case 0: unary_code = 0; break;
        case 2: unary_code = 1; break;
        case 4: unary_code = 2; break;
        case 5: unary_code = 3; break;
        case 6: unary_code = 4; break;
        case 8: unary_code = 5; break;
        case 10: unary_code = 6; break;
        case 13: unary_code = 7; break;
        default: return ORACLE_INVALID_SHAPE;
        }
        /* fallthrough */
    case 8: case 9: case 10: case 11: case 12:
        if (unary_code < 0) unary_code = (int)r->op; /* 8..12: sqr sqrt ln sin cos */
        /* fallthrough */
    case 0:
        if (!(v0 && vd && c0 == cd)) return ORACLE_INVALID_SHAPE;
        for (uint64_t i = 0; i < c0; ++i) {
            float x = generic_read(r->src0, n0, i);
            generic_write(r->dst, nd, i, r->op == 0 ? x : generic_unary_apply(unary_code, x));
        }
        return ORACLE_OK;
    case 1: case 5: case 6: case 7: { /* execute_generic_binary (generic.rs:1280-1305) */
        if (!(v0 && v1 && vd && c0 == c1 && c0 == cd)) return ORACLE_INVALID_SHAPE;
        for (uint64_t i = 0; i < c0; ++i) {
            float a = generic_read(r->src0, n0, i), b = generic_read(r->src1, n1, i), y;
            switch (r->op) {
            case 1: y = a + b; break;
            case 5: y = a - b; break;
            case 6: y = a * b; break;
            default: y = a / b; break;
            }
            generic_write(r->dst, nd, i, y);
        }
        return ORACLE_OK;
    }
    case 3: case 32: case 70: { /* execute_generic_scalar (generic.rs:1515-1544) */
        if (!(v0 && vd && c0 == cd && generic_param(r, 0, &pa) && isfinite(pa))) return ORACLE_INVALID_SHAPE;
        for (uint64_t i = 0; i < c0; ++i) {
            float x = generic_read(r->src0, n0, i);
            float y = r->op == 3 ? x + pa : (r->op == 32 ? x * pa : (x < 0.0f ? x * pa : x));
            generic_write(r->dst, nd, i, y);
        }
        return ORACLE_OK;
    }
    case 50: /* execute_generic_clamp (generic.rs:1546-1563): f32::clamp */
        if (!(v0 && vd && c0 == cd && generic_param(r, 0, &pa) && generic_param(r, 1, &pb) && isfinite(pa) &&
              isfinite(pb) && pa <= pb))
            return ORACLE_INVALID_SHAPE;
        for (uint64_t i = 0; i < c0; ++i) generic_write(r->dst, nd, i, clampf_rs(generic_read(r->src0, n0, i), pa, pb));
        return ORACLE_OK;
    case 22: /* execute_generic_silu_back (generic.rs:1565-1585) */
        if (!(v0 && v1 && vd && same_ne(r->src0, r->src1) && same_ne(r->src0, r->dst))) return ORACLE_INVALID_SHAPE;
        for (uint64_t i = 0; i < c0; ++i) {
            float x = generic_read(r->src0, n0, i);
            float sigmoid = 1.0f / (1.0f + expf(-x));
            float derivative = sigmoid * (1.0f + x * (1.0f - sigmoid));
            generic_write(r->dst, nd, i, generic_read(r->src1, n1, i) * derivative);
        }
        return ORACLE_OK;
    case 19: { /* execute_generic_repeat (generic.rs:1641-1665) */
        if (!(v0 && vd)) return ORACLE_INVALID_SHAPE;
        for (int d = 0; d < 4; ++d)
            if (r->dst->ne[d] % r->src0->ne[d] != 0) return ORACLE_INVALID_SHAPE;
        for (uint64_t o = 0; o < cd; ++o) {
            uint64_t rest = o, src_ordinal = 0, stride = 1;
            for (int d = 0; d < 4; ++d) {
                uint64_t coordinate = rest % r->dst->ne[d];
                rest /= r->dst->ne[d];
                src_ordinal += (coordinate % r->src0->ne[d]) * stride;
                stride *= r->src0->ne[d];
            }
            uint32_t word; /* a raw copy */
            memcpy(&word, (const unsigned char*)r->src0->data + ordinal_offset(r->src0, n0, src_ordinal), 4);
            memcpy((unsigned char*)r->dst->data + ordinal_offset(r->dst, nd, o), &word, 4);
        }
        return ORACLE_OK;
    }
    case 13: case 16: { /* execute_generic_reduce_sum / _mean (generic.rs:1354-1392) */
        if (!(v0 && vd && cd == 1)) return ORACLE_INVALID_SHAPE;
        double sum = 0.0;
        for (uint64_t i = 0; i < c0; ++i) sum += (double)generic_read(r->src0, n0, i);
        generic_write(r->dst, nd, 0, r->op == 13 ? (float)sum : (float)(sum / (double)c0));
        return ORACLE_OK;
    }
    case 17: { /* execute_generic_argmax (generic.rs:1394-1416) */
        if (!(v0 && vd && cd == 1)) return ORACLE_INVALID_SHAPE;
        uint64_t best_index = 0;
        float best = generic_read(r->src0, n0, 0);
        for (uint64_t i = 1; i < c0; ++i) {
            float x = generic_read(r->src0, n0, i);
            if (x > best) {
                best = x;
                best_index = i;
            }
        }
        generic_write(r->dst, nd, 0, (float)best_index);
        return ORACLE_OK;
    }
    case 46: { /* execute_generic_soft_max (generic.rs:1952-1989) */
        if (!(v0 && vd && c0 == cd)) return ORACLE_INVALID_SHAPE;
        uint64_t width = r->src0->ne[0], rows = c0 / width;
        for (uint64_t row = 0; row < rows; ++row) {
            float maximum = -INFINITY;
            for (uint64_t c = 0; c < width; ++c) maximum = rs_max(maximum, generic_read(r->src0, n0, row * width + c));
            float sum = 0.0f;
            for (uint64_t c = 0; c < width; ++c) {
                float e = expf(generic_read(r->src0, n0, row * width + c) - maximum);
                generic_write(r->dst, nd, row * width + c, e);
                sum += e;
            }
            for (uint64_t c = 0; c < width; ++c)
                generic_write(r->dst, nd, row * width + c, generic_read(r->dst, nd, row * width + c) / sum);
        }
        return ORACLE_OK;
    }
    case 23: case 24: { /* execute_generic_norm (generic.rs:1992-2050) */
        if (!(v0 && vd && same_ne(r->src0, r->dst) && generic_param(r, 0, &pa) && isfinite(pa) && pa >= 0.0f))
            return ORACLE_INVALID_SHAPE;
        const int rms = r->op == 24;
        uint64_t width = r->src0->ne[0], rows = c0 / width;
        for (uint64_t row = 0; row < rows; ++row) {
            double sum = 0.0;
            for (uint64_t c = 0; c < width; ++c) {
                float x = generic_read(r->src0, n0, row * width + c);
                sum += rms ? (double)(x * x) : (double)x;
            }
            float mean = (float)(sum / (double)width);
            double variance = 0.0;
            if (!rms) {
                for (uint64_t c = 0; c < width; ++c) {
                    float centered = generic_read(r->src0, n0, row * width + c) - mean;
                    variance += (double)(centered * centered);
                }
                variance /= (double)width;
            }
            float scale = (float)(1.0 / sqrt((rms ? (double)mean : variance) + (double)pa));
            for (uint64_t c = 0; c < width; ++c) {
                float x = generic_read(r->src0, n0, row * width + c);
                generic_write(r->dst, nd, row * width + c, rms ? x * scale : (x - mean) * scale);
            }
        }
        return ORACLE_OK;
    }
    default:
        return ORACLE_UNSUPPORTED_OPERATION;
    }
}
