// GGUF tensor tables feeding device buffers: the scanner of emel-gguf's
// loader (crates/emel-gguf/src/loader/detail.rs: probe 294-359, parse
// 361-530; lifecycle Loader::probe / bind / parse, loader/mod.rs:137-232)
// restated for the tensor records, with the same error classes, plus the
// upload of one tensor's serialized blocks into device memory and the view
// the device kernels consume (row gather, vocabulary argmax).
//
// Image layout (GGUF v3): "GGUF", version u32, tensor_count u64, kv_count
// u64; kv_count entries (key string, value type u32, value); tensor_count
// records (name string, dimension count u32, dimensions u64 each, type u32,
// data offset u64); padding to the alignment (general.alignment, default
// 32); the tensor-data section, each tensor at its offset, every offset the
// running sum of the previous tensors' sizes padded to the alignment.
#include <cstring>
#include <string>
#include <unordered_set>

#include <cuda_runtime.h>

#include "emel_cuda.h"

namespace {

constexpr uint32_t kVersion = 3;
constexpr uint32_t kDefaultAlignment = 32;
constexpr uint32_t kMaxDims = 4;
constexpr uint64_t kMaxString = 1024ull * 1024 * 1024;
constexpr uint64_t kMaxArray = 1024ull * 1024 * 1024;
enum : uint32_t { kU8, kI8, kU16, kI16, kU32, kI32, kF32, kBool, kString, kArray, kU64, kI64, kF64, kTypeCount };
constexpr char kAlignmentKey[] = "general.alignment";

// Serialized layout of a tensor type: `bytes` per group of `columns` values
// of `rows` rows; `min_dims` dimensions at least (emel-tensor dtype.rs:
// wire codes 176-212, layouts 261-320).  bytes == 0: not a GGUF type.
struct Layout {
    uint32_t columns, rows, bytes, min_dims;
};

Layout layout_of(uint32_t code) {
    switch (code) {
    case 0: case 26: return {1, 1, 4, 0};             // F32, I32
    case 1: case 25: case 30: return {1, 1, 2, 0};    // F16, I16, BF16
    case 2: case 20: return {32, 1, 18, 0};           // Q4_0, IQ4_NL
    case 3: return {32, 1, 20, 0};                    // Q4_1
    case 6: return {32, 1, 22, 0};                    // Q5_0
    case 7: return {32, 1, 24, 0};                    // Q5_1
    case 8: return {32, 1, 34, 0};                    // Q8_0
    case 9: return {32, 1, 36, 0};                    // Q8_1
    case 10: return {256, 1, 84, 0};                  // Q2_K
    case 11: case 21: return {256, 1, 110, 0};        // Q3_K, IQ3_S
    case 12: return {256, 1, 144, 0};                 // Q4_K
    case 13: return {256, 1, 176, 0};                 // Q5_K
    case 14: return {256, 1, 210, 0};                 // Q6_K
    case 15: return {256, 1, 292, 0};                 // Q8_K
    case 16: case 35: return {256, 1, 66, 0};         // IQ2_XXS, TQ2_0
    case 17: return {256, 1, 74, 0};                  // IQ2_XS
    case 18: return {256, 1, 98, 0};                  // IQ3_XXS
    case 19: return {256, 1, 50, 0};                  // IQ1_S
    case 22: return {256, 1, 82, 0};                  // IQ2_S
    case 23: return {256, 1, 136, 0};                 // IQ4_XS
    case 24: return {1, 1, 1, 0};                     // I8
    case 27: case 28: return {1, 1, 8, 0};            // I64, F64
    case 29: return {256, 1, 56, 0};                  // IQ1_M
    case 34: return {256, 1, 54, 0};                  // TQ1_0
    case 39: return {32, 1, 17, 0};                   // MXFP4
    case 41: case 42: return {256, 8, 1152, 2};       // Q4_K x8 interleaved (two block-row layouts)
    default: return {0, 0, 0, 0};
    }
}

bool mul_ok(uint64_t a, uint64_t b, uint64_t* out) { return !__builtin_mul_overflow(a, b, out); }
bool add_ok(uint64_t a, uint64_t b, uint64_t* out) { return !__builtin_add_overflow(a, b, out); }

// Unpadded payload size (dtype.rs serialized_data_size): the first
// dimension in whole groups of columns, the rest multiplied into rows,
// rounded up to whole row groups.
emel_cuda_status data_size(uint32_t code, const uint64_t dims[4], uint32_t count, uint64_t* out) {
    const Layout l = layout_of(code);
    if (l.bytes == 0) return EMEL_CUDA_MODEL_INVALID;
    if (count < l.min_dims) return EMEL_CUDA_MODEL_INVALID;
    const uint64_t columns = count > 0 ? dims[0] : 1;
    if (columns % l.columns != 0) return EMEL_CUDA_MODEL_INVALID;
    uint64_t rows = 1;
    for (uint32_t d = 1; d < count; ++d)
        if (!mul_ok(rows, dims[d], &rows)) return EMEL_CUDA_CAPACITY;
    const uint64_t row_groups = rows / l.rows + (rows % l.rows != 0 ? 1 : 0);
    uint64_t groups = 0;
    if (!mul_ok(columns / l.columns, row_groups, &groups) || !mul_ok(groups, l.bytes, out)) return EMEL_CUDA_CAPACITY;
    return EMEL_CUDA_OK;
}

emel_cuda_status align_up(uint64_t v, uint32_t a, uint64_t* out) {
    const uint64_t r = v % a;
    if (r == 0) {
        *out = v;
        return EMEL_CUDA_OK;
    }
    return add_ok(v, a - r, out) ? EMEL_CUDA_OK : EMEL_CUDA_CAPACITY;
}

struct Reader {
    const uint8_t* p;
    uint64_t n, off;
    bool take(uint64_t count, const uint8_t** at) {
        if (count > n - off) return false;
        *at = p + off;
        off += count;
        return true;
    }
    bool u32(uint32_t* v) {
        const uint8_t* at;
        if (!take(4, &at)) return false;
        std::memcpy(v, at, 4);  // little-endian host
        return true;
    }
    bool u64(uint64_t* v) {
        const uint8_t* at;
        if (!take(8, &at)) return false;
        std::memcpy(v, at, 8);
        return true;
    }
    bool str(const uint8_t** s, uint64_t* len) {
        uint64_t l;
        if (!u64(&l) || l > kMaxString) return false;
        *len = l;
        return take(l, s);
    }
};

uint32_t scalar_bytes(uint32_t t) {
    switch (t) {
    case kU8: case kI8: case kBool: return 1;
    case kU16: case kI16: return 2;
    case kU32: case kI32: case kF32: return 4;
    case kU64: case kI64: case kF64: return 8;
    default: return 0;
    }
}

// One metadata value (detail.rs scan_value 173-237): validated and skipped;
// general.alignment must be a u32 power of two and sets the alignment.
emel_cuda_status scan_value(Reader& r, uint32_t type, bool is_alignment, uint32_t* alignment) {
    if (type >= kTypeCount) return EMEL_CUDA_MODEL_INVALID;
    if (is_alignment && type != kU32) return EMEL_CUDA_MODEL_INVALID;
    const uint8_t* s;
    uint64_t len;
    if (type == kString) return r.str(&s, &len) ? EMEL_CUDA_OK : EMEL_CUDA_PARSE_FAILED;
    if (type == kArray) {
        uint32_t et;
        uint64_t count;
        if (!r.u32(&et) || !r.u64(&count)) return EMEL_CUDA_PARSE_FAILED;
        if (et >= kTypeCount || et == kArray || count > kMaxArray) return EMEL_CUDA_MODEL_INVALID;
        if (et == kString) {
            for (uint64_t i = 0; i < count; ++i)
                if (!r.str(&s, &len)) return EMEL_CUDA_PARSE_FAILED;
            return EMEL_CUDA_OK;
        }
        uint64_t bytes;
        if (!mul_ok(count, scalar_bytes(et), &bytes)) return EMEL_CUDA_CAPACITY;
        return r.take(bytes, &s) ? EMEL_CUDA_OK : EMEL_CUDA_PARSE_FAILED;
    }
    if (is_alignment) {
        uint32_t v;
        if (!r.u32(&v)) return EMEL_CUDA_PARSE_FAILED;
        if (v == 0 || (v & (v - 1)) != 0) return EMEL_CUDA_MODEL_INVALID;
        *alignment = v;
        return EMEL_CUDA_OK;
    }
    return r.take(scalar_bytes(type), &s) ? EMEL_CUDA_OK : EMEL_CUDA_PARSE_FAILED;
}

// The walk shared by probe and parse.  tensors == nullptr: probe only.
emel_cuda_status walk(const uint8_t* image, uint64_t size, emel_gguf_requirements* req, emel_gguf_tensor_info* tensors) {
    Reader r{image, size, 0};
    const uint8_t* magic;
    uint32_t version;
    uint64_t tensor_count, kv_count;
    if (!r.take(4, &magic) || std::memcmp(magic, "GGUF", 4) != 0 || !r.u32(&version) || !r.u64(&tensor_count) ||
        !r.u64(&kv_count) || version != kVersion)
        return size < 4 ? EMEL_CUDA_PARSE_FAILED : EMEL_CUDA_MODEL_INVALID;  // detail.rs header_error
    if (tensor_count > UINT32_MAX || kv_count > UINT32_MAX) return EMEL_CUDA_CAPACITY;
    if (tensors != nullptr && (tensor_count != req->tensor_count || kv_count != req->kv_count))
        return EMEL_CUDA_INVALID_REQUEST;  // parse of a different image than the one probed
    emel_gguf_requirements q{};
    q.tensor_count = (uint32_t)tensor_count;
    q.kv_count = (uint32_t)kv_count;
    uint32_t alignment = kDefaultAlignment;
    std::unordered_set<std::string> seen;
    for (uint64_t i = 0; i < kv_count; ++i) {
        const uint8_t* key;
        uint64_t klen;
        if (!r.str(&key, &klen)) return EMEL_CUDA_PARSE_FAILED;
        if (klen == 0 || !seen.emplace(reinterpret_cast<const char*>(key), klen).second) return EMEL_CUDA_MODEL_INVALID;
        uint32_t type;
        if (!r.u32(&type)) return EMEL_CUDA_PARSE_FAILED;
        const uint64_t start = r.off;
        const bool is_alignment = klen == sizeof(kAlignmentKey) - 1 && std::memcmp(key, kAlignmentKey, klen) == 0;
        const emel_cuda_status st = scan_value(r, type, is_alignment, &alignment);
        if (st != EMEL_CUDA_OK) return st;
        const uint64_t vlen = r.off - start;
        if (klen > UINT32_MAX || vlen > UINT32_MAX) return EMEL_CUDA_CAPACITY;
        if (klen > q.max_key_bytes) q.max_key_bytes = (uint32_t)klen;
        if (vlen > q.max_value_bytes) q.max_value_bytes = (uint32_t)vlen;
    }
    seen.clear();
    uint64_t expected = 0;
    for (uint64_t i = 0; i < tensor_count; ++i) {
        const uint64_t name_at = r.off + 8;
        const uint8_t* name;
        uint64_t nlen;
        if (!r.str(&name, &nlen)) return EMEL_CUDA_PARSE_FAILED;
        if (!seen.emplace(reinterpret_cast<const char*>(name), nlen).second) return EMEL_CUDA_MODEL_INVALID;
        uint32_t ndims;
        if (!r.u32(&ndims)) return EMEL_CUDA_PARSE_FAILED;
        if (ndims > kMaxDims) return EMEL_CUDA_MODEL_INVALID;
        uint64_t dims[4] = {1, 1, 1, 1};
        for (uint32_t d = 0; d < ndims; ++d)
            if (!r.u64(&dims[d])) return EMEL_CUDA_PARSE_FAILED;
        uint32_t type;
        if (!r.u32(&type)) return EMEL_CUDA_PARSE_FAILED;
        if (layout_of(type).bytes == 0) return EMEL_CUDA_MODEL_INVALID;
        uint64_t offset;
        if (!r.u64(&offset)) return EMEL_CUDA_PARSE_FAILED;
        uint64_t bytes;
        emel_cuda_status st = data_size(type, dims, ndims, &bytes);
        if (st != EMEL_CUDA_OK) return st;
        if (!add_ok(q.tensor_data_bytes, bytes, &q.tensor_data_bytes)) return EMEL_CUDA_CAPACITY;
        if (offset != expected) return EMEL_CUDA_PARSE_FAILED;
        uint64_t padded;
        if ((st = align_up(bytes, alignment, &padded)) != EMEL_CUDA_OK) return st;
        if (!add_ok(expected, padded, &expected)) return EMEL_CUDA_CAPACITY;
        if (tensors != nullptr) {
            emel_gguf_tensor_info& t = tensors[i];
            std::memset(&t, 0, sizeof(t));
            if (name_at > UINT32_MAX || nlen > UINT32_MAX) return EMEL_CUDA_CAPACITY;
            t.name_offset = (uint32_t)name_at;
            t.name_length = (uint32_t)nlen;
            t.tensor_type = type;
            t.dimension_count = ndims;
            for (int d = 0; d < 4; ++d) t.dimensions[d] = dims[d];
            t.data_offset = offset;
            t.alignment = alignment;
            t.data_size = bytes;
        }
    }
    if (tensor_count != 0) {
        uint64_t aligned;
        const emel_cuda_status st = align_up(r.off, alignment, &aligned);
        if (st != EMEL_CUDA_OK) return st;
        if (aligned > size) return EMEL_CUDA_PARSE_FAILED;
        r.off = aligned;
    }
    const uint64_t section = r.off;
    uint64_t required;
    if (!add_ok(section, expected, &required)) return EMEL_CUDA_CAPACITY;
    if (required > size) return EMEL_CUDA_PARSE_FAILED;
    if (tensors != nullptr) {
        for (uint64_t i = 0; i < tensor_count; ++i) {
            emel_gguf_tensor_info& t = tensors[i];
            if (t.data_offset % alignment != 0) return EMEL_CUDA_PARSE_FAILED;
            t.data_section_offset = section;
            uint64_t end;
            if (!add_ok(section, t.data_offset, &t.file_offset) || !add_ok(t.file_offset, t.data_size, &end))
                return EMEL_CUDA_CAPACITY;
            if (end > size) return EMEL_CUDA_PARSE_FAILED;
        }
    } else {
        *req = q;
    }
    return EMEL_CUDA_OK;
}

// Device dtype and element size of the tensor types the kernels consume.
bool device_dtype(uint32_t code, uint32_t* dtype, uint64_t* elem) {
    switch (code) {
    case 0: *dtype = EMEL_DTYPE_F32; *elem = 4; return true;
    case 1: *dtype = EMEL_DTYPE_F16; *elem = 2; return true;
    case 30: *dtype = EMEL_DTYPE_BF16; *elem = 2; return true;
    case 2: case 3: case 6: case 8: case 10: case 11: case 12: case 14: *dtype = code; *elem = 0; return true;
    default: return false;
    }
}

}  // namespace

extern "C" {

emel_cuda_status emel_gguf_probe(const uint8_t* image, uint64_t image_bytes, emel_gguf_requirements* out) {
    if (out == nullptr || (image == nullptr && image_bytes != 0)) return EMEL_CUDA_INVALID_REQUEST;
    std::memset(out, 0, sizeof(*out));
    try {
        return walk(image, image_bytes, out, nullptr);
    } catch (...) {
        return EMEL_CUDA_OUT_OF_MEMORY;
    }
}

emel_cuda_status emel_gguf_parse(const uint8_t* image, uint64_t image_bytes, const emel_gguf_requirements* probed,
                                 emel_gguf_tensor_info* tensors, uint32_t tensor_capacity) {
    if (probed == nullptr || (image == nullptr && image_bytes != 0)) return EMEL_CUDA_INVALID_REQUEST;
    if (tensor_capacity < probed->tensor_count || (probed->tensor_count != 0 && tensors == nullptr))
        return EMEL_CUDA_CAPACITY;
    emel_gguf_requirements q = *probed;
    emel_gguf_tensor_info scratch{};
    try {
        return walk(image, image_bytes, &q, tensors != nullptr ? tensors : &scratch);
    } catch (...) {
        return EMEL_CUDA_OUT_OF_MEMORY;
    }
}

emel_cuda_status emel_gguf_tensor_view(const emel_gguf_tensor_info* t, void* data, uint64_t storage_bytes,
                                       emel_tensor_view* out) {
    if (t == nullptr || out == nullptr) return EMEL_CUDA_INVALID_ARGUMENT;
    uint32_t dtype;
    uint64_t elem;
    if (!device_dtype(t->tensor_type, &dtype, &elem)) return EMEL_CUDA_UNSUPPORTED_OPERATION;
    if (storage_bytes < t->data_size) return EMEL_CUDA_INVALID_ARGUMENT;
    std::memset(out, 0, sizeof(*out));
    for (int d = 0; d < 4; ++d) out->ne[d] = t->dimensions[d];
    if (elem != 0) {
        // dense elements
        out->nb[0] = elem;
        for (int d = 1; d < 4; ++d) out->nb[d] = out->nb[d - 1] * out->ne[d - 1];
    } else {
        // packed blocks: rows of ne[0] values as whole blocks, nb[0] == 1
        // (the block views of the row gather and vocabulary argmax kernels)
        const Layout l = layout_of(t->tensor_type);
        out->nb[0] = 1;
        out->nb[1] = t->dimensions[0] / l.columns * l.bytes;
        out->nb[2] = out->nb[1] * t->dimensions[1];
        out->nb[3] = out->nb[2] * t->dimensions[2];
    }
    out->data = data;
    out->storage_bytes = storage_bytes;
    out->dtype = dtype;
    return EMEL_CUDA_OK;
}

emel_cuda_status emel_gguf_upload(emel_cuda_context* ctx, void* stream, const uint8_t* image, uint64_t image_bytes,
                                  const emel_gguf_tensor_info* t, void* device_dst, uint64_t device_bytes,
                                  emel_tensor_view* view_out) {
    if (ctx == nullptr || image == nullptr || t == nullptr || device_dst == nullptr || view_out == nullptr)
        return EMEL_CUDA_INVALID_ARGUMENT;
    uint64_t end;
    if (!add_ok(t->file_offset, t->data_size, &end) || end > image_bytes) return EMEL_CUDA_PARSE_FAILED;
    const emel_cuda_status st = emel_gguf_tensor_view(t, device_dst, device_bytes, view_out);
    if (st != EMEL_CUDA_OK) return st;
    return emel_cuda_memcpy_h2d(ctx, stream, device_dst, image + t->file_offset, t->data_size);
}

}  // extern "C"
