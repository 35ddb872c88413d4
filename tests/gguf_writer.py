"""Writes GGUF v3 images (the layout emel-gguf's loader reads,
crates/emel-gguf/src/loader/detail.rs): header, metadata entries, tensor
records, padding to the alignment, tensor data at padded running offsets.
Used by the tests to build synthetic model files from seeded blocks."""

import struct

GGUF_U8, GGUF_I8, GGUF_U16, GGUF_I16, GGUF_U32, GGUF_I32, GGUF_F32, GGUF_BOOL, GGUF_STRING, GGUF_ARRAY, GGUF_U64, \
    GGUF_I64, GGUF_F64 = range(13)


def u32(v):
    return struct.pack("<I", v)


def u64(v):
    return struct.pack("<Q", v)


def string(b):
    return u64(len(b)) + b


def kv(key, kind, payload):
    return string(key) + u32(kind) + payload


def array(kind, count, payload):
    return u32(kind) + u64(count) + payload


def pad_to(buf, alignment):
    return buf + b"\0" * ((-len(buf)) % alignment)


def image(tensors, metadata=(), alignment=None, version=3):
    """tensors: list of (name bytes, dims list (ne order), type code,
    payload bytes).  metadata: list of (key, kind, payload).  With
    `alignment`, a general.alignment entry is written first."""
    entries = list(metadata)
    if alignment is not None:
        entries.insert(0, (b"general.alignment", GGUF_U32, u32(alignment)))
    align = alignment or 32
    out = b"GGUF" + u32(version) + u64(len(tensors)) + u64(len(entries))
    for key, kind, payload in entries:
        out += kv(key, kind, payload)
    offset = 0
    for name, dims, ttype, payload in tensors:
        out += string(name) + u32(len(dims)) + b"".join(u64(d) for d in dims) + u32(ttype) + u64(offset)
        offset += len(payload) + (-len(payload)) % align
    if tensors:
        out = pad_to(out, align)
    for _, _, _, payload in tensors:
        out += pad_to(payload, align)
    return out
