"""The GGUF tensor-table loader (emel_gguf_probe / emel_gguf_parse /
emel_gguf_tensor_view) against the reference loader's own known answers
(crates/emel-gguf/src/loader/detail.rs tests 560-688 and
crates/emel-gguf/tests/loader.rs: the fixtures are rebuilt byte for byte
from those tests' construction steps), plus images written by
tests/gguf_writer.py.  Host code only: no device is touched."""

import ctypes

import pytest

import gguf_writer as gw
from gguf_writer import GGUF_ARRAY, GGUF_F32, GGUF_STRING, GGUF_U16, GGUF_U32, GGUF_U64, GGUF_U8, u32, u64


def probe(emel, data):
    buf = ctypes.create_string_buffer(bytes(data), max(1, len(data)))
    req = emel.CGgufRequirements()
    st = emel.lib().emel_gguf_probe(buf if data else None, len(data), ctypes.byref(req))
    return emel.Status(st), req


def parser_fixture():
    """detail.rs parser_fixture: ten metadata entries (alignment 64 first),
    one F32 tensor of 4 values at offset 0, data section padded to 64."""
    strings = gw.string(b"one") + gw.string(b"two")
    entries = [(b"general.alignment", GGUF_U32, u32(64)), (b"byte", GGUF_U8, bytes([7])),
               (b"word", GGUF_U16, (513).to_bytes(2, "little")), (b"wide", GGUF_U64, u64(9)),
               (b"float", GGUF_F32, bytes.fromhex("0000a03f")), (b"text", GGUF_STRING, gw.string(b"value")),
               (b"bytes", GGUF_ARRAY, gw.array(GGUF_U8, 3, bytes([1, 2, 3]))),
               (b"words", GGUF_ARRAY, gw.array(GGUF_U16, 2, bytes([1, 0, 2, 0]))),
               (b"wide-array", GGUF_ARRAY, gw.array(GGUF_U64, 1, u64(5))),
               (b"strings", GGUF_ARRAY, gw.array(GGUF_STRING, 2, strings))]
    out = b"GGUF" + u32(3) + u64(1) + u64(len(entries))
    for k, t, p in entries:
        out += gw.kv(k, t, p)
    out += gw.string(b"weight") + u32(1) + u64(4) + u32(0) + u64(0)
    out = gw.pad_to(out, 64) + b"\0" * 64
    return out


def serialized_tensor_fixture(ttype, dims, data_size):
    """tests/loader.rs serialized_tensor_fixture: one tensor "packed"."""
    out = b"GGUF" + u32(3) + u64(1) + u64(0) + gw.string(b"packed") + u32(len(dims))
    out += b"".join(u64(d) for d in dims) + u32(ttype) + u64(0)
    return gw.pad_to(out, 32) + bytes([7]) * data_size


def test_parser_fixture_known_answers(emel):
    img = emel.GgufImage(parser_fixture())
    req = img.requirements
    assert req.kv_count == 10 and req.tensor_count == 1 and req.tensor_data_bytes == 16
    name, t = img.tensors[0]
    assert name == "weight" and t.data_size == 16 and t.file_offset % 64 == 0 and t.alignment == 64
    assert list(t.dimensions) == [4, 1, 1, 1] and t.dimension_count == 1 and t.tensor_type == 0
    assert img.image[t.file_offset:t.file_offset + 16] == b"\0" * 16


def test_headers_and_alignment_values(emel):
    assert probe(emel, b"")[0] == emel.Status.PARSE_FAILED
    assert probe(emel, b"nope")[0] == emel.Status.MODEL_INVALID
    bad_align = b"GGUF" + u32(3) + u64(0) + u64(1) + gw.kv(b"general.alignment", GGUF_U32, u32(3))
    assert probe(emel, bad_align)[0] == emel.Status.MODEL_INVALID
    assert probe(emel, b"GGUF" + u32(2) + u64(0) + u64(0))[0] == emel.Status.MODEL_INVALID  # version 3 only


def test_packed_wire_codes_and_size_overflows(emel):
    for code in (41, 42):  # Q4_K x8 interleaved: 256 columns x 8 rows per 1152-byte group
        st, req = probe(emel, serialized_tensor_fixture(code, [256, 9], 2304))
        assert st == emel.Status.OK and req.tensor_data_bytes == 2304
    for code in (31, 32, 33, 36, 37, 38, 40, 43, 44, 45, 256, 0xffffffff):
        assert probe(emel, serialized_tensor_fixture(code, [256, 8], 4096))[0] == emel.Status.MODEL_INVALID
    assert probe(emel, serialized_tensor_fixture(0, [2 ** 64 - 1, 2], 0))[0] == emel.Status.CAPACITY
    assert probe(emel, serialized_tensor_fixture(28, [2 ** 64 - 1], 0))[0] == emel.Status.CAPACITY
    assert probe(emel, serialized_tensor_fixture(41, [255, 8], 0))[0] == emel.Status.MODEL_INVALID


def test_truncated_and_inconsistent_tensor_records(emel):
    assert probe(emel, serialized_tensor_fixture(0, [1, 2, 3, 4, 5], 0))[0] == emel.Status.MODEL_INVALID
    truncated = serialized_tensor_fixture(0, [1, 2], 0)[:24 + 8 + 4 + 8]
    assert probe(emel, truncated)[0] == emel.Status.PARSE_FAILED
    wrong = bytearray(serialized_tensor_fixture(0, [4], 4))
    wrong[54:62] = u64(32)  # header 24, name 14, dimension count 4, dimension 8, type 4
    assert probe(emel, bytes(wrong))[0] == emel.Status.PARSE_FAILED
    assert probe(emel, serialized_tensor_fixture(0, [4], 0))[0] == emel.Status.PARSE_FAILED  # missing payload


def test_duplicates_and_malformed_metadata(emel):
    dup_tensor = b"GGUF" + u32(3) + u64(2) + u64(0)
    for offset in (0, 32):
        dup_tensor += gw.string(b"weight") + u32(1) + u64(4) + u32(0) + u64(offset)
    dup_tensor = gw.pad_to(dup_tensor, 32) + b"\0" * 64
    assert probe(emel, dup_tensor)[0] == emel.Status.MODEL_INVALID
    dup_key = b"GGUF" + u32(3) + u64(0) + u64(2) + gw.kv(b"a", GGUF_U8, b"\1") + gw.kv(b"a", GGUF_U8, b"\2")
    assert probe(emel, dup_key)[0] == emel.Status.MODEL_INVALID
    empty_key = b"GGUF" + u32(3) + u64(0) + u64(1) + gw.kv(b"", GGUF_U8, b"\1")
    assert probe(emel, empty_key)[0] == emel.Status.MODEL_INVALID
    unknown_type = b"GGUF" + u32(3) + u64(0) + u64(1) + gw.kv(b"unknown", 13, b"")
    assert probe(emel, unknown_type)[0] == emel.Status.MODEL_INVALID
    nested = b"GGUF" + u32(3) + u64(0) + u64(1) + gw.kv(b"n", GGUF_ARRAY, gw.array(GGUF_ARRAY, 0, b""))
    assert probe(emel, nested)[0] == emel.Status.MODEL_INVALID
    short_value = b"GGUF" + u32(3) + u64(0) + u64(1) + gw.kv(b"w", GGUF_U64, b"\1\2")
    assert probe(emel, short_value)[0] == emel.Status.PARSE_FAILED


def test_parse_needs_the_probed_capacity(emel):
    data = parser_fixture()
    st, req = probe(emel, data)
    assert st == emel.Status.OK
    buf = ctypes.create_string_buffer(data, len(data))
    recs = (emel.CGgufTensorInfo * 1)()
    assert emel.lib().emel_gguf_parse(buf, len(data), ctypes.byref(req), recs, 0) == int(emel.Status.CAPACITY)
    req.tensor_count = 2  # not the image that was probed
    recs2 = (emel.CGgufTensorInfo * 2)()
    assert emel.lib().emel_gguf_parse(buf, len(data), ctypes.byref(req), recs2, 2) == int(emel.Status.INVALID_REQUEST)


def test_written_model_views(emel):
    """A model image from the writer: F32 and F16 tables and Q8_0 / Q4_K
    matrices; each record's view is the one the device kernels consume."""
    q8 = bytes(range(256)) * (34 * 2 * 3 // 256 + 1)
    tensors = [(b"tok_embd.weight", [64, 10], 0, bytes(64 * 10 * 4)),
               (b"norm.weight", [64], 1, bytes(64 * 2)),
               (b"output.weight", [64, 3], 8, q8[:34 * 2 * 3]),
               (b"ffn.weight", [512, 5], 12, bytes(144 * 2 * 5))]
    img = emel.GgufImage(gw.image(tensors, metadata=[(b"general.name", GGUF_STRING, gw.string(b"synthetic"))],
                                  alignment=32))
    assert [n for n, _ in img.tensors] == ["tok_embd.weight", "norm.weight", "output.weight", "ffn.weight"]
    want = {"tok_embd.weight": (0, [64, 10, 1, 1], [4, 256, 2560, 2560]),
            "norm.weight": (1, [64, 1, 1, 1], [2, 128, 128, 128]),
            "output.weight": (8, [64, 3, 1, 1], [1, 68, 204, 204]),
            "ffn.weight": (12, [512, 5, 1, 1], [1, 288, 1440, 1440])}
    for name, t in img.tensors:
        v = emel.CView()
        assert emel.lib().emel_gguf_tensor_view(ctypes.byref(t), ctypes.c_void_p(0x10000), t.data_size,
                                                ctypes.byref(v)) == 0
        dtype, ne, nb = want[name]
        assert (v.dtype, list(v.ne), list(v.nb)) == (dtype, ne, nb), name
        assert img.image[t.file_offset:t.file_offset + t.data_size] == dict((n.decode(), p) for n, _, _, p in tensors)[name]
    # a type with no device kernel
    other = emel.GgufImage(gw.image([(b"q5k", [256, 2], 13, bytes(176 * 2))]))
    v = emel.CView()
    st = emel.lib().emel_gguf_tensor_view(ctypes.byref(other.tensors[0][1]), ctypes.c_void_p(0x10000), 1 << 20,
                                          ctypes.byref(v))
    assert st == int(emel.Status.UNSUPPORTED_OPERATION)
