"""The get_rows oracle (oracle_get_rows, restating get_rows.rs and the
quant.rs / quant_more.rs block decoders) pinned on the reference's own
tests (tests/any/get_rows_ops.rs:395-440, 628-742, read as known answers),
plus its guard order: InvalidView, ShapeMismatch, UnsupportedSourceStride,
IndexOutOfBounds -- a rejected request writes nothing."""

import ctypes

import numpy as np
import pytest

import oracle

B = ctypes.byref
F32, F16, I32, Q4_0, Q8_0, Q4_K, BF16 = 0, 1, 26, 2, 8, 12, 30
INVALID_VIEW, SHAPE_MISMATCH, INDEX_OOB, UNSUPPORTED_STRIDE = 1, 2, 9, 10


@pytest.fixture(scope="module")
def lib():
    return oracle.load()


def contiguous_nb(ne, size=4):
    nb = [size]
    for d in range(1, 4):
        nb.append(nb[-1] * ne[d - 1])
    return nb


def v(arr, ne, nb, code):
    return oracle.make_view(arr.ctypes.data, arr.nbytes, ne, nb, code)


def idx_view(indices, ne3):
    a = np.asarray(indices, np.int32)
    ne = list(ne3) + [1]
    return a, v(a, ne, contiguous_nb(ne), I32)


def gather(lib, src, src_ne, src_nb, code, indices, idx_ne, out_len, dst_ne=None, fill=0.0):
    ia, iv = idx_view(indices, idx_ne)
    out = np.full(out_len, fill, np.float32)
    dst_ne = dst_ne or [src_ne[0]] + list(idx_ne)
    st = lib.oracle_get_rows(B(v(src, src_ne, src_nb, code)), B(iv), B(v(out, dst_ne, contiguous_nb(dst_ne), F32)))
    return st, out


def packed(cols, rows, bv, bb, code, outer=(1, 1)):
    row = cols // bv * bb
    return [cols, rows, outer[0], outer[1]], [1, row, row * rows, row * rows * outer[0]]


def q4_0_block(scale, packed_byte):
    return np.frombuffer(np.uint16(scale).tobytes() + bytes([packed_byte]) * 16, np.uint8)


def q8_0_block(scale, value):
    return np.frombuffer(np.uint16(scale).tobytes() + np.int8(value).tobytes() * 32, np.uint8)


def q4_k_block(scale, minimum, packed_byte, scales=(1, 1, 1, 1, 1, 1, 1, 1, 0x11, 0x11, 0x11, 0x11)):
    return np.frombuffer(np.uint16(scale).tobytes() + np.uint16(minimum).tobytes() + bytes(scales) +
                         bytes([packed_byte]) * 128, np.uint8)


def test_f32_row_and_batch_order(lib):
    src = np.array([1, 2, 3, 4, 5, 6, 10, 20, 30, 40, 50, 60], np.float32)
    st, out = gather(lib, src, [3, 2, 2, 1], contiguous_nb([3, 2, 2, 1]), F32, [1, 0, 0, 1], [2, 2, 1], 12)
    assert st == 0
    assert out.tolist() == [4, 5, 6, 1, 2, 3, 10, 20, 30, 40, 50, 60]


def test_f32_strided_source_rows(lib):
    src = np.array([1, 2, 99, 3, 4], np.float32)
    st, out = gather(lib, src, [2, 2, 1, 1], [4, 12, 24, 24], F32, [1, 0], [2, 1, 1], 4)
    assert st == 0 and out.tolist() == [3, 4, 1, 2]


def test_q4_0_dequantized_row_order(lib):
    src = np.concatenate([q4_0_block(0x3c00, 0x98), q4_0_block(0x3c00, 0xa7)])
    ne, nb = packed(32, 2, 32, 18, Q4_0)
    st, out = gather(lib, src, ne, nb, Q4_0, [1, 0], [2, 1, 1], 64)
    assert st == 0
    assert out[:16].tolist() == [-1.0] * 16 and out[16:32].tolist() == [2.0] * 16
    assert out[32:48].tolist() == [0.0] * 16 and out[48:].tolist() == [1.0] * 16


def test_q8_0_dequantized_row_order(lib):
    src = np.concatenate([q8_0_block(0x3c00, -2), q8_0_block(0x3c00, 1)])
    ne, nb = packed(32, 2, 32, 34, Q8_0)
    st, out = gather(lib, src, ne, nb, Q8_0, [1, 0], [2, 1, 1], 64)
    assert st == 0 and out[:32].tolist() == [1.0] * 32 and out[32:].tolist() == [-2.0] * 32


def test_q4_k_dequantized_row_order(lib):
    src = np.concatenate([q4_k_block(0x3c00, 0x3800, 0x43), q4_k_block(0x3c00, 0x3800, 0x21)])
    ne, nb = packed(256, 2, 256, 144, Q4_K)
    st, out = gather(lib, src, ne, nb, Q4_K, [1, 0], [2, 1, 1], 512)
    assert st == 0
    for k in range(4):
        assert out[64 * k:64 * k + 32].tolist() == [0.5] * 32 and out[64 * k + 32:64 * k + 64].tolist() == [1.5] * 32
        o = 256 + 64 * k
        assert out[o:o + 32].tolist() == [2.5] * 32 and out[o + 32:o + 64].tolist() == [3.5] * 32


def test_q4_k_upper_scale_min_groups(lib):
    src = q4_k_block(0x3c00, 0x3800, 0x21, scales=(0x41, 0x82, 0xc3, 0x04, 0x45, 0x86, 0xc7, 0x08, 0x89, 0x9a, 0xab, 0xbc))
    ne, nb = packed(256, 1, 256, 144, Q4_K)
    st, out = gather(lib, src, ne, nb, Q4_K, [0], [1, 1, 1], 256)
    assert st == 0
    for g, (low, high) in enumerate([(-1.5, 1.0), (-0.5, 4.0), (13.0, 63.5), (30.0, 18.5)]):
        assert out[64 * g:64 * g + 32].tolist() == [low] * 32 and out[64 * g + 32:64 * g + 64].tolist() == [high] * 32


def test_f16_and_bf16_sources_convert_bits(lib):
    halves = np.array([0x3c00, 0x7c01, 0x0001, 0x8400, 0xfc00, 0x7e00], np.uint16)  # 1, sNaN, subnormal, -2^-14, -inf, qNaN
    st, out = gather(lib, halves, [3, 2, 1, 1], contiguous_nb([3, 2, 1, 1], 2), F16, [1, 0], [2, 1, 1], 6)
    assert st == 0
    assert out.view(np.uint32).tolist() == [0xb8800000, 0xff800000, 0x7fc00000, 0x3f800000, 0x7f802000, 0x33800000]
    st, out = gather(lib, halves, [3, 2, 1, 1], contiguous_nb([3, 2, 1, 1], 2), BF16, [0, 1], [2, 1, 1], 6)
    assert st == 0 and out.view(np.uint32).tolist() == [int(h) << 16 for h in halves]


def test_guard_order_and_no_mutation(lib):
    src = np.arange(12, dtype=np.float32)
    ne = [3, 4, 1, 1]
    nb = contiguous_nb(ne)
    # index out of range (negative and too large)
    for bad in ([0, -1], [0, 4]):
        st, out = gather(lib, src, ne, nb, F32, bad, [2, 1, 1], 6, fill=7.0)
        assert st == INDEX_OOB and np.all(out == 7.0)
    # destination extents that do not match [ne0, idx0, idx1, idx2]
    st, out = gather(lib, src, ne, nb, F32, [0, 1], [2, 1, 1], 6, dst_ne=[6, 1, 1, 1], fill=7.0)
    assert st == SHAPE_MISMATCH and np.all(out == 7.0)
    # an index view over too little storage
    ia = np.zeros(1, np.int32)
    out = np.full(6, 7.0, np.float32)
    st = lib.oracle_get_rows(B(v(src, ne, nb, F32)), B(v(ia, [2, 1, 1, 1], [4, 8, 8, 8], I32)),
                             B(v(out, [3, 2, 1, 1], contiguous_nb([3, 2, 1, 1]), F32)))
    assert st == INVALID_VIEW and np.all(out == 7.0)


def test_empty_indices_are_a_no_op(lib):
    src = np.arange(12, dtype=np.float32)
    ia = np.zeros(1, np.int32)
    out = np.full(4, 7.0, np.float32)
    st = lib.oracle_get_rows(B(v(src, [3, 4, 1, 1], contiguous_nb([3, 4, 1, 1]), F32)),
                             B(v(ia, [0, 1, 1, 1], [4, 4, 4, 4], I32)),
                             B(v(out, [3, 0, 1, 1], [4, 12, 0, 0], F32)))  # Layout::contiguous strides
    assert st == 0 and np.all(out == 7.0)


def f32_bytes_known_source(length):
    # tests/any/get_rows_ops.rs:440-479: rows at byte offsets 0 and 9
    src = np.zeros(length, np.uint8)
    src[0:8] = np.array([1.0, 2.0], np.float32).view(np.uint8)
    if length >= 17:
        src[9:17] = np.array([3.0, 4.0], np.float32).view(np.uint8)
    return src


def test_f32_bytes_reads_unaligned_outer_source_rows(lib):
    src = f32_bytes_known_source(17)
    idx, iv = idx_view([1, 0], [2, 1, 1])
    out = np.zeros(4, np.float32)
    st = lib.oracle_get_rows_f32_bytes(B(v(src, [2, 2, 1, 1], [4, 9, 18, 18], F32)), B(iv),
                                       B(v(out, [2, 2, 1, 1], contiguous_nb([2, 2, 1, 1]), F32)))
    assert st == 0 and out.tolist() == [3.0, 4.0, 1.0, 2.0]


def test_f32_bytes_rejects_short_unaligned_outer_storage(lib):
    src = np.zeros(16, np.uint8)
    idx, iv = idx_view([1, 0], [2, 1, 1])
    out = np.full(4, 9.0, np.float32)
    st = lib.oracle_get_rows_f32_bytes(B(v(src, [2, 2, 1, 1], [4, 9, 18, 18], F32)), B(iv),
                                       B(v(out, [2, 2, 1, 1], contiguous_nb([2, 2, 1, 1]), F32)))
    assert st == INVALID_VIEW and out.tolist() == [9.0] * 4


def test_f32_bytes_guard_order(lib):
    src = f32_bytes_known_source(17)
    out = np.full(4, 9.0, np.float32)
    ov = v(out, [2, 2, 1, 1], contiguous_nb([2, 2, 1, 1]), F32)
    idx, iv = idx_view([1, 0], [2, 1, 1])
    # nb[0] not a multiple of 4: InvalidView (no UnsupportedSourceStride variant on this path)
    assert lib.oracle_get_rows_f32_bytes(B(v(src, [2, 2, 1, 1], [2, 9, 18, 18], F32)), B(iv), B(ov)) == INVALID_VIEW
    # an F16 source: InvalidView
    assert lib.oracle_get_rows_f32_bytes(B(v(src, [2, 2, 1, 1], [4, 9, 18, 18], F16)), B(iv), B(ov)) == INVALID_VIEW
    # destination rows differ from the index count: ShapeMismatch
    bad_out = v(out, [2, 1, 1, 1], contiguous_nb([2, 1, 1, 1]), F32)
    assert lib.oracle_get_rows_f32_bytes(B(v(src, [2, 2, 1, 1], [4, 9, 18, 18], F32)), B(iv),
                                         B(bad_out)) == SHAPE_MISMATCH
    # an index past the rows: IndexOutOfBounds
    idx, iv = idx_view([2, 0], [2, 1, 1])
    assert lib.oracle_get_rows_f32_bytes(B(v(src, [2, 2, 1, 1], [4, 9, 18, 18], F32)), B(iv), B(ov)) == INDEX_OOB
    assert out.tolist() == [9.0] * 4
    # no indices: the metadata-only rules, nothing read
    idx, iv = idx_view(np.zeros(0), [0, 1, 1])
    empty = np.zeros(1, np.float32)
    assert lib.oracle_get_rows_f32_bytes(B(v(src, [2, 2, 1, 1], [4, 9, 18, 18], F32)), B(iv),
                                         B(v(empty, [2, 0, 1, 1], [4, 8, 0, 0], F32))) == 0


def test_f32_bytes_matches_the_aligned_gather_on_aligned_rows(lib):
    rng = np.random.default_rng(5)
    src = rng.standard_normal(64 * 10).astype(np.float32)
    idx, iv = idx_view(rng.integers(0, 10, 12), [12, 1, 1])
    a = np.zeros(64 * 12, np.float32)
    b = np.ones(64 * 12, np.float32)
    sv = v(src, [64, 10, 1, 1], contiguous_nb([64, 10, 1, 1]), F32)
    dn = [64, 12, 1, 1]
    assert lib.oracle_get_rows(B(sv), B(iv), B(v(a, dn, contiguous_nb(dn), F32))) == 0
    assert lib.oracle_get_rows_f32_bytes(B(sv), B(iv), B(v(b, dn, contiguous_nb(dn), F32))) == 0
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))
