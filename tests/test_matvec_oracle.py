"""The vocabulary matvec + argmax oracle (oracle_mul_mat_argmax, restating
matmul.rs OpMulMatArgmax) on the reference's tests
(tests/any/matmul_ops.rs:1092-1178, read as known answers) and on the scan
rules: first row on ties, a NaN at row 0 pins the answer."""

import ctypes

import numpy as np
import pytest

import oracle

B = ctypes.byref


@pytest.fixture(scope="module")
def lib():
    return oracle.load()


def nb_of(ne):
    nb = [4]
    for d in range(1, 4):
        nb.append(nb[-1] * ne[d - 1])
    return nb


def run(lib, lhs, lne, rhs, rne, dne=(1, 1, 1, 1), rnb=None, fill=9.0):
    lhs, rhs = np.asarray(lhs, np.float32), np.asarray(rhs, np.float32)
    out = np.full(int(np.prod(dne)), fill, np.float32)
    idx = ctypes.c_int32(-7)
    st = lib.oracle_mul_mat_argmax(B(oracle.make_view(lhs.ctypes.data, lhs.nbytes, list(lne), nb_of(lne), 0)),
                                   B(oracle.make_view(rhs.ctypes.data, rhs.nbytes, list(rne), rnb or nb_of(rne), 0)),
                                   B(oracle.make_view(out.ctypes.data, out.nbytes, list(dne), nb_of(dne), 0)), B(idx))
    return st, out, idx.value


def test_returns_index_and_writes_best_score(lib):
    st, out, idx = run(lib, [1, 2, 3, 4, 5, 6], [3, 2, 1, 1], [1, 1, 1], [1, 3, 1, 1])
    assert st == 0 and idx == 1 and out.tolist() == [15.0]


def test_rejects_invalid_shapes_without_writing(lib):
    st, out, _ = run(lib, [1] * 6, [3, 2, 1, 1], [1, 1], [1, 2, 1, 1])
    assert st == 2 and out.tolist() == [9.0]
    st, out, _ = run(lib, [1] * 6, [3, 2, 1, 1], [1, 1, 1], [3, 1, 1, 1])  # the legacy [k] rhs
    assert st == 2 and out.tolist() == [9.0]


def test_rejects_strided_rhs_view(lib):
    st, out, _ = run(lib, [1] * 6, [3, 2, 1, 1], [1] * 5, [1, 3, 1, 1], rnb=[4, 8, 24, 24])
    assert st == 1 and out.tolist() == [9.0]


def test_scan_rules(lib):
    k = 4
    rows = np.array([[1, 1, 1, 1], [2, 0, 0, 0], [0, 4, 0, 0], [3, 1, 0, 0]], np.float32)  # scores 4, 2, 4, 4
    st, out, idx = run(lib, rows.ravel(), [k, 4, 1, 1], np.ones(k), [1, k, 1, 1])
    assert st == 0 and idx == 0 and out[0] == 4.0
    rows[0, 0] = np.nan  # row 0 NaN: pinned
    st, out, idx = run(lib, rows.ravel(), [k, 4, 1, 1], np.ones(k), [1, k, 1, 1])
    assert st == 0 and idx == 0 and np.isnan(out[0])
    rows[0, 0] = -np.inf  # row 0 -inf, a NaN row never wins
    rows[1, 1] = np.nan
    st, out, idx = run(lib, rows.ravel(), [k, 4, 1, 1], np.ones(k), [1, k, 1, 1])
    assert st == 0 and idx == 2 and out[0] == 4.0


def test_sequential_binary32_order(lib):
    """The score is the left-to-right binary32 sum: 1e8 + 1 - 1e8 == 0."""
    st, out, idx = run(lib, [1e8, 1, -1e8, 0.5, 0.25, 0], [3, 2, 1, 1], [1, 1, 1], [1, 3, 1, 1])
    assert st == 0 and out[0] == 0.75 and idx == 1


# ---- Q8_0 rows (matmul.rs OpMulMatArgmaxQ8_0) ---------------------------------

def q8_layout(k, rows):
    rb = k // 32 * 34
    return [k, rows, 1, 1], [1, rb, rb * rows, rb * rows]


def run_q8(lib, lhs_bytes, k, rows, rhs, fill=9.0, rne=None, rnb=None, code=8):
    lhs = np.frombuffer(bytes(lhs_bytes), np.uint8).copy()
    rhs = np.asarray(rhs, np.float32)
    out = np.full(1, fill, np.float32)
    idx = ctypes.c_int32(-7)
    lne, lnb = q8_layout(k, rows)
    rne = rne or [1, k, 1, 1]
    st = lib.oracle_mul_mat_argmax_q8_0(B(oracle.make_view(lhs.ctypes.data, lhs.nbytes, lne, lnb, code)),
                                        B(oracle.make_view(rhs.ctypes.data, rhs.nbytes, rne, rnb or nb_of(rne), 0)),
                                        B(oracle.make_view(out.ctypes.data, out.nbytes, [1, 1, 1, 1], nb_of([1, 1, 1, 1]), 0)),
                                        B(idx))
    return st, out, idx.value


def q8_constant_block(encoded):
    # tests/any/matmul_ops.rs:76-82: scale 1.0 (0x3C00), every quant `encoded`
    return bytes([0x00, 0x3C]) + bytes([encoded & 0xFF]) * 32


def test_q8_0_reference_golden_vector(lib):
    # snapshots/parity/kernel-argmax-parity/manifest.txt case=q8_0_success:
    # index=1 output_bits=437ffc00, inputs from
    # tools/emel-kernel-argmax-parity/src/main.rs:61-71 and 114-127
    # (16 blocks of scale 1.0, blocks 8..15 with every quant 1; rhs 256 ones)
    lhs = bytearray(544)
    for b in range(16):
        lhs[b * 34:b * 34 + 2] = bytes([0x00, 0x3C])
        if b >= 8:
            lhs[b * 34 + 2:b * 34 + 34] = bytes([1]) * 32
    st, out, idx = run_q8(lib, lhs, 256, 2, np.ones(256), fill=np.float32(np.uint32(0x7FC01234).view(np.float32)))
    assert st == 0 and idx == 1 and int(out.view(np.uint32)[0]) == 0x437FFC00


def test_q8_0_known_answers(lib):
    # tests/any/matmul_ops.rs:1266-1308: rows of constant quants 1 and 2
    st, out, idx = run_q8(lib, q8_constant_block(1) + q8_constant_block(2), 32, 2, np.ones(32))
    assert st == 0 and idx == 1 and out[0] > 0
    # first row on ties
    st, out, idx = run_q8(lib, q8_constant_block(3) + q8_constant_block(3), 32, 2, np.ones(32))
    assert st == 0 and idx == 0


def test_q8_0_guards(lib):
    blk = q8_constant_block(1) * 2
    assert run_q8(lib, blk, 32, 2, np.ones(31), rne=[1, 31, 1, 1])[0] == 2       # rhs length differs
    assert run_q8(lib, blk, 32, 2, np.ones(32), code=2)[0] == 1                  # not a Q8_0 view
    assert run_q8(lib, blk, 32, 2, np.ones(64), rne=[1, 32, 1, 1], rnb=[8, 8, 256, 256])[0] == 1  # rhs not dense
    big = q8_constant_block(1) * 1025                                             # 1025 blocks > 1024
    assert run_q8(lib, big, 32 * 1025, 1, np.ones(32 * 1025))[0] == 1


def test_q8_0_matches_float_scores(lib):
    # the quantized score tracks the float score: argmax of a planted row
    rng = np.random.default_rng(4)
    k, rows = 256, 40
    w = rng.standard_normal((rows, k)).astype(np.float32) * 0.05
    w[17] = np.abs(w[17]) + 0.05
    x = np.abs(rng.standard_normal(k)).astype(np.float32)
    blob = bytearray()
    for r in range(rows):
        for b in range(k // 32):
            blk = w[r, b * 32:(b + 1) * 32]
            d = np.float16(np.max(np.abs(blk)) / 127.0)
            q = np.clip(np.round(blk / np.float32(d)), -127, 127).astype(np.int8)
            blob += d.tobytes() + q.tobytes()
    st, out, idx = run_q8(lib, blob, k, rows, x)
    assert st == 0 and idx == 17


# ---- Q4_0 / Q4_1 / Q5_0 rows (matmul.rs OpMulMatArgmaxQ4_0 / Q4_1 / Q5_0) -------

BLOCK_BYTES = {2: 18, 3: 20, 6: 22, 8: 34}
ORACLE_FN = {2: "oracle_mul_mat_argmax_q4_0", 3: "oracle_mul_mat_argmax_q4_1", 6: "oracle_mul_mat_argmax_q5_0",
             8: "oracle_mul_mat_argmax_q8_0"}


def run_packed(lib, code, lhs_bytes, k, rows, rhs, fill=9.0):
    lhs = np.frombuffer(bytes(lhs_bytes), np.uint8).copy()
    rhs = np.asarray(rhs, np.float32)
    out = np.full(1, fill, np.float32)
    idx = ctypes.c_int32(-7)
    rb = k // 32 * BLOCK_BYTES[code]
    st = getattr(lib, ORACLE_FN[code])(
        B(oracle.make_view(lhs.ctypes.data, lhs.nbytes, [k, rows, 1, 1], [1, rb, rb * rows, rb * rows], code)),
        B(oracle.make_view(rhs.ctypes.data, rhs.nbytes, [1, k, 1, 1], nb_of([1, k, 1, 1]), 0)),
        B(oracle.make_view(out.ctypes.data, out.nbytes, [1, 1, 1, 1], nb_of([1, 1, 1, 1]), 0)), B(idx))
    return st, out, idx.value


def test_q5_0_reference_golden_vector(lib):
    # snapshots/parity/kernel-argmax-parity/manifest.txt case=q5_0_success:
    # index=1 output_bits=44effc40; inputs from
    # tools/emel-kernel-argmax-parity/src/main.rs:49-59 and 114-127
    lhs = bytearray(352)
    for b in range(16):
        lhs[b * 22:b * 22 + 2] = bytes([0x00, 0x3C])
        if b >= 8:
            lhs[b * 22 + 2:b * 22 + 6] = bytes([0xFF]) * 4
            lhs[b * 22 + 6:b * 22 + 22] = bytes([0x0F]) * 16
    st, out, idx = run_packed(lib, 6, lhs, 256, 2, np.ones(256))
    assert st == 0 and idx == 1 and int(out.view(np.uint32)[0]) == 0x44EFFC40


def nibble_block(code, encoded):
    # tests/any/matmul_ops.rs:49-74: scale 1.0, every nibble `encoded`
    byte = bytes([encoded | (encoded << 4)])
    if code == 2:
        return bytes([0x00, 0x3C]) + byte * 16
    if code == 3:
        return bytes([0x00, 0x3C, 0x00, 0x00]) + byte * 16
    return bytes([0x00, 0x3C]) + bytes([0xFF]) * 4 + byte * 16


def test_q4_q5_known_answers(lib):
    # matmul_ops.rs:1266-1340: the second row wins, with a positive score
    for code, (a, b) in ((2, (0x09, 0x0A)), (3, (1, 2)), (6, (0x01, 0x02))):
        st, out, idx = run_packed(lib, code, nibble_block(code, a) + nibble_block(code, b), 32, 2, np.ones(32))
        assert st == 0 and idx == 1 and out[0] > 0, code
    # matmul_ops.rs:1342-1360: a Q4_1 row stride that is not 20 bytes is rejected
    lhs = np.zeros(21, np.uint8)
    rhs = np.ones(32, np.float32)
    out = np.full(1, 9.0, np.float32)
    idx = ctypes.c_int32()
    st = lib.oracle_mul_mat_argmax_q4_1(B(oracle.make_view(lhs.ctypes.data, 21, [32, 1, 1, 1], [1, 21, 21, 21], 3)),
                                        B(oracle.make_view(rhs.ctypes.data, 128, [1, 32, 1, 1], nb_of([1, 32, 1, 1]), 0)),
                                        B(oracle.make_view(out.ctypes.data, 4, [1, 1, 1, 1], nb_of([1, 1, 1, 1]), 0)),
                                        B(idx))
    assert st == 1 and out[0] == 9.0


def test_q4_q5_decoding_matches_float_dot(lib):
    # a row's score equals the float dot of its decoded weights with the
    # quantized rhs (all terms exact here: integer scales, one block)
    rng = np.random.default_rng(21)
    x = rng.integers(-127, 128, 32).astype(np.float32)
    x[0] = 127.0  # amax 127: rhs scale 1, quants equal x
    for code in (2, 3, 6):
        nib = rng.integers(0, 16, 32)
        hb = rng.integers(0, 2, 32)
        if code == 2:
            w = nib - 8
            blk = bytes([0x00, 0x3C]) + bytes(int(nib[i] | (nib[i + 16] << 4)) for i in range(16))
        elif code == 3:
            w = nib + 2.0  # min 2.0 (0x4000)
            blk = bytes([0x00, 0x3C, 0x00, 0x40]) + bytes(int(nib[i] | (nib[i + 16] << 4)) for i in range(16))
        else:
            w = (nib | (hb << 4)) - 16
            high = sum(int(hb[i]) << i for i in range(32))
            blk = bytes([0x00, 0x3C]) + high.to_bytes(4, "little") + bytes(int(nib[i] | (nib[i + 16] << 4))
                                                                            for i in range(16))
        st, out, idx = run_packed(lib, code, blk, 32, 1, x)
        assert st == 0 and out[0] == np.float32(np.dot(w.astype(np.float64), x.astype(np.float64))), code


# ---- K-quant rows (matmul.rs OpMulMatArgmaxQ4K / Q6K) -------------------------

K_BYTES = {10: 84, 11: 110, 12: 144, 14: 210}
K_FN = {10: "oracle_mul_mat_argmax_q2_k", 11: "oracle_mul_mat_argmax_q3_k", 12: "oracle_mul_mat_argmax_q4_k",
        14: "oracle_mul_mat_argmax_q6_k"}


def run_k(lib, code, lhs_bytes, k, rows, rhs):
    lhs = np.frombuffer(bytes(lhs_bytes), np.uint8).copy()
    rhs = np.asarray(rhs, np.float32)
    out = np.full(1, np.float32(np.uint32(0x7FC01234).view(np.float32)), np.float32)
    idx = ctypes.c_int32(-7)
    rb = k // 256 * K_BYTES[code]
    st = getattr(lib, K_FN[code])(
        B(oracle.make_view(lhs.ctypes.data, lhs.nbytes, [k, rows, 1, 1], [1, rb, rb * rows, rb * rows], code)),
        B(oracle.make_view(rhs.ctypes.data, rhs.nbytes, [1, k, 1, 1], nb_of([1, k, 1, 1]), 0)),
        B(oracle.make_view(out.ctypes.data, out.nbytes, [1, 1, 1, 1], nb_of([1, 1, 1, 1]), 0)), B(idx))
    return st, out, idx.value


def test_k_quant_reference_golden_vectors(lib):
    # snapshots/parity/kernel-argmax-parity/manifest.txt: q4_k_success index=1
    # bits 45700000, q6_k_success index=1 bits 45f80000; inputs from
    # tools/emel-kernel-argmax-parity/src/main.rs:82-98 and 114-127
    q4 = bytearray(288)
    q4[144:146] = bytes([0x00, 0x3C])
    q4[148:160] = bytes([1]) * 12
    q4[160:] = bytes([0xFF]) * 128
    st, out, idx = run_k(lib, 12, q4, 256, 2, np.ones(256))
    assert st == 0 and idx == 1 and int(out.view(np.uint32)[0]) == 0x45700000
    q6 = bytearray(420)
    q6[210:338] = bytes([0xFF]) * 128
    q6[338:402] = bytes([0xFF]) * 64
    q6[402:418] = bytes([1]) * 16
    q6[418:420] = bytes([0x00, 0x3C])
    st, out, idx = run_k(lib, 14, q6, 256, 2, np.ones(256))
    assert st == 0 and idx == 1 and int(out.view(np.uint32)[0]) == 0x45F80000


def test_k_quant_guards(lib):
    blk = bytes(144)
    assert run_k(lib, 12, blk, 256, 1, np.ones(255))[0] in (1, 2)
    assert run_k(lib, 12, blk * 129, 256 * 129, 1, np.ones(256 * 129))[0] == 1   # 129 blocks > 128


def test_q2_k_q3_k_reference_golden_vectors(lib):
    # kernel-argmax-parity manifest: q2_k_success index=1 bits 46340000,
    # q3_k_success index=0 bits 00000000; inputs from
    # tools/emel-kernel-argmax-parity/src/main.rs:73-89 and 114-127
    q2 = bytearray(168)
    q2[84 + 80:84 + 82] = bytes([0x00, 0x3C])
    q2[84:84 + 16] = bytes([0xFF]) * 16
    q2[84 + 16:84 + 80] = bytes([0xFF]) * 64
    st, out, idx = run_k(lib, 10, q2, 256, 2, np.ones(256))
    assert st == 0 and idx == 1 and int(out.view(np.uint32)[0]) == 0x46340000
    q3 = bytearray(220)
    q3[110:142] = bytes([0xFF]) * 32
    q3[142:206] = bytes([0xFF]) * 64
    q3[206:218] = bytes([0x21]) * 12
    q3[218:220] = bytes([0x00, 0x3C])
    st, out, idx = run_k(lib, 11, q3, 256, 2, np.ones(256))
    assert st == 0 and idx == 0 and int(out.view(np.uint32)[0]) == 0x00000000
