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
