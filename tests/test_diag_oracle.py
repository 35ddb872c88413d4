"""The diagonal-family oracle (oracle_diag / oracle_diag_mask, restating
diag.rs OpDiag / OpDiagMaskInf / OpDiagMaskZero) on the reference's own unit
tests (diag.rs:393-466, read as known answers) and on its shape guards."""

import ctypes

import numpy as np
import pytest

import oracle


@pytest.fixture(scope="module")
def lib():
    return oracle.load()


def diag(lib, inp, out_len, fill=9.0):
    inp = np.asarray(inp, np.float32)
    out = np.full(max(out_len, 1), fill, np.float32)
    st = lib.oracle_diag(inp.ctypes.data, inp.size, out.ctypes.data, out_len)
    return st, out


def mask(lib, mode, inp, out_len, n_past, fill=9.0):
    inp = np.asarray(inp, np.float32)
    out = np.full(max(out_len, 1), fill, np.float32)
    st = lib.oracle_diag_mask(mode, inp.ctypes.data, inp.size, out.ctypes.data, out_len, n_past)
    return st, out


def test_diag_writes_the_main_diagonal(lib):
    # diag.rs:397-409
    st, out = diag(lib, [1.0, 2.0], 4)
    assert st == 0 and out.view(np.uint32).tolist() == np.array([1, 0, 0, 2], np.float32).view(np.uint32).tolist()


def test_mask_inf_above_the_causal_diagonal(lib):
    # diag.rs:411-422
    st, out = mask(lib, 0, [1.0, 2.0, 3.0, 4.0], 4, 0)
    assert st == 0 and out[0] == 1.0 and np.isneginf(out[1]) and out[2] == 3.0 and out[3] == 4.0


def test_invalid_diag_does_not_mutate(lib):
    # diag.rs:424-435
    st, out = diag(lib, [1.0, 2.0], 3, fill=7.0)
    assert st == 6 and out.tolist() == [7.0, 7.0, 7.0]


def test_mask_zero_rejects_negative_n_past(lib):
    # diag.rs:437-447
    st, out = mask(lib, 1, [1.0, 2.0, 3.0, 4.0], 4, -1, fill=8.0)
    assert st == 6 and out.tolist() == [8.0] * 4


def test_mask_zero_writes_positive_zero_and_keeps_bits(lib):
    # diag.rs:449-466 (zero mask), NaN payloads and n_past wider than the side
    side = 5
    x = np.arange(side * side, dtype=np.float32) - 7.0
    x[6] = np.float32(-0.0)
    x.view(np.uint32)[12] = 0x7FA00001
    st, out = mask(lib, 1, x, side * side, 1)
    assert st == 0
    for r in range(side):
        for c in range(side):
            i = r * side + c
            want = np.float32(0.0) if c > r + 1 else x[i]
            assert out.view(np.uint32)[i] == np.array([want], np.float32).view(np.uint32)[0]
    st, out = mask(lib, 0, x, side * side, 100)
    assert st == 0 and out.view(np.uint32).tolist() == x.view(np.uint32).tolist()


def test_shape_guards(lib):
    assert mask(lib, 0, [1.0, 2.0, 3.0], 3, 0)[0] == 6        # not a perfect square
    assert mask(lib, 0, [1.0] * 4, 9, 0)[0] == 6              # lengths differ
    assert mask(lib, 0, [], 0, 0)[0] == 6                     # empty
    assert diag(lib, [], 0)[0] == 6
    assert diag(lib, [1.0, 2.0, 3.0], 9)[0] == 0


def softmax_causal(lib, x, side, n_past):
    x = np.asarray(x, np.float32)
    out = np.full(side * side, 7.0, np.float32)
    scratch = np.zeros(side * side, np.float32)
    st = lib.oracle_soft_max_diag_mask_inf(x.ctypes.data, x.size, out.ctypes.data, out.size, n_past,
                                           scratch.ctypes.data)
    return st, out


def test_softmax_after_causal_mask(lib):
    # the two reference events in sequence: row 0 keeps one column, row 1 both
    st, out = softmax_causal(lib, [1.0, 2.0, 3.0, 4.0], 2, 0)
    assert st == 0
    e = np.exp(np.float64(3.0) - 4.0)
    assert out[0] == 1.0 and out[1] == 0.0
    assert abs(out[2] - e / (1 + e)) < 1e-7 and abs(out[3] - 1 / (1 + e)) < 1e-7
    # n_past beyond the side: plain soft_max rows
    st, out = softmax_causal(lib, [1.0, 2.0, 3.0, 4.0], 2, 5)
    assert st == 0 and abs(out[0] + out[1] - 1.0) < 1e-7 and out[1] > out[0]
    # the mask's guards
    assert softmax_causal(lib, [1.0, 2.0, 3.0], 2, 0)[0] == 6
    assert softmax_causal(lib, [1.0] * 4, 2, -1)[0] == 6
