"""The shape-copy oracle (oracle_cpy / oracle_cont, restating shape.rs) on
the reference's own shape tests (tests/any/shape_ops.rs:17-42, 85-104,
140-165, read as known answers)."""

import ctypes

import numpy as np
import pytest

import oracle

B = ctypes.byref


@pytest.fixture(scope="module")
def lib():
    return oracle.load()


def view(arr, ne, nb):
    return oracle.make_view(arr.ctypes.data, arr.nbytes, ne, nb, 0)


DENSE_2x2 = ([2, 2, 1, 1], [4, 8, 16, 16])
STRIDED_2x2 = ([2, 2, 1, 1], [8, 16, 32, 64])


def test_cpy_and_cont_materialize_strided_source(lib):
    source = np.array([1, 99, 2, 99, 3, 99, 4], np.float32)
    copied = np.zeros(7, np.float32)
    assert lib.oracle_cpy(B(view(source, *STRIDED_2x2)), B(view(copied, *STRIDED_2x2))) == 0
    assert copied.tolist() == [1, 0, 2, 0, 3, 0, 4]
    materialized = np.zeros(4, np.float32)
    assert lib.oracle_cont(B(view(source, *STRIDED_2x2)), B(view(materialized, *DENSE_2x2))) == 0
    assert materialized.tolist() == [1, 2, 3, 4]


def test_cont_into_strided_destination_is_invalid_layout(lib):
    source = np.array([1, 2, 3, 4], np.float32)
    output = np.full(7, 7.0, np.float32)
    assert lib.oracle_cont(B(view(source, *DENSE_2x2)), B(view(output, *STRIDED_2x2))) == 8
    assert np.all(output == 7.0)


def test_copy_and_cont_shape_mismatch(lib):
    source = np.ones(4, np.float32)
    dest = np.full(3, 9.0, np.float32)
    for fn in (lib.oracle_cpy, lib.oracle_cont):
        assert fn(B(view(source, [4, 1, 1, 1], [4, 16, 16, 16])), B(view(dest, [3, 1, 1, 1], [4, 12, 12, 12]))) == 2
        assert np.all(dest == 9.0)


def test_implicit_destination_strides_copy_but_are_not_dense_for_cont(lib):
    """nb[0] == 0 is the implicit contiguous form: OpCpy resolves it, while
    Layout::is_dense_contiguous compares the stored strides (InvalidLayout)."""
    source = np.arange(6, dtype=np.float32)
    out = np.zeros(6, np.float32)
    assert lib.oracle_cpy(B(view(source, [3, 2, 1, 1], [4, 12, 24, 24])), B(view(out, [6, 1, 1, 1], [0, 0, 0, 0]))) == 0
    assert out.tolist() == source.tolist()
    out[:] = 5
    assert lib.oracle_cont(B(view(source, [3, 2, 1, 1], [4, 12, 24, 24])), B(view(out, [6, 1, 1, 1], [0, 0, 0, 0]))) == 8
    assert np.all(out == 5)


def test_transposed_source_reshaped_destination(lib):
    """A [3, 4] transposed view of [4, 3] storage copied by ordinal into a
    [2, 6] dense destination."""
    base = np.arange(12, dtype=np.float32)  # storage rows of 3
    out = np.zeros(12, np.float32)
    src = view(base, [4, 3, 1, 1], [12, 4, 48, 48])  # element (i0, i1) = base[i0 * 3 + i1]
    assert lib.oracle_cont(B(src), B(view(out, [2, 6, 1, 1], [4, 8, 48, 48]))) == 0
    want = [base[i0 * 3 + i1] for i1 in range(3) for i0 in range(4)]
    assert out.tolist() == want
