"""The RoPE oracle (oracle_rope, restating rope.rs) on the reference's own
tests (tests/any/rope_ops.rs:84-247, read as known answers with their 1e-5
tolerance) and on the guard order view -> parameters -> mode / shape."""

import ctypes
import math

import numpy as np
import pytest

import oracle

B = ctypes.byref
F32, I32 = 0, 26
NORM, NEOX, TIMESTEP = 0, 2, 4


@pytest.fixture(scope="module")
def lib():
    return oracle.load()


def nb_of(ne):
    nb = [4]
    for d in range(1, 4):
        nb.append(nb[-1] * ne[d - 1])
    return nb


def params(mode, **kw):
    p = oracle.RopeParams(n_dims=4, mode=mode, freq_base=10000.0, freq_scale=1.0, ext_factor=0.0, attn_factor=1.0)
    for k, v in kw.items():
        setattr(p, k, v)
    return p


def rope(lib, src, ne, pos, p, src_nb=None, dst_ne=None, pos_code=I32, fill=0.0):
    src = np.asarray(src, np.float32)
    pos = np.asarray(pos, np.int32)
    dne = dst_ne or ne
    out = np.full(int(np.prod(dne)), fill, np.float32)
    sv = oracle.make_view(src.ctypes.data, src.nbytes, ne, src_nb or nb_of(ne), F32)
    pv = oracle.make_view(pos.ctypes.data, pos.nbytes, [pos.size, 1, 1, 1], nb_of([pos.size, 1, 1, 1]), pos_code)
    dv = oracle.make_view(out.ctypes.data, out.nbytes, dne, nb_of(dne), F32)
    return lib.oracle_rope(B(sv), B(pv), B(dv), B(p)), out


def expected_rotation(x, position, neox):
    out = list(x)
    theta_scale = np.float32(10000.0) ** np.float32(-2.0 / 4.0)
    theta = position
    for pair in range(2):
        c, s = math.cos(theta), math.sin(theta)
        a, b = (pair, pair + 2) if neox else (2 * pair, 2 * pair + 1)
        out[a] = x[a] * c - x[b] * s
        out[b] = x[a] * s + x[b] * c
        theta *= float(theta_scale)
    return out


def test_norm_pairing_copies_the_tail(lib):
    src = [1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12]
    st, out = rope(lib, src, [6, 1, 2, 1], [1, 2], params(NORM))
    assert st == 0
    want = expected_rotation(src[:6], 1.0, False) + expected_rotation(src[6:], 2.0, False)
    assert np.allclose(out, want, atol=1e-5, rtol=0)


def test_neox_split_half_pairing(lib):
    st, out = rope(lib, [1, 2, 3, 4], [4, 1, 1, 1], [1], params(NEOX))
    assert st == 0 and np.allclose(out, expected_rotation([1, 2, 3, 4], 1.0, True), atol=1e-5, rtol=0)


def test_timestep_split_real_and_imaginary(lib):
    src = [1.0, 2.0, 3.0, 4.0]
    st, out = rope(lib, src, [4, 1, 1, 1], [1], params(TIMESTEP))
    assert st == 0
    want = [0.0] * 4
    for pair in range(2):
        f = math.exp(-math.log(10000.0) * pair / 2)
        c, s = math.cos(f), math.sin(f)
        want[pair] = src[2 * pair] * c - src[2 * pair + 1] * s
        want[2 + pair] = src[2 * pair] * s + src[2 * pair + 1] * c
    assert np.allclose(out, want, atol=1e-5, rtol=0)


def test_guard_classification_writes_nothing(lib):
    src = [1, 2, 3, 4]
    st, out = rope(lib, src, [4, 1, 1, 1], [1], params(99), fill=9.0)
    assert st == 11 and np.all(out == 9.0)  # InvalidMode
    st, out = rope(lib, src, [4, 1, 1, 1], [1], params(NORM, freq_base=0.0), fill=9.0)
    assert st == 3 and np.all(out == 9.0)  # InvalidParameters
    st, out = rope(lib, src, [4, 1, 1, 1], [1], params(NORM), dst_ne=[2, 1, 1, 1], fill=9.0)
    assert st == 2 and np.all(out == 9.0)  # ShapeMismatch
    st, out = rope(lib, src, [4, 1, 1, 1], [1], params(NORM), pos_code=F32, fill=9.0)
    assert st == 1 and np.all(out == 9.0)  # InvalidView: F32 positions


def test_timestep_requires_dense_layout(lib):
    src = [1, 2, 3, 4, 99, 98, 97, 96]
    st, out = rope(lib, src, [4, 1, 1, 1], [1], params(TIMESTEP), src_nb=[8, 8, 32, 32], fill=9.0)
    assert st == 2 and np.all(out == 9.0)


@pytest.mark.parametrize("mode", [NORM, NEOX])
def test_rotation_against_binary64(lib, mode):
    """128 dims, 8 heads, 33 positions, half the dims rotated: within a few
    ulp of the same rotation in binary64 (theta chain kept in binary32)."""
    rng = np.random.default_rng(mode)
    cols, rows, npos, n_dims = 128, 8, 33, 64
    x = rng.standard_normal(cols * rows * npos).astype(np.float32)
    pos = rng.integers(0, 4096, size=npos).astype(np.int32)
    st, out = rope(lib, x, [cols, rows, npos, 1], pos, params(mode, n_dims=n_dims, freq_scale=0.5, attn_factor=1.25))
    assert st == 0
    x3 = x.reshape(npos, rows, cols).astype(np.float64)
    o3 = out.reshape(npos, rows, cols)
    half = n_dims // 2
    ts = np.float32(10000.0) ** np.float32(-2.0 / n_dims)
    for p in range(npos):
        theta = np.float32(pos[p])
        for k in range(half):
            ang = float(theta) * 0.5
            c, s = math.cos(ang) * 1.25, math.sin(ang) * 1.25
            a, b = (k, k + half) if mode == NEOX else (2 * k, 2 * k + 1)
            wa = x3[p, :, a] * c - x3[p, :, b] * s
            wb = x3[p, :, a] * s + x3[p, :, b] * c
            assert np.allclose(o3[p, :, a], wa, atol=2e-5, rtol=1e-5)
            assert np.allclose(o3[p, :, b], wb, atol=2e-5, rtol=1e-5)
            theta = np.float32(theta * ts)
        assert np.array_equal(o3[p, :, n_dims:].view(np.uint32), x.reshape(npos, rows, cols)[p, :, n_dims:].view(np.uint32))
