"""The GLU oracle (oracle_glu, a restatement of glu.rs) pinned on the
reference's own unit tests (glu.rs:298-363, read as known answers) and on
the x86 semantics of f32::max / f32::min with a constant operand."""

import ctypes
import math

import numpy as np
import pytest

import oracle

REGLU, GEGLU, SWIGLU, SWIGLU_OAI, GEGLU_ERF, GEGLU_QUICK = range(6)


@pytest.fixture(scope="module")
def lib():
    return oracle.load()


def run(lib, subop, values, out_len=None, fill=9.0):
    x = np.asarray(values, np.float32)
    n = out_len if out_len is not None else x.size // 2
    out = np.full(max(n, 1), fill, np.float32)
    st = lib.oracle_glu(subop, x.ctypes.data, x.size, out.ctypes.data, n)
    return st, out


def bits(a):
    return np.asarray(a, np.float32).view(np.uint32)


def test_reglu_multiplies_relu_gate(lib):
    # glu.rs:302-313
    st, out = run(lib, REGLU, [1.0, -2.0, 3.0, 4.0])
    assert st == 0
    assert bits(out).tolist() == bits([3.0, -8.0]).tolist()


def test_odd_length_is_invalid_and_does_not_mutate(lib):
    # glu.rs:315-326
    st, out = run(lib, SWIGLU, [1.0, 2.0, 3.0], out_len=1)
    assert st == 6  # InvalidShape
    assert bits(out).tolist() == bits([9.0]).tolist()


@pytest.mark.parametrize("values,out_len", [([], 0), ([1.0, 2.0, 3.0, 4.0], 1), ([1.0, 2.0], 2)])
def test_split_length_rules(lib, values, out_len):
    # glu.rs:84-91: empty, output length != input / 2
    st, out = run(lib, REGLU, values, out_len=out_len)
    assert st == 6
    assert np.all(out == 9.0)


@pytest.mark.parametrize("subop", [GEGLU, SWIGLU, SWIGLU_OAI, GEGLU_ERF, GEGLU_QUICK])
def test_remaining_subops_write_finite_gated_products(lib, subop):
    # glu.rs:328-349: input [2, 1]
    st, out = run(lib, subop, [2.0, 1.0])
    assert st == 0 and math.isfinite(out[0]) and bits(out)[0] != bits([9.0])[0]


def test_public_kernel_dispatches_reglu(lib):
    # glu.rs:352-362
    st, out = run(lib, REGLU, [1.0, 2.0])
    assert st == 0 and bits(out).tolist() == bits([2.0]).tolist()


def test_formulas_against_binary64(lib):
    """Each subop close to the same formula in binary64 on ordinary inputs:
    absolute error within 4e-6 of |value| * max(1, |gate input|), the scale of
    the product (binary32 cancellation in 1 + tanh and 1 - poly * exp makes a
    relative bound meaningless near zero)."""
    rng = np.random.default_rng(7)
    n = 4096
    v = (rng.standard_normal(n) * 3).astype(np.float32)
    g = (rng.standard_normal(n) * 3).astype(np.float32)
    x = np.concatenate([v, g])
    vd, gd = v.astype(np.float64), g.astype(np.float64)
    silu = lambda t: t / (1 + np.exp(-t))
    erf = np.vectorize(math.erf)
    want = {
        REGLU: vd * np.maximum(gd, 0),
        GEGLU: vd * 0.5 * gd * (1 + np.tanh(0.7978846 * gd * (1 + 0.044715 * gd * gd))),
        SWIGLU: vd * silu(gd),
        SWIGLU_OAI: silu(1.702 * np.minimum(gd, 7)) / 1.702 * (np.minimum(vd, 7) + 1),
        GEGLU_QUICK: vd / (1 + np.exp(-1.702 * gd)),
        GEGLU_ERF: vd * 0.5 * gd * (1 + erf(gd / math.sqrt(2))),
    }
    scale = np.maximum(np.abs(vd), 1.0) * np.maximum(np.abs(gd), 1.0)
    for subop, w in want.items():
        st, out = run(lib, subop, x)
        assert st == 0
        err = np.abs(out.astype(np.float64) - w) / scale
        assert float(err.max()) < 4e-6, (subop, float(err.max()))


def test_x86_max_min_semantics(lib):
    """f32::max(0.0): NaN and -0.0 give +0.0; f32::min(7.0): NaN gives 7."""
    nan = np.float32("nan")
    st, out = run(lib, REGLU, [-1.0, 5.0, -0.0, nan])
    assert st == 0
    # -1 * relu(-0.0) = -1 * +0 = -0.0; 5 * relu(NaN) = 5 * 0 = +0
    assert bits(out).tolist() == bits([-0.0, 0.0]).tolist()
    st, a = run(lib, SWIGLU_OAI, [1.0, nan])
    st2, b = run(lib, SWIGLU_OAI, [1.0, 7.0])
    assert st == st2 == 0 and bits(a).tolist() == bits(b).tolist()
    st, a = run(lib, SWIGLU_OAI, [nan, 1.0])
    st2, b = run(lib, SWIGLU_OAI, [7.0, 1.0])
    assert bits(a).tolist() == bits(b).tolist()
