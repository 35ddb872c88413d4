"""emel_cuda_glu (glu.rs OpGlu on the device) against the oracle
restatement, through the C ABI.

Bars: ReGlu bit-exact against the glibc oracle (no libm call); SwiGlu,
SwiGluOai and GeGluQuick (value times a sigmoid of the gate, binary32
exponential core) within 4 ulp of the correctly-rounded oracle: the
exponential is within 1 ulp, and each later binary32 rounding of the gate
(add, divide, the OAI variant's divide by 1.702 and its (v + 1) product) can
carry a difference of its input into at most one more ulp; GeGlu and
GeGluErf, whose 1 + tanh / 1 - erf cancels for negative gates, within an
absolute 1e-6 of the output scale; NaN positions and payloads bit-exact
everywhere (x86 rules; for GeGluErf up to the sign, see test_glu_parity).  Sizes cover 16-byte vector halves
(n % 4 == 0), unaligned halves (n odd) and tails."""

import ctypes

import numpy as np
import pytest

import gpu_helpers as gh
import oracle

pytestmark = pytest.mark.gpu

SUBOPS = [0, 1, 2, 3, 4, 5]


@pytest.fixture(scope="module")
def kern(emel):
    return emel.Kernel(device=0, synchronize=True)


@pytest.fixture(scope="module")
def cr_lib():
    return oracle.load(cr=True)


def special_input(rng, n):
    x = (rng.standard_normal(2 * n) * 4).astype(np.float32)
    sp = np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 7.0, 7.5, -7.5, 1e-40, -1e-40, 20.0, -20.0, 89.0, -104.0,
                   np.uint32(0x7fa00011).view(np.float32), np.uint32(0xffc00123).view(np.float32)], np.float32)
    k = min(sp.size, n)
    x[:k] = sp[:k]              # values
    x[n:n + k] = sp[::-1][:k]   # gates
    if n > 2 * k:
        x[k:2 * k] = sp[:k]     # the specials against ordinary partners too
        x[n + k + 3:n + 2 * k + 3] = sp[:k]
    return x


def run_device(emel, kern, subop, x, n, out_fill=3.0):
    ctx = kern.ctx
    bi = emel.DeviceBuffer(ctx, x.nbytes)
    bi.upload(x)
    out = np.full(n, out_fill, np.float32)
    bo = emel.DeviceBuffer(ctx, max(out.nbytes, 4))
    bo.upload(out)
    st = kern.process_event(emel.OpGlu((bi.ptr, x.size), (bo.ptr, n), emel.GluSubOp(subop)))
    got = bo.download(np.empty_like(out))
    bi.free()
    bo.free()
    return st, got


def run_oracle(lib, subop, x, n):
    out = np.full(n, 3.0, np.float32)
    assert lib.oracle_glu(subop, x.ctypes.data, x.size, out.ctypes.data, n) == 0
    return out


def libm_close(got, want, what, nan_sign=True, cancelling=False):
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan), f"{what}: NaN positions"
    if nan_sign:
        gh.assert_bits_equal(got[nan], want[nan], f"{what}: NaN payloads")
    else:
        g, w = got[nan].view(np.uint32) & 0x7fffffff, want[nan].view(np.uint32) & 0x7fffffff
        assert np.array_equal(g, w), f"{what}: NaN payloads"
    if cancelling:
        g, w = got[~nan].astype(np.float64), want[~nan].astype(np.float64)
        fin = np.isfinite(w)
        assert np.array_equal(np.isfinite(g), fin), f"{what}: non-finite positions"
        err = float(np.max(np.abs(g[fin] - w[fin]), initial=0.0))
        assert err <= 1e-6 * max(1.0, float(np.max(np.abs(w[fin]), initial=0.0))), f"{what}: absolute error {err}"
        return
    d = gh.ulp_diff_f32(got[~nan], want[~nan])
    assert int(d.max(initial=0)) <= 4, f"{what}: {int(np.count_nonzero(d))} differ, max {d.max()} ulp"


@pytest.mark.parametrize("subop", SUBOPS)
@pytest.mark.parametrize("n", [1, 7, 4096, 65537, 1 << 20])
def test_glu_parity(emel, kern, oracle_lib, cr_lib, subop, n):
    rng = np.random.default_rng(subop * 100 + n % 97)
    x = special_input(rng, n)
    st, got = run_device(emel, kern, subop, x, n)
    assert st == emel.Status.OK, kern.ctx.last_error
    if subop == 0:
        gh.assert_bits_equal(got, run_oracle(oracle_lib, subop, x, n), f"reglu n={n}")
    else:
        # GeGluErf: a NaN gate reaches `polynomial * exp(-x * x)` as two NaNs
        # of opposite sign (x and -x); which one a commutative multiply
        # returns is the compiler's operand order, not the source's (the C
        # oracle's compiler swaps them), so only that sign is left open
        libm_close(got, run_oracle(cr_lib, subop, x, n), f"glu {subop} n={n}", nan_sign=subop != 4,
                   cancelling=subop in (1, 4))


@pytest.mark.parametrize("in_len,out_len", [(0, 0), (7, 3), (8, 3), (8, 5)])
def test_glu_invalid_shape_writes_nothing(emel, kern, in_len, out_len):
    ctx = kern.ctx
    bi = emel.DeviceBuffer(ctx, 64)
    bo = emel.DeviceBuffer(ctx, 64)
    bo.upload(np.full(16, 9.0, np.float32))
    st = kern.process_event(emel.OpGlu((bi.ptr, in_len), (bo.ptr, out_len), emel.GluSubOp.SWIGLU))
    assert st == emel.Status.INVALID_SHAPE
    assert np.all(bo.download(np.empty(16, np.float32)) == 9.0)
    bi.free()
    bo.free()


def test_glu_unknown_subop_and_null_pointer(emel, kern):
    lib = emel.lib()
    ctx = kern.ctx
    b = emel.DeviceBuffer(ctx, 64)
    assert lib.emel_cuda_glu(ctx.handle, None, 6, ctypes.c_void_p(b.ptr), 8, ctypes.c_void_p(b.ptr), 4) == \
        emel.Status.INVALID_ARGUMENT
    assert lib.emel_cuda_glu(ctx.handle, None, 0, None, 8, ctypes.c_void_p(b.ptr), 4) == emel.Status.INVALID_ARGUMENT
    b.free()


@pytest.mark.parametrize("half", [0, 1])
def test_glu_in_place_over_either_half(emel, kern, cr_lib, half):
    """output may be exactly the values half or the gates half."""
    n = 10000
    rng = np.random.default_rng(3 + half)
    x = (rng.standard_normal(2 * n) * 3).astype(np.float32)
    want = run_oracle(cr_lib, 2, x, n)
    ctx = kern.ctx
    bi = emel.DeviceBuffer(ctx, x.nbytes)
    bi.upload(x)
    out_ptr = bi.ptr + half * n * 4
    st = kern.process_event(emel.OpGlu((bi.ptr, 2 * n), (out_ptr, n), emel.GluSubOp.SWIGLU))
    assert st == emel.Status.OK
    got = bi.download(np.empty_like(x))[half * n:(half + 1) * n]
    bi.free()
    libm_close(got, want, f"in-place swiglu half={half}")
