"""Generic operation envelope on the GPU (emel_cuda_generic) against the
oracle's restatement of the generic loops (generic.rs:1263-2050), on
seeded inputs including strided, permuted and count-equal reshaped views.

Bars: bit-exact for copies, arithmetic, scalar ops, clamp, abs/neg/relu,
sqr/sqrt, repeat and argmax (glibc oracle); tanh, log, sin, cos and
silu_back (binary64 evaluation rounded once) bit-exact against the
correctly-rounded oracle up to rare double-rounding ties (at most max(2,
n/10^6) elements, 1 ulp); elu, silu and exp (binary32 exponential core)
within 2 ulp of it; GELU (1 + tanh cancels for negative inputs) within an
absolute 1e-6 of the output scale; soft_max and sum/mean/norm within 1e-5
relative."""

import ctypes
import struct

import numpy as np
import pytest

import gpu_helpers as gh
import oracle

pytestmark = pytest.mark.gpu


def f32_params(*values):
    return b"".join(struct.pack("=f", v) for v in values)


@pytest.fixture(scope="module")
def kern(emel):
    return emel.Kernel(device=0, synchronize=True)


@pytest.fixture(scope="module")
def cr_lib():
    return oracle.load(cr=True)


def run_generic(emel, kern, olib, op, srcs, dst_ne, dst_nb=None, params=b"", unary=0, dst_fill=3.0):
    """srcs: list of (array, ne, nb).  Returns (device output, oracle output)."""
    ctx = kern.ctx
    pairs = [gh.Pair(emel, ctx, a, ne, nb) for a, ne, nb in srcs]
    span = 1 if dst_nb is None else None
    n = int(np.prod(dst_ne))
    if dst_nb is not None:
        n = sum((dst_ne[d] - 1) * dst_nb[d] for d in range(4)) // 4 + 1
    out = np.full(n, dst_fill, np.float32)
    po = gh.Pair(emel, ctx, out, dst_ne, dst_nb)
    views = [p.dview() for p in pairs] + [None] * (3 - len(pairs))
    ev = emel.GenericEvent(op, src0=views[0], src1=views[1], dst=po.dview(), params=params, unary=unary)
    st = kern.process_event(ev)
    assert st == emel.Status.OK, (op, st, ctx.last_error)
    got = po.download()
    want = out.copy()
    ovs = [p.oview() for p in pairs] + [None] * (2 - len(pairs))
    wv = oracle.make_view(want.ctypes.data, want.nbytes, po.ne, po.nb, 0)
    r = oracle.generic_request(op, ovs[0], ovs[1], None, wv, params, unary)
    assert olib.oracle_generic(ctypes.byref(r)) == 0
    for p in pairs + [po]:
        p.free()
    return got, want


def libm_close(got, want, what, max_ulp=1):
    """max_ulp 1: the correctly rounded oracle up to rare double-rounding
    ties; 2: the binary32 exponential core's bar."""
    g, w = got.view(np.uint32).astype(np.int64), want.view(np.uint32).astype(np.int64)
    both_nan = np.isnan(got) & np.isnan(want)
    d = np.where(both_nan, 0, np.abs(g - w))
    bad = int(np.count_nonzero(d))
    if max_ulp == 1:
        assert int(d.max(initial=0)) <= 1 and bad <= max(2, got.size // 1_000_000), f"{what}: {bad} differ, max {d.max()}"
    else:
        assert int(d.max(initial=0)) <= max_ulp, f"{what}: {bad} differ, max {d.max()}"


def abs_close(got, want, what):
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan), f"{what}: NaN positions"
    g, w = got[~nan].astype(np.float64), want[~nan].astype(np.float64)
    fin = np.isfinite(w)
    assert np.array_equal(np.isfinite(g), fin), f"{what}: non-finite positions"
    err = float(np.max(np.abs(g[fin] - w[fin]), initial=0.0))
    assert err <= 1e-6 * max(1.0, float(np.max(np.abs(w[fin]), initial=0.0))), f"{what}: absolute error {err}"


def rel_close(got, want, what, tol=1e-5):
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan), f"{what}: NaN positions"
    err = gh.max_rel_err(got[~nan], want[~nan], 1e-30)
    assert err <= tol, f"{what}: relative error {err}"


def rand(rng, n, scale=3.0):
    return (rng.standard_normal(n) * scale).astype(np.float32)


# ---- elementwise ---------------------------------------------------------------
EXACT_UNARY = [(85, 0, "abs"), (85, 2, "neg"), (85, 6, "relu"), (8, 0, "sqr"), (9, 0, "sqrt")]
LIBM_UNARY = [(85, 4, "tanh"), (85, 5, "elu"), (85, 8, "gelu"), (85, 10, "silu"), (85, 13, "exp"),
              (10, 0, "log"), (11, 0, "sin"), (12, 0, "cos")]


@pytest.mark.parametrize("op,sub,name", EXACT_UNARY + LIBM_UNARY)
def test_generic_unary(emel, kern, oracle_lib, cr_lib, op, sub, name):
    rng = np.random.default_rng(op * 31 + sub)
    x = np.concatenate([rand(rng, 200000), np.array([0.0, -0.0, np.inf, -np.inf, np.nan, 1e-40, -11.0, 11.0,
                                                     88.0, -104.0], np.float32)])
    if name in ("sqrt", "log"):
        x = np.abs(x)
    lib = cr_lib if (op, sub, name) in LIBM_UNARY else oracle_lib
    got, want = run_generic(emel, kern, lib, op, [(x, None, None)], [x.size, 1, 1, 1], unary=sub)
    if name == "gelu":
        abs_close(got, want, f"generic {name}")
    elif name in ("elu", "silu", "exp"):
        libm_close(got, want, f"generic {name}", max_ulp=2)
    elif lib is cr_lib:
        libm_close(got, want, f"generic {name}")
    else:
        gh.assert_bits_equal(got, want, f"generic {name}")


def test_generic_unary_on_a_permuted_view_into_other_extents(emel, kern, cr_lib):
    rng = np.random.default_rng(3)
    x = rand(rng, 24 * 50)
    # [50, 24] storage read as a transposed [24, 50] view; dst [1200] contiguous (count-equal)
    got, want = run_generic(emel, kern, cr_lib, 85, [(x, [24, 50, 1, 1], [200, 4, 4800, 4800])], [1200, 1, 1, 1],
                            unary=8)
    abs_close(got, want, "generic gelu permuted")


@pytest.mark.parametrize("op", [1, 5, 6, 7])
def test_generic_binary_count_equal(emel, kern, oracle_lib, op):
    rng = np.random.default_rng(op)
    a = rand(rng, 6 * 40 * 3)
    b = (rng.uniform(0.5, 2.0, 720) * np.sign(rng.standard_normal(720))).astype(np.float32)
    b[:5] = [np.nan, np.inf, -np.inf, 0.0, -0.0]
    got, want = run_generic(emel, kern, oracle_lib, op, [(a, [6, 40, 3, 1], None), (b, [720, 1, 1, 1], None)],
                            [40, 18, 1, 1])
    gh.assert_bits_equal(got, want, f"generic binary {op}")


@pytest.mark.parametrize("op,params", [(3, f32_params(0.75)), (32, f32_params(-1.5)), (70, f32_params(0.1)),
                                       (50, f32_params(-0.5, 0.25))])
def test_generic_scalar_and_clamp(emel, kern, oracle_lib, op, params):
    rng = np.random.default_rng(op)
    x = rand(rng, 70001)
    x[:3] = [np.nan, np.inf, -np.inf]
    got, want = run_generic(emel, kern, oracle_lib, op, [(x, None, None)], [x.size, 1, 1, 1], params=params)
    gh.assert_bits_equal(got, want, f"generic scalar op {op}")


def test_generic_silu_back(emel, kern, cr_lib):
    rng = np.random.default_rng(22)
    x, g = rand(rng, 50000), rand(rng, 50000)
    got, want = run_generic(emel, kern, cr_lib, 22, [(x, [500, 100, 1, 1], None), (g, [500, 100, 1, 1], None)],
                            [500, 100, 1, 1])
    libm_close(got, want, "generic silu_back")


@pytest.mark.parametrize("src_ne,dst_ne", [([4, 3, 1, 1], [8, 6, 2, 3]), ([1, 5, 1, 2], [7, 10, 3, 4]),
                                           ([128, 1, 64, 1], [128, 8, 64, 2])])
def test_generic_repeat(emel, kern, oracle_lib, src_ne, dst_ne):
    rng = np.random.default_rng(sum(dst_ne))
    x = rand(rng, int(np.prod(src_ne)))
    x[0] = np.uint32(0x7fa00005).view(np.float32)  # a signalling NaN is copied bit for bit
    got, want = run_generic(emel, kern, oracle_lib, 19, [(x, src_ne, None)], dst_ne)
    gh.assert_bits_equal(got, want, f"generic repeat {src_ne}->{dst_ne}")


# ---- reductions and rows ----------------------------------------------------------
def test_generic_sum_mean_argmax(emel, kern, oracle_lib):
    rng = np.random.default_rng(13)
    x = rand(rng, 300 * 97 * 2)
    ne, nb = [300, 97, 1, 1], [8, 2400, 232800, 232800]
    for op in (13, 16):
        got, want = run_generic(emel, kern, oracle_lib, op, [(x, ne, nb)], [1, 1, 1, 1])
        assert abs(float(got[0]) - float(want[0])) <= 1e-5 * max(1.0, abs(float(want[0]))), (op, got, want)
    x[[5000, 20000]] = 50.0  # tie: earliest
    got, want = run_generic(emel, kern, oracle_lib, 17, [(x, ne, nb)], [1, 1, 1, 1])
    assert got[0] == want[0]


@pytest.mark.parametrize("width", [7, 1000, 5000, 70000])
def test_generic_soft_max(emel, kern, cr_lib, width):
    rng = np.random.default_rng(width)
    rows = max(2, min(40, 300000 // width))
    x = rand(rng, width * rows, 4.0).reshape(rows, width)
    x[0, 0] = np.nan   # generic: skipped by the maximum, NaN only through its own exp
    x[1, :] = -np.inf
    got, want = run_generic(emel, kern, cr_lib, 46, [(x.ravel(), [width, rows, 1, 1], None)], [width, rows, 1, 1])
    rel_close(got, want, f"generic soft_max width={width}")


def test_generic_soft_max_reshaped_destination(emel, kern, cr_lib):
    rng = np.random.default_rng(9)
    x = rand(rng, 64 * 30)
    got, want = run_generic(emel, kern, cr_lib, 46, [(x, [64, 30, 1, 1], None)], [30, 64, 1, 1])
    rel_close(got, want, "generic soft_max into other extents")


@pytest.mark.parametrize("op", [23, 24])
@pytest.mark.parametrize("width", [33, 4096, 40000])
def test_generic_norms(emel, kern, oracle_lib, op, width):
    rng = np.random.default_rng(op + width)
    rows = max(1, min(64, 400000 // width))
    x = rand(rng, width * rows, 2.0)
    got, want = run_generic(emel, kern, oracle_lib, op, [(x, [width, rows, 1, 1], None)], [width, rows, 1, 1],
                            params=f32_params(1e-5))
    err = gh.max_rel_err(got, want, 1e-6)
    assert err <= 1e-5, (op, width, err)
