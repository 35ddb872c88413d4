"""Elementwise parity on the GPU: binary (equal-count ordinal contract), row
broadcast, repeat broadcast and the unary family, against the oracle on the
same seeded inputs.  Bit-exact for add/sub/mul/div, copies and every
non-transcendental formula; where the reference calls libm, within 2 ulp of
the glibc oracle for binary32 results (the tolerance for transcendental
unary ops) and within one binary16 step for binary16 results and GELU (whose
formula rounds its output through binary16)."""

import numpy as np
import pytest

import gpu_helpers as gh

pytestmark = pytest.mark.gpu

LIBM = {4, 5, 7, 8, 9, 10, 13, 14, 15, 16, 66, 67, 68}  # formulas that call exp/tanh/log/sin/cos
# binary32 results evaluated in binary64 and rounded once: the standalone
# tanh, log, sin, cos (bit-exact against the correctly rounded oracle up to
# rare double-rounding ties)
CR_OPS = {4, 66, 67, 68}


@pytest.fixture(scope="module")
def kern(emel):
    return emel.Kernel(device=0, synchronize=True)


@pytest.fixture(scope="module")
def olib(oracle_lib):
    return oracle_lib


def run_binary(emel, kern, olib, fn_dev, fn_or, op, a, b, out_ne=None, out_nb=None, a_ne=None, a_nb=None, b_ne=None,
               b_nb=None, out_storage=None):
    ctx = kern.ctx
    pa = gh.Pair(emel, ctx, a, a_ne, a_nb)
    pb = gh.Pair(emel, ctx, b, b_ne, b_nb)
    out_host = np.full(out_storage if out_storage is not None else a.size, 7.0, dtype=a.dtype)
    po = gh.Pair(emel, ctx, out_host, out_ne or pa.ne, out_nb)
    st = kern.process_event(fn_dev(op, pa.dview(), pb.dview(), po.dview()))
    assert st == emel.Status.OK, kern.ctx.last_error
    got = po.download()
    want = out_host.copy()
    wv = gh.oracle.make_view(want.ctypes.data, want.nbytes, po.ne, po.nb, po.code)
    assert gh.oracle_call(fn_or, op, pa.oview(), pb.oview(), wv) == 0
    for p in (pa, pb, po):
        p.free()
    return got, want


def dev_binary(emel):
    return lambda op, a, b, o: [emel.OpAdd, emel.OpSub, emel.OpMul, emel.OpDiv][op](a, b, o)


def dev_row(emel):
    return lambda op, a, b, o: [emel.OpAddBroadcastRow, emel.OpSubBroadcastRow, emel.OpMulBroadcastRow,
                                emel.OpDivBroadcastRow][op](a, b, o)


def dev_repeat(emel):
    return lambda op, a, b, o: emel.OpBinaryRepeat(emel.BinaryOp(op), a, b, o)


# ---------------------------------------------------------------------------
# binary.rs equal-count contract
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("n", [1, 3, 4, 127, 4097, 1 << 20])
@pytest.mark.parametrize("op", [0, 1, 2, 3])
@pytest.mark.parametrize("dtype", [np.float32, np.float16])
def test_binary_dense_bit_exact(emel, kern, olib, n, op, dtype):
    rng = np.random.default_rng(n * 10 + op)
    a = rng.standard_normal(n).astype(dtype)
    b = rng.uniform(0.5, 1.5, n).astype(dtype)
    got, want = run_binary(emel, kern, olib, dev_binary(emel), olib.oracle_binary, op, a, b)
    gh.assert_bits_equal(got, want, f"binary op={op} n={n} {np.dtype(dtype).name}")


def test_binary_strided_views_and_different_extents(emel, kern, olib):
    rng = np.random.default_rng(11)
    # lhs: a 2x3 view with padded rows; rhs: [6] dense; out: a transposed view
    a = rng.standard_normal(16).astype(np.float32)
    b = rng.standard_normal(6).astype(np.float32)
    got, want = run_binary(emel, kern, olib, dev_binary(emel), olib.oracle_binary, 2, a, b,
                           a_ne=[3, 2, 1, 1], a_nb=[4, 32, 64, 64], b_ne=[6, 1, 1, 1], b_nb=[4, 24, 24, 24],
                           out_ne=[2, 3, 1, 1], out_nb=[12, 4, 24, 24], out_storage=6)
    gh.assert_bits_equal(got, want, "binary mixed extents")


def test_binary_permuted_and_implicit_views(emel, kern, olib):
    rng = np.random.default_rng(12)
    ne = [64, 48, 5, 3]
    a = rng.standard_normal(int(np.prod(ne))).astype(np.float32)
    b = rng.standard_normal(int(np.prod(ne))).astype(np.float32)
    # a: dims 1 and 2 swapped over storage [64, 5, 48, 3]
    sn = [64, 5, 48, 3]
    snb = gh.contiguous_nb(sn, 4)
    got, want = run_binary(emel, kern, olib, dev_binary(emel), olib.oracle_binary, 0, a, b,
                           a_ne=[64, 48, 5, 3], a_nb=[snb[0], snb[2], snb[1], snb[3]],
                           b_ne=ne, b_nb=[0, 0, 0, 0], out_ne=ne, out_nb=[0, 0, 0, 0])
    gh.assert_bits_equal(got, want, "binary permuted/implicit")
    # non-unit element stride in dim 0 (generic kernel) and a singleton zero stride
    got, want = run_binary(emel, kern, olib, dev_binary(emel), olib.oracle_binary, 3, a, b,
                           a_ne=[100, 7, 1, 1], a_nb=[8, 800, 0, 0], b_ne=[100, 7, 1, 1], b_nb=[4, 400, 0, 0],
                           out_ne=[100, 7, 1, 1], out_nb=[12, 1200, 0, 0], out_storage=2100)
    gh.assert_bits_equal(got, want, "binary strided dim0")


def test_binary_misaligned_base_uses_scalar_path(emel, kern, olib):
    """A view starting 4 bytes into its buffer cannot use 16-byte vectors."""
    rng = np.random.default_rng(13)
    a = rng.standard_normal(1001).astype(np.float32)
    b = rng.standard_normal(1001).astype(np.float32)
    ctx = kern.ctx
    pa, pb = gh.Pair(emel, ctx, a), gh.Pair(emel, ctx, b)
    po = gh.Pair(emel, ctx, np.zeros(1001, np.float32))
    ne = [1000, 1, 1, 1]
    nb = gh.contiguous_nb(ne, 4)
    L = emel.Layout.new(0, ne, nb)
    va = emel.TensorView(pa.buf.ptr + 4, 4000, L)
    vb = emel.TensorView(pb.buf.ptr + 4, 4000, L)
    vo = emel.TensorView(po.buf.ptr + 4, 4000, L)
    assert kern.process_event(emel.OpMul(va, vb, vo)) == emel.Status.OK
    got = po.download()[1:]
    assert np.array_equal(got.view(np.uint32), (a[1:] * b[1:]).view(np.uint32))
    for p in (pa, pb, po):
        p.free()


def test_binary_nan_payloads_follow_sse_rules(emel, kern, olib):
    a = np.array([np.nan, 1.0, 0.0, np.inf, 2.0, -0.0], dtype=np.float32)
    a.view(np.uint32)[0] = 0x7FC01234
    b = np.array([3.0, np.nan, 0.0, np.inf, -0.0, 0.0], dtype=np.float32)
    b.view(np.uint32)[1] = 0xFFC05678
    for op in range(4):
        got, want = run_binary(emel, kern, olib, dev_binary(emel), olib.oracle_binary, op, a, b)
        gh.assert_bits_equal(got, want, f"binary NaN op={op}")


def test_binary_subnormals_are_kept(emel, kern, olib):
    a = (np.arange(1, 513, dtype=np.uint32)).view(np.float32)  # subnormals
    b = np.full(512, 3.0, dtype=np.float32)
    for op in range(4):
        got, want = run_binary(emel, kern, olib, dev_binary(emel), olib.oracle_binary, op, a, b)
        gh.assert_bits_equal(got, want, f"binary subnormal op={op}")


# ---------------------------------------------------------------------------
# broadcast.rs row contract and the repeat broadcast
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("op", [0, 1, 2, 3])
def test_cfg1_row_broadcast_full_size(emel, kern, olib, op):
    from emel_rs_b200 import workloads
    src0, src1 = workloads.cfg1()
    got, want = run_binary(emel, kern, olib, dev_row(emel), olib.oracle_broadcast_row, op, src0, src1)
    gh.assert_bits_equal(got, want, f"cfg1 op={op}")


@pytest.mark.parametrize("ne0,rows", [(1, 5), (3, 7), (4, 1000), (130, 33), (8192, 3)])
def test_row_broadcast_shapes(emel, kern, olib, ne0, rows):
    rng = np.random.default_rng(ne0 + rows)
    a = rng.standard_normal(ne0 * rows).astype(np.float32)
    b = rng.uniform(0.5, 1.5, ne0).astype(np.float32)
    for op in range(4):
        got, want = run_binary(emel, kern, olib, dev_row(emel), olib.oracle_broadcast_row, op, a, b,
                               a_ne=[ne0, rows, 1, 1])
        gh.assert_bits_equal(got, want, f"row ne0={ne0} rows={rows} op={op}")


@pytest.mark.parametrize("s1ne", [[8, 1, 6, 1], [1, 5, 1, 2], [8, 5, 6, 2], [1, 1, 1, 1], [4, 5, 3, 1]])
def test_repeat_broadcast_patterns(emel, kern, olib, s1ne):
    rng = np.random.default_rng(sum(s1ne))
    ne = [8, 5, 6, 2]
    a = rng.standard_normal(int(np.prod(ne))).astype(np.float32)
    b = rng.standard_normal(int(np.prod(s1ne))).astype(np.float32)
    for op in range(4):
        got, want = run_binary(emel, kern, olib, dev_repeat(emel), olib.oracle_binary_repeat, op, a, b,
                               a_ne=ne, b_ne=s1ne)
        gh.assert_bits_equal(got, want, f"repeat {s1ne} op={op}")


@pytest.mark.parametrize("op", [2, 0])
def test_cfg5_permuted_repeat_full_size(emel, kern, olib, op):
    """Config 5: src0 is a dims-1/2-swapped view of [128, 8192, 32, 8];
    src1 [128, 1, 8192, 1] repeats over dims 1 and 3."""
    from emel_rs_b200 import workloads
    src0, src1 = workloads.cfg5()
    ne, nb = workloads.cfg5_src0_view()
    got, want = run_binary(emel, kern, olib, dev_repeat(emel), olib.oracle_binary_repeat, op, src0, src1,
                           a_ne=ne, a_nb=nb, b_ne=[128, 1, 8192, 1], out_ne=ne,
                           out_nb=gh.contiguous_nb(ne, 4))
    gh.assert_bits_equal(got, want, f"cfg5 op={op}")


# ---------------------------------------------------------------------------
# unary family
# ---------------------------------------------------------------------------
UNARY_ALL = [0, 1, 2, 3, 4, 5, 6, 7, 8, 9, 10, 11, 12, 13, 14, 15, 16, 18, 19, 20, 21, 64, 65, 66, 67, 68]


def run_unary(emel, kern, olib, op, x, ne=None, nb=None, out_ne=None, out_nb=None):
    """Runs op on the device; returns (device, glibc-oracle, CR-oracle) outputs."""
    ctx = kern.ctx
    px = gh.Pair(emel, ctx, x, ne, nb)
    po = gh.Pair(emel, ctx, np.zeros_like(x), out_ne or px.ne, out_nb)
    st = kern.process_event(emel.OpUnaryTyped(emel.UnaryOp(op), px.dview(), po.dview()))
    assert st == emel.Status.OK, ctx.last_error
    got = po.download()
    outs = []
    for lib in (olib, gh.oracle.load(cr=True)):
        want = np.zeros_like(x)
        wv = gh.oracle.make_view(want.ctypes.data, want.nbytes, po.ne, po.nb, po.code)
        assert gh.oracle_call(lib.oracle_unary, op, px.oview(), wv) == 0
        outs.append(want)
    px.free()
    po.free()
    return got, outs[0], outs[1]


# GELU rounds its input and output through binary16 (unary.rs:533-539), so a
# libm difference shows up as at most one binary16 step of the output.
GELU = 8
# Formulas where 1 + tanh(...) or 1 - erf(...) cancels: compared by absolute error.
CANCELLING = {9, 15, 16}


def ulps(got, want):
    d = gh.ulp_diff_f16(got, want) if got.dtype == np.float16 else gh.ulp_diff_f32(got, want)
    both_nan = np.isnan(got.astype(np.float32)) & np.isnan(want.astype(np.float32))
    return np.where(both_nan, 0, d)


# sigmoid 1 / (1 + exp(-x)) and silu x / (1 + exp(-x)): from -x > 15.9 on
# exp(-x) >= 2^23 and the sum 1 + exp(-x) rounds, so the one-ulp rounding
# differences of glibc's expf (not correctly rounded everywhere) become up to
# 4 ulp of the reference's own quotient.  There the device evaluates the
# gate with the correctly rounded exp, and is compared with the correctly
# rounded oracle's formula; everywhere else with both oracles.
GATE_OPS = {7, 10}
GATE_CR_FROM = 15.9


def check_unary(op, got, want, want_cr, what, x=None):
    if op not in LIBM:
        gh.assert_bits_equal(got, want, what)
        return
    if op in GATE_OPS and x is not None and got.dtype == np.float32:
        band = -x.astype(np.float32) > np.float32(GATE_CR_FROM)
        d_band = ulps(got[band], want_cr[band])
        assert int(d_band.max(initial=0)) <= 1, f"{what}: {int(d_band.max())} ulp from the CR oracle in the gate band"
        got, want, want_cr = got[~band], want[~band], want_cr[~band]
    d = ulps(got, want)
    if got.dtype == np.float16:
        assert int(d.max(initial=0)) <= 1, f"{what}: {int(d.max())} binary16 ulp from glibc oracle"
    elif op == GELU:
        # outputs below |10| are binary16 values; above, the input passes through
        small = np.abs(want) < 10.0
        d16 = ulps(got[small].astype(np.float16), want[small].astype(np.float16))
        assert int(d16.max(initial=0)) <= 1, f"{what}: {int(d16.max())} binary16 steps from glibc oracle"
        gh.assert_bits_equal(got[~small], want[~small], what + " (|x| >= 10 passthrough)")
    elif op in CANCELLING:
        fin = np.isfinite(want)
        assert np.array_equal(np.isfinite(got), fin), f"{what}: non-finite positions"
        err = np.abs(got[fin].astype(np.float64) - want[fin].astype(np.float64))
        assert float(err.max(initial=0)) <= 1e-6 * max(1.0, float(np.abs(want[fin]).max(initial=0))), (
            f"{what}: absolute error {float(err.max())}")
    else:
        assert int(d.max(initial=0)) <= 2, f"{what}: {int(d.max())} ulp from glibc oracle"
        d_cr = ulps(got, want_cr)
        if op in CR_OPS:
            # binary64 evaluation rounded once: the correctly rounded oracle up
            # to rare double-rounding ties
            assert int(d_cr.max(initial=0)) <= 1 and int(np.count_nonzero(d_cr)) <= max(2, d_cr.size // 1_000_000), (
                f"{what}: vs CR oracle {int(np.count_nonzero(d_cr))} elements differ, max {int(d_cr.max())} ulp")
        else:
            # the binary32 exponential core (within 1 ulp of the correctly
            # rounded exp / expm1 over every binary32 input)
            assert int(d_cr.max(initial=0)) <= 2, f"{what}: {int(d_cr.max())} ulp from the CR oracle"


@pytest.mark.parametrize("op", UNARY_ALL)
@pytest.mark.parametrize("dtype", [np.float32, np.float16])
def test_unary_formulas_over_a_sweep(emel, kern, olib, op, dtype):
    rng = np.random.default_rng(op)
    x = np.concatenate([rng.standard_normal(100000) * 4,
                        np.array([0.0, -0.0, 10.0, -10.0, 10.1, -10.1, 1e-40, -1e-40, 88.0, -104.0, 3.5, -2.5,
                                  np.inf, -np.inf, np.nan])]).astype(np.float32)
    if op in (65, 66):
        x = np.abs(x) + np.float32(1e-3)
    x = x.astype(dtype)
    got, want, want_cr = run_unary(emel, kern, olib, op, x)
    check_unary(op, got, want, want_cr, f"unary op={op} {np.dtype(dtype).name}", x=x)


@pytest.mark.parametrize("dtype", [np.float32, np.float16])
def test_cfg2_unary_sweep_full_size(emel, kern, olib, dtype):
    from emel_rs_b200 import workloads
    x, xa = workloads.cfg2()
    ops = {"silu": 10, "gelu": 8, "relu": 6, "exp": 13, "neg": 2, "sqr": 64, "sqrt": 65, "pow2": 64}
    for name, op in ops.items():
        src = (xa if name in ("sqrt", "pow2") else x).astype(dtype)
        got, want, want_cr = run_unary(emel, kern, olib, op, src)
        check_unary(op, got, want, want_cr, f"cfg2 {name} {np.dtype(dtype).name}")


@pytest.mark.parametrize("op", UNARY_ALL)
def test_f16_every_input_large_tensor_matches_small(emel, kern, olib, op):
    """Every binary16 bit pattern (NaN payloads, infinities, subnormals, both
    zeros), once in a small tensor and 16 times plus a 5-element tail in a
    tensor of more than 2^20 elements (grid-stride loops, vector tails): both
    must give the same bits, and match the oracle."""
    every = np.arange(65536, dtype=np.uint16).view(np.float16)
    small, want, want_cr = run_unary(emel, kern, olib, op, every)
    check_unary(op, small, want, want_cr, f"f16 every input op={op}")
    big = np.concatenate([np.tile(every, 16), every[1000:1005]])
    got_big, _, _ = run_unary_device_only(emel, kern, op, big)
    gh.assert_bits_equal(got_big, np.concatenate([np.tile(small, 16), small[1000:1005]]),
                         f"f16 op={op}: large vs small tensor")


def test_gelu_f32_large_tensor_matches_small(emel, kern, olib):
    """binary32 GELU (the formula sees only binary16-rounded inputs and rounds
    its result through binary16) on more than 2^20 dense elements and on the
    same values split in four smaller tensors: both agree bit for bit,
    including inputs next to +-10 that round to +-10 in binary16, NaN
    payloads and infinities, and match the oracle."""
    rng = np.random.default_rng(8)
    near = np.array([9.99609375, 9.996094, 9.9960937, 9.999999, 10.0, -9.99609375, -9.996094, -9.999999, -10.0,
                     np.nextafter(np.float32(10), np.float32(0)), np.nextafter(np.float32(-10), np.float32(0)),
                     65519.0, 65520.0, 1e-8, -1e-8, 6e-8, 0.0, -0.0, np.inf, -np.inf], dtype=np.float32)
    nans = np.array([0x7fc00000, 0xffc00000, 0x7f800001, 0xff812345, 0x7fbfffff], dtype=np.uint32).view(np.float32)
    x = np.concatenate([rng.uniform(-11, 11, 1 << 21).astype(np.float32), near, nans,
                        (rng.standard_normal(1 << 16) * 1e-3).astype(np.float32)])
    got_big, _, _ = run_unary_device_only(emel, kern, 8, x)
    parts = [run_unary_device_only(emel, kern, 8, c)[0] for c in np.array_split(x, 4)]
    gh.assert_bits_equal(got_big, np.concatenate(parts), "gelu f32: one large tensor vs four smaller ones")
    small = np.concatenate([near, nans, x[:200000]])
    got, want, want_cr = run_unary(emel, kern, olib, 8, small)
    check_unary(8, got, want, want_cr, "gelu f32 edge values")


def run_unary_device_only(emel, kern, op, x):
    ctx = kern.ctx
    px = gh.Pair(emel, ctx, x)
    po = gh.Pair(emel, ctx, np.zeros_like(x))
    st = kern.process_event(emel.OpUnaryTyped(emel.UnaryOp(op), px.dview(), po.dview()))
    assert st == emel.Status.OK, ctx.last_error
    got = po.download()
    px.free()
    po.free()
    return got, None, None


def test_unary_strided_and_count_equal_views(emel, kern, olib):
    rng = np.random.default_rng(3)
    x = rng.standard_normal(4000).astype(np.float32)
    got, want, want_cr = run_unary(emel, kern, olib, 10, x, ne=[50, 20, 1, 1], nb=[8, 400, 8000, 8000],
                                   out_ne=[20, 50, 1, 1], out_nb=[4, 80, 4000, 4000])
    check_unary(10, got[:1000], want[:1000], want_cr[:1000], "unary strided/count-equal")


@pytest.mark.parametrize("op", [7, 8, 10, 13])  # sigmoid, gelu, silu, exp
def test_packed_pairs_match_scalar_pass(emel, kern, olib, op):
    """Dense binary32 tensors run these formulas two elements per packed
    instruction; a strided view of the same values runs them one element at a
    time.  Both must give the same bits on random bit patterns of every
    exponent, the exp range edges (-86, 88.72, -104, 89), +-10, zeros,
    infinities and NaN payloads, and stay within the oracle's bar."""
    rng = np.random.default_rng(op + 100)
    pats = rng.integers(0, 1 << 32, 1 << 20, dtype=np.uint64).astype(np.uint32).view(np.float32)
    edges = np.array([-86.0, np.nextafter(np.float32(-86), np.float32(-87)), 88.72, np.nextafter(np.float32(88.72),
                      np.float32(89)), -104.0, 89.0, -87.5, 10.0, -10.0, 0.0, -0.0, 1e-40, -1e-40, np.inf, -np.inf],
                     dtype=np.float32)
    nans = np.array([0x7fc00000, 0xffc00000, 0x7f800001, 0xff812345], dtype=np.uint32).view(np.float32)
    smooth = (rng.standard_normal(1 << 18) * 8).astype(np.float32)
    x = np.concatenate([pats, edges, nans, smooth, edges[::-1]])
    n = x.size
    dense, _, _ = run_unary_device_only(emel, kern, op, x)
    # every other element of a twice-as-long buffer: the per-element path
    wide = np.zeros(2 * n, dtype=np.float32)
    wide[::2] = x
    strided, _, _ = run_unary(emel, kern, olib, op, wide, ne=[n, 1, 1, 1], nb=[8, 8 * n, 8 * n, 8 * n],
                              out_ne=[n, 1, 1, 1], out_nb=[4, 4 * n, 4 * n, 4 * n])
    gh.assert_bits_equal(dense, strided[:n], f"op={op}: packed pairs vs the per-element pass")
    got, want, want_cr = run_unary(emel, kern, olib, op, x)
    gh.assert_bits_equal(got, dense, f"op={op}: repeat run")
    check_unary(op, got, want, want_cr, f"op={op} packed pairs vs oracle", x=x)


def test_parameterised_activations(emel, kern, olib):
    rng = np.random.default_rng(5)
    x = (rng.standard_normal(70001) * 3).astype(np.float32)
    x[:3] = [np.nan, np.inf, -np.inf]
    ctx = kern.ctx
    px = gh.Pair(emel, ctx, x)
    po = gh.Pair(emel, ctx, np.zeros_like(x))
    cases = [
        (emel.OpScale(px.dview(), po.dview(), 1.5), lambda o: olib.oracle_scale(*o, 1.5)),
        (emel.OpClamp(px.dview(), po.dview(), -1.0, 1.0), lambda o: olib.oracle_clamp(*o, -1.0, 1.0)),
        (emel.OpLeakyRelu(px.dview(), po.dview(), 0.125), lambda o: olib.oracle_leaky_relu(*o, 0.125)),
        (emel.OpAdd1(px.dview(), po.dview(), 0.3), lambda o: olib.oracle_add1(*o, 0.3)),
        (emel.CopyTensor(px.dview(), po.dview()), lambda o: olib.oracle_copy(*o)),
    ]
    import ctypes
    for ev, orc in cases:
        assert kern.process_event(ev) == emel.Status.OK
        got = po.download()
        want = np.zeros_like(x)
        wv = gh.oracle.make_view(want.ctypes.data, want.nbytes, po.ne, po.nb, 0)
        assert orc((ctypes.byref(px.oview()), ctypes.byref(wv))) == 0
        gh.assert_bits_equal(got, want, type(ev).__name__)
    px.free()
    po.free()


def test_silu_back(emel, kern, olib):
    import ctypes
    rng = np.random.default_rng(9)
    x = (rng.standard_normal(5000) * 3).astype(np.float32)
    g = rng.standard_normal(5000).astype(np.float32)
    ctx = kern.ctx
    px, pg, po = gh.Pair(emel, ctx, x), gh.Pair(emel, ctx, g), gh.Pair(emel, ctx, np.zeros_like(x))
    assert kern.process_event(emel.OpSiluBack(px.dview(), pg.dview(), po.dview())) == emel.Status.OK
    got = po.download()
    want = np.zeros_like(x)
    wv = gh.oracle.make_view(want.ctypes.data, want.nbytes, po.ne, po.nb, 0)
    assert olib.oracle_silu_back(ctypes.byref(px.oview()), ctypes.byref(pg.oview()), ctypes.byref(wv)) == 0
    assert int(gh.ulp_diff_f32(got, want).max()) <= 2
