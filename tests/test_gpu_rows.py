"""Row-operator parity on the GPU: norm, rms_norm (+ fused weight), soft_max
(+ scale and f16 mask), sum_rows and per-row argmax, across every kernel
tier (warp / CTA / 1024-thread rows held in registers, cluster rows with
DSMEM exchange, streaming fallback, non-dense sequential-f32 softmax).

Tolerance: 1e-5 relative (the f64 accumulators only change summation
order); argmax indices are exact."""

import ctypes

import numpy as np
import pytest

import gpu_helpers as gh

pytestmark = pytest.mark.gpu

RTOL = 1e-5


@pytest.fixture(scope="module")
def kern(emel):
    return emel.Kernel(device=0, synchronize=True)


def run_row_op(emel, kern, olib, kind, x, ne, nb=None, eps=1e-5, weight=None, mask=None, scale=1.0,
               out_ne=None, out_nb=None, out_dtype=np.float32):
    ctx = kern.ctx
    px = gh.Pair(emel, ctx, x, ne, nb)
    if kind in ("sum_rows", "argmax_rows"):
        o_ne = [1] + list(ne[1:])
        out_host = np.zeros(int(np.prod(o_ne)), dtype=out_dtype)
        po = gh.Pair(emel, ctx, out_host, o_ne)
    else:
        out_host = np.full(x.size, 3.0, dtype=np.float32)
        po = gh.Pair(emel, ctx, out_host, out_ne or ne, out_nb)
    pw = gh.Pair(emel, ctx, weight) if weight is not None else None
    pm = gh.Pair(emel, ctx, mask[0], mask[1], mask[2]) if mask is not None else None
    B = ctypes.byref
    want = out_host.copy()
    wv = gh.oracle.make_view(want.ctypes.data, want.nbytes, po.ne, po.nb, po.code)
    if kind == "norm":
        ev = emel.OpNorm(px.dview(), po.dview(), eps)
        ost = olib.oracle_norm(B(px.oview()), B(wv), eps)
    elif kind == "rms_norm":
        ev = emel.OpRmsNorm(px.dview(), po.dview(), eps)
        ost = olib.oracle_rms_norm(B(px.oview()), B(wv), eps)
    elif kind == "rms_norm_mul":
        ev = emel.OpRmsNormMul(px.dview(), pw.dview(), po.dview(), eps)
        ost = olib.oracle_rms_norm_mul(B(px.oview()), B(pw.oview()), B(wv), eps)
    elif kind == "soft_max":
        ev = emel.OpSoftMax(px.dview(), po.dview())
        ost = olib.oracle_soft_max(B(px.oview()), B(wv))
    elif kind == "soft_max_ext":
        ev = emel.OpSoftMaxExt(px.dview(), pm.dview() if pm else None, po.dview(), scale)
        ost = olib.oracle_soft_max_ext(B(px.oview()), B(pm.oview()) if pm else None, B(wv), scale)
    elif kind == "sum_rows":
        ev = emel.OpSumRows(px.dview(), po.dview())
        ost = olib.oracle_sum_rows(B(px.oview()), B(wv))
    elif kind == "argmax_rows":
        ev = emel.OpArgmaxRows(px.dview(), po.dview())
        ost = olib.oracle_argmax_rows(B(px.oview()), B(wv))
    else:
        raise AssertionError(kind)
    st = kern.process_event(ev)
    assert st == emel.Status.OK, (kind, st, ctx.last_error)
    assert ost == 0
    got = po.download()
    for p in (px, po, pw, pm):
        if p is not None:
            p.free()
    return got, want


def close(got, want, floor, what):
    err = gh.max_rel_err(got, want, floor)
    exact = float(np.mean(got.view(np.uint32) == want.view(np.uint32)))
    assert err <= RTOL, f"{what}: max relative error {err:.3e} (bit-exact fraction {exact:.6f})"
    return exact


# ---- tiers -------------------------------------------------------------------
WIDTHS = [1, 7, 32, 1000, 1024, 1025, 4096, 8192, 8193, 32768, 40000]


@pytest.mark.parametrize("width", WIDTHS)
@pytest.mark.parametrize("kind", ["norm", "rms_norm", "soft_max"])
def test_row_tiers(emel, kern, oracle_lib, width, kind):
    rows = max(1, min(64, 200000 // width))
    rng = np.random.default_rng(width)
    x = (rng.standard_normal(width * rows) * 2).astype(np.float32)
    got, want = run_row_op(emel, kern, oracle_lib, kind, x, [width, rows, 1, 1], eps=1e-5)
    close(got, want, 1e-6 if kind != "soft_max" else 1e-30, f"{kind} width={width}")


@pytest.mark.parametrize("width", [151936, 300000])
def test_softmax_vocab_width_rows(emel, kern, oracle_lib, width):
    """151936 wide: cluster of CTAs with DSMEM; 300000: streaming fallback."""
    rng = np.random.default_rng(width)
    x = (rng.standard_normal(width * 3) * 3).astype(np.float32)
    got, want = run_row_op(emel, kern, oracle_lib, "soft_max", x, [width, 3, 1, 1])
    close(got, want, 1e-30, f"soft_max width={width}")


def test_row_ops_on_strided_views(emel, kern, oracle_lib):
    rng = np.random.default_rng(21)
    x = rng.standard_normal(2000).astype(np.float32)
    ne, nb = [64, 9, 1, 1], [8, 640, 5760, 5760]  # every other element, padded rows
    for kind in ("norm", "rms_norm", "soft_max"):
        got, want = run_row_op(emel, kern, oracle_lib, kind, x, ne, nb, eps=1e-5, out_ne=ne, out_nb=nb)
        close(got, want, 1e-30, f"{kind} strided")


def test_softmax_non_dense_keeps_sequential_f32_sum(emel, kern, oracle_lib):
    """reductions.rs:603-638: non-dense views sum in f32, in row order."""
    rng = np.random.default_rng(22)
    x = rng.standard_normal(3000 * 2 * 4).astype(np.float32)
    ne, nb = [3000, 4, 1, 1], [8, 24000, 96000, 96000]
    got, want = run_row_op(emel, kern, oracle_lib, "soft_max", x, ne, nb, out_ne=ne, out_nb=nb)
    close(got, want, 1e-30, "softmax sparse")


def test_softmax_count_equal_different_destination_extents(emel, kern, oracle_lib):
    rng = np.random.default_rng(23)
    x = rng.standard_normal(6 * 40).astype(np.float32)
    got, want = run_row_op(emel, kern, oracle_lib, "soft_max", x, [6, 40, 1, 1], out_ne=[40, 6, 1, 1])
    close(got, want, 1e-30, "softmax dense dst other extents")
    got, want = run_row_op(emel, kern, oracle_lib, "soft_max", x, [6, 40, 1, 1], out_ne=[10, 24, 1, 1],
                           out_nb=[4, 40, 960, 960])
    close(got, want, 1e-30, "softmax ordinal dst")


# ---- config 3 ----------------------------------------------------------------
@pytest.fixture(scope="module")
def cfg3_data(emel):
    from emel_rs_b200 import workloads
    return workloads.cfg3()


def test_cfg3_rms_norm_then_weight_full_size(emel, kern, oracle_lib, cfg3_data):
    x, w = cfg3_data
    ne = [4096, 8192, 1, 1]
    got, want = run_row_op(emel, kern, oracle_lib, "rms_norm", x, ne, eps=1e-6)
    exact = close(got, want, 1e-6, "cfg3 rms_norm")
    assert exact > 0.999
    got, want = run_row_op(emel, kern, oracle_lib, "rms_norm_mul", x, ne, eps=1e-6, weight=w)
    close(got, want, 1e-6, "cfg3 rms_norm * weight")


def test_cfg3_fused_weight_equals_two_events(emel, kern, oracle_lib, cfg3_data):
    """emel_cuda_rms_norm_mul is bit-identical to OpRmsNorm then OpMulBroadcastRow."""
    x, w = cfg3_data
    x = x[:512]
    ctx = kern.ctx
    ne = [4096, 512, 1, 1]
    px, pw = gh.Pair(emel, ctx, x, ne), gh.Pair(emel, ctx, w)
    pt, p1, p2 = (gh.Pair(emel, ctx, np.zeros_like(x), ne) for _ in range(3))
    assert kern.process_event(emel.OpRmsNorm(px.dview(), pt.dview(), 1e-6)) == emel.Status.OK
    assert kern.process_event(emel.OpMulBroadcastRow(pt.dview(), pw.dview(), p1.dview())) == emel.Status.OK
    assert kern.process_event(emel.OpRmsNormMul(px.dview(), pw.dview(), p2.dview(), 1e-6)) == emel.Status.OK
    gh.assert_bits_equal(p2.download(), p1.download(), "fused vs two events")


def test_cfg3_norm_and_sum_rows_full_size(emel, kern, oracle_lib, cfg3_data):
    x, _ = cfg3_data
    ne = [4096, 8192, 1, 1]
    got, want = run_row_op(emel, kern, oracle_lib, "norm", x, ne, eps=1e-5)
    close(got, want, 1e-6, "cfg3 norm")
    got, want = run_row_op(emel, kern, oracle_lib, "sum_rows", x, ne)
    close(got, want, 1e-6, "cfg3 sum_rows")


# ---- config 4 ----------------------------------------------------------------
def test_cfg4a_masked_scaled_softmax_full_size(emel, kern, oracle_lib):
    from emel_rs_b200 import workloads
    scores, mask = workloads.cfg4a()
    kv, q, h = workloads.CFG4A_NE
    got, want = run_row_op(emel, kern, oracle_lib, "soft_max_ext", scores, [kv, q, h, 1],
                           mask=(mask, [kv, q, 1, 1], None), scale=float(workloads.CFG4A_SCALE))
    close(got, want, 1e-30, "cfg4a soft_max_ext")
    # masked positions are exactly zero
    m = np.broadcast_to(mask[None].astype(np.float32), scores.shape).ravel()
    assert np.all(got[np.isneginf(m)] == 0.0)


def test_cfg4b_vocab_softmax_and_argmax_full_size(emel, kern, oracle_lib):
    from emel_rs_b200 import workloads
    logits, cols = workloads.cfg4b()
    v, rows = workloads.CFG4B_NE
    got, want = run_row_op(emel, kern, oracle_lib, "soft_max", logits, [v, rows, 1, 1])
    close(got, want, 1e-30, "cfg4b soft_max")
    for dt in (np.int64, np.int32, np.float32):
        got, want = run_row_op(emel, kern, oracle_lib, "argmax_rows", logits, [v, rows, 1, 1], out_dtype=dt)
        assert np.array_equal(got, want), f"cfg4b argmax_rows {np.dtype(dt).name}"
        assert np.array_equal(got.astype(np.int64), cols)


def test_argmax_rows_ties_and_nans(emel, kern, oracle_lib):
    x = np.array([1, 5, 5, 2,   # tie -> first
                  np.nan, 9, 9, 1,  # NaN first -> 0
                  -np.inf, -np.inf, -np.inf, -np.inf,  # all equal -> 0
                  0, np.nan, 3, 3], dtype=np.float32)  # NaN skipped
    got, want = run_row_op(emel, kern, oracle_lib, "argmax_rows", x, [4, 4, 1, 1], out_dtype=np.int64)
    assert got.tolist() == want.tolist() == [1, 0, 0, 2]


def test_mask_broadcast_over_heads_with_f32_mask(emel, kern, oracle_lib):
    rng = np.random.default_rng(31)
    kv, q, h = 256, 16, 4
    x = rng.standard_normal(kv * q * h).astype(np.float32)
    mask = np.where(rng.random((q + 3) * kv) < 0.2, -np.inf, rng.standard_normal((q + 3) * kv)).astype(np.float32)
    got, want = run_row_op(emel, kern, oracle_lib, "soft_max_ext", x, [kv, q, h, 1],
                           mask=(mask, [kv, q + 3, 1, 1], None), scale=0.37)
    close(got, want, 1e-30, "softmax f32 mask with extra rows")


# ---- ring-staged rows (bulk copies into shared memory) -----------------------
# Rows of >= 1024 floats with unit dim-0 stride and 16-byte aligned starts run
# on the ring kernel; these cases cover its addressing: padded row strides,
# 4-D views, strided destinations and weights, masks broadcast over dims 2/3,
# and masks that cannot be bulk-copied.
def padded_view(ne, pad_elems):
    """Contiguous rows of ne0 floats padded by pad_elems, dims 1..3 nested."""
    nb = [4, (ne[0] + pad_elems) * 4]
    nb.append(nb[1] * ne[1])
    nb.append(nb[2] * ne[2])
    return nb


def storage_for(ne, nb, rng, dtype=np.float32):
    span = sum((ne[d] - 1) * nb[d] for d in range(4)) // np.dtype(dtype).itemsize + 1
    return (rng.standard_normal(span) * 2).astype(dtype)


@pytest.mark.parametrize("kind", ["norm", "rms_norm", "soft_max"])
def test_ring_padded_4d_rows(emel, kern, oracle_lib, kind):
    rng = np.random.default_rng(41)
    ne = [2048, 5, 3, 2]
    nb = padded_view(ne, 12)
    x = storage_for(ne, nb, rng)
    if kind == "soft_max":  # soft_max's f64 path needs dense views: pad only the destination
        xd = (rng.standard_normal(int(np.prod(ne))) * 2).astype(np.float32)
        got, want = run_row_op(emel, kern, oracle_lib, kind, xd, ne, out_ne=ne)
    else:
        got, want = run_row_op(emel, kern, oracle_lib, kind, x, ne, nb, eps=1e-5, out_ne=ne, out_nb=nb)
    close(got, want, 1e-30, f"ring {kind} padded 4-D")


@pytest.mark.parametrize("kind", ["norm", "rms_norm"])
def test_ring_strided_destination(emel, kern, oracle_lib, kind):
    rng = np.random.default_rng(42)
    ne = [1024, 37, 1, 1]
    x = (rng.standard_normal(int(np.prod(ne))) * 3).astype(np.float32)
    out_nb = [8, 8 * 1024, 8 * 1024 * 37, 8 * 1024 * 37]  # every other float
    ctx = kern.ctx
    px = gh.Pair(emel, ctx, x, ne)
    po = gh.Pair(emel, ctx, np.full(2 * x.size, 3.0, np.float32), ne, out_nb)
    want = po.host.copy()
    B = ctypes.byref
    wv = gh.oracle.make_view(want.ctypes.data, want.nbytes, po.ne, po.nb, po.code)
    if kind == "norm":
        ost = oracle_lib.oracle_norm(B(px.oview()), B(wv), 1e-6)
        ev = emel.OpNorm(px.dview(), po.dview(), 1e-6)
    else:
        ost = oracle_lib.oracle_rms_norm(B(px.oview()), B(wv), 1e-6)
        ev = emel.OpRmsNorm(px.dview(), po.dview(), 1e-6)
    assert ost == 0
    assert kern.process_event(ev) == emel.Status.OK
    got = po.download()
    for p in (px, po):
        p.free()
    close(got, want, 1e-30, f"ring {kind} strided dst")
    assert np.all(got[1::2] == 3.0)  # the skipped floats are untouched


def test_ring_rms_norm_mul_strided_weight_many_rows(emel, kern, oracle_lib):
    rng = np.random.default_rng(43)
    ne = [1024, 5000, 1, 1]  # many rows per CTA: every stage's phase wraps several times
    x = rng.standard_normal(int(np.prod(ne))).astype(np.float32)
    w = rng.uniform(0.5, 1.5, 2048).astype(np.float32)
    ctx = kern.ctx
    px = gh.Pair(emel, ctx, x, ne)
    pw = gh.Pair(emel, ctx, w, [1024, 1, 1, 1], [8, 8192, 8192, 8192])
    po = gh.Pair(emel, ctx, np.zeros_like(x), ne)
    want = np.zeros_like(x)
    B = ctypes.byref
    wv = gh.oracle.make_view(want.ctypes.data, want.nbytes, po.ne, po.nb, po.code)
    assert oracle_lib.oracle_rms_norm_mul(B(px.oview()), B(pw.oview()), B(wv), 1e-6) == 0
    assert kern.process_event(emel.OpRmsNormMul(px.dview(), pw.dview(), po.dview(), 1e-6)) == emel.Status.OK
    got = po.download()
    for p in (px, pw, po):
        p.free()
    close(got, want, 1e-30, "ring rms_norm * strided weight")


@pytest.mark.parametrize("mask_kind", ["f16_broadcast_dims23", "f32_extra_rows", "f16_unaligned"])
def test_ring_softmax_ext_masks(emel, kern, oracle_lib, mask_kind):
    rng = np.random.default_rng(44)
    kv, q, h, b = 1536, 6, 4, 3
    x = (rng.standard_normal(kv * q * h * b) * 2).astype(np.float32)
    if mask_kind == "f16_broadcast_dims23":
        m = np.where(rng.random(kv * q * 2) < 0.3, -np.inf, rng.standard_normal(kv * q * 2)).astype(np.float16)
        mask = (m, [kv, q, 2, 1], None)  # dim 2 repeats every 2 heads, dim 3 broadcast
    elif mask_kind == "f32_extra_rows":
        m = np.where(rng.random(kv * (q + 5)) < 0.3, -np.inf, rng.standard_normal(kv * (q + 5))).astype(np.float32)
        mask = (m, [kv, q + 5, 1, 1], None)
    else:  # starts one element in: not 16-byte aligned, read with plain loads
        m = np.where(rng.random(kv * q + 1) < 0.3, -np.inf, rng.standard_normal(kv * q + 1)).astype(np.float16)
        mask = (m[1:].copy(), [kv, q, 1, 1], None)
        full = m  # device copy below keeps the one-element offset
        ctx = kern.ctx
        pfull = gh.Pair(emel, ctx, full, [kv * q + 1, 1, 1, 1])
        pm_view = pfull.dview()
        px = gh.Pair(emel, ctx, x, [kv, q, h, b])
        po = gh.Pair(emel, ctx, np.zeros_like(x), [kv, q, h, b])
        mv = emel.TensorView(pm_view.ptr + 2, pm_view.storage_bytes - 2,
                             emel.Layout.new(1, [kv, q, 1, 1], [2, 2 * kv, 2 * kv * q, 2 * kv * q]))
        want = np.zeros_like(x)
        B = ctypes.byref
        host_mask = mask[0]
        hm = gh.oracle.host_view(host_mask, [kv, q, 1, 1])
        wv = gh.oracle.make_view(want.ctypes.data, want.nbytes, po.ne, po.nb, po.code)
        assert oracle_lib.oracle_soft_max_ext(B(px.oview()), B(hm), B(wv), 0.3) == 0
        assert kern.process_event(emel.OpSoftMaxExt(px.dview(), mv, po.dview(), 0.3)) == emel.Status.OK
        got = po.download()
        for p in (pfull, px, po):
            p.free()
        close(got, want, 1e-30, "ring softmax unaligned f16 mask")
        return
    got, want = run_row_op(emel, kern, oracle_lib, "soft_max_ext", x, [kv, q, h, b], mask=mask, scale=0.3)
    close(got, want, 1e-30, f"ring softmax {mask_kind}")


@pytest.mark.parametrize("kv", [2048, 6000, 20000])
def test_ring_softmax_special_rows_take_the_exact_pass(emel, kern, oracle_lib, kv):
    """Rows with NaN (first element, middle), +inf, all -inf and a NaN in the
    mask: the fast pass hands these rows to the exact one, whose NaN payloads
    follow the reference; ordinary rows alongside stay exact too, including
    exps far below 2^-60 (subnormal quotients).  Widths 2048 and 6000 keep
    the row in registers (6000: a partial last vector slot), 20000 loops."""
    rng = np.random.default_rng(45)
    q = 8
    x = (rng.standard_normal(kv * q) * 3).astype(np.float32).reshape(q, kv)
    x[0, 10:30] = np.linspace(-110.0, -40.0, 20, dtype=np.float32)
    x[1, 0] = np.uint32(0x7fa00001).view(np.float32)  # signalling NaN first
    x[2, 700] = np.nan
    x[3, 5] = np.inf
    x[4, :] = -np.inf
    x[5, 3] = -np.inf
    mask = np.zeros((q, kv), np.float16)
    mask[6, 1000] = np.float16(np.nan)
    mask[7, :] = -np.inf
    mask[7, 9] = 0
    for scale, m in ((1.0, None), (0.5, (mask.ravel(), [kv, q, 1, 1], None))):
        kind = "soft_max" if m is None else "soft_max_ext"
        got, want = run_row_op(emel, kern, oracle_lib, kind, x.ravel(), [kv, q, 1, 1], mask=m, scale=scale)
        nan = np.isnan(want)
        assert np.array_equal(np.isnan(got), nan), f"ring {kind}: NaN positions"
        gh.assert_bits_equal(got[nan], want[nan], f"ring {kind} special rows: NaN payloads")
        close(got[~nan], want[~nan], 1e-30, f"ring {kind} special rows")


# ---- few long rows: one cluster of CTAs per row --------------------------------
def test_split_argmax_rows_ties_across_chunks_and_nans(emel, kern, oracle_lib):
    """Rows of 151936 split over eight CTAs: equal maxima in two chunks pick
    the earlier column; a NaN at column 0 pins 0; NaNs elsewhere are skipped;
    an all-NaN row gives 0."""
    rng = np.random.default_rng(46)
    v, rows = 151936, 10
    x = rng.standard_normal(v * rows).astype(np.float32).reshape(rows, v)
    x[6, :] = np.nan
    x[6, 0] = -np.inf        # comparable, so no NaN pin at column 0
    x[6, 140000] = -5.0      # the only other comparable value, late in the last chunk
    x[7, :] = 0.0
    x[7, 0] = -0.0           # -0 and +0 tie: the first column
    x[8, :] = -np.inf
    x[8, 3] = -1e30
    x[9, 1:40000] = np.nan   # NaNs ahead of every lane chain's first value
    x[9, 0] = -50.0
    x[9, 40001] = 7.0
    x[0, 150000] = 50.0
    x[0, 19000] = 50.0       # same maximum, earlier chunk
    x[1, 0] = np.nan
    x[1, 77] = 99.0
    x[2, ::3] = np.nan
    x[3, :] = np.nan
    x[4, 151935] = 1e30      # last column
    x[5, :] = -np.inf
    for dt in (np.int64, np.int32, np.float32):
        got, want = run_row_op(emel, kern, oracle_lib, "argmax_rows", x.ravel(), [v, rows, 1, 1], out_dtype=dt)
        assert np.array_equal(got, want), (np.dtype(dt).name, got, want)
    assert got.astype(np.int64).tolist()[:2] == [19000, 0]
    assert got.astype(np.int64).tolist()[6:] == [140000, 0, 3, 40001]


@pytest.mark.parametrize("width", [40001, 151936])
def test_split_sum_rows(emel, kern, oracle_lib, width):
    rng = np.random.default_rng(width)
    x = (rng.standard_normal(width * 5) * 10).astype(np.float32)
    got, want = run_row_op(emel, kern, oracle_lib, "sum_rows", x, [width, 5, 1, 1])
    close(got, want, 1e-3, f"split sum_rows width={width}")


def test_split_softmax_special_rows_and_mask(emel, kern, oracle_lib):
    rng = np.random.default_rng(47)
    v, rows = 40000, 6
    x = (rng.standard_normal(v * rows) * 3).astype(np.float32).reshape(rows, v)
    x[1, 0] = np.uint32(0x7fa00001).view(np.float32)
    x[2, 30000] = np.nan
    x[3, 123] = np.inf
    x[4, :] = -np.inf
    mask = np.where(rng.random((rows, v)) < 0.1, -np.inf, 0.0).astype(np.float16)
    mask[5, 5] = np.float16(np.nan)
    for kind, m, scale in (("soft_max", None, 1.0), ("soft_max_ext", (mask.ravel(), [v, rows, 1, 1], None), 0.7)):
        got, want = run_row_op(emel, kern, oracle_lib, kind, x.ravel(), [v, rows, 1, 1], mask=m, scale=scale)
        nan = np.isnan(want)
        assert np.array_equal(np.isnan(got), nan), f"split {kind}: NaN positions"
        gh.assert_bits_equal(got[nan], want[nan], f"split {kind}: NaN payloads")
        close(got[~nan], want[~nan], 1e-30, f"split {kind}")


@pytest.mark.parametrize("width,rows", [(16388, 5), (151936, 1), (40000, 148), (65540, 3)])
def test_split_rows_soft_max_scale_and_argmax(emel, kern, oracle_lib, width, rows):
    """Few long rows at widths whose chunk boundaries fall at arbitrary
    columns (16388 columns = 4097 vectors per row), one row, and as many
    rows as SMs: soft_max_ext with a scale and no mask (one row with an
    infinite maximum, redone with the x86 NaN rules) and argmax ties across
    chunks (the earlier column wins)."""
    rng = np.random.default_rng(width + rows)
    x = (rng.standard_normal(width * rows) * 3).astype(np.float32).reshape(rows, width)
    x[:, width // 3] = 50.0     # tie with the last column: the earlier one wins
    x[:, width - 1] = 50.0
    if rows > 2:
        x[2, 0] = np.inf        # an infinite maximum: the row is redone exactly
    got, want = run_row_op(emel, kern, oracle_lib, "soft_max_ext", x.ravel(), [width, rows, 1, 1], scale=0.37)
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan), "split soft_max_ext: NaN positions"
    close(got[~nan], want[~nan], 1e-30, f"split soft_max_ext {width}x{rows}")
    got, want = run_row_op(emel, kern, oracle_lib, "argmax_rows", x.ravel(), [width, rows, 1, 1], out_dtype=np.int32)
    assert np.array_equal(got, want), f"split argmax_rows {width}x{rows}"
