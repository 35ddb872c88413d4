"""Whole-tensor reductions on the GPU: sum / mean (f64 accumulation, 1e-5
relative) and argmax (exact first index, the reference's NaN rule), for
dense and strided views, plus the per-shard partial + combine path used by
multi-GPU runs."""

import ctypes

import numpy as np
import pytest

import gpu_helpers as gh

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def kern(emel):
    return emel.Kernel(device=0, synchronize=True)


def scalar_out(emel, ctx, dtype):
    return gh.Pair(emel, ctx, np.zeros(1, dtype=dtype), [1, 1, 1, 1])


def device_sum(emel, kern, x, ne, nb=None, event="sum"):
    ctx = kern.ctx
    px = gh.Pair(emel, ctx, x, ne, nb)
    po = scalar_out(emel, ctx, np.float32)
    ev = emel.OpSum if event == "sum" else emel.OpMean
    assert kern.process_event(ev(px.dview(), po.dview())) == emel.Status.OK, ctx.last_error
    got = po.download()[0]
    want = np.zeros(1, np.float32)
    wv = gh.oracle.make_view(want.ctypes.data, 4, [1, 1, 1, 1], [4, 4, 4, 4], 0)
    return got, want, px, po, wv


@pytest.mark.parametrize("n", [1, 5, 4096, 1000003, 1 << 24])
def test_sum_and_mean_dense(emel, kern, oracle_lib, n):
    rng = np.random.default_rng(n)
    x = rng.standard_normal(n).astype(np.float32)
    for event in ("sum", "mean"):
        got, want, px, po, wv = device_sum(emel, kern, x, [n, 1, 1, 1], event=event)
        fn = oracle_lib.oracle_sum if event == "sum" else oracle_lib.oracle_mean
        assert fn(ctypes.byref(px.oview()), ctypes.byref(wv)) == 0
        assert abs(float(got) - float(want[0])) <= 1e-5 * max(abs(float(want[0])), 1e-3), (event, got, want)
        px.free()
        po.free()


def test_sum_strided_view(emel, kern, oracle_lib):
    rng = np.random.default_rng(3)
    x = rng.standard_normal(100 * 37 * 2).astype(np.float32)
    ne, nb = [100, 37, 1, 1], [8, 800, 29600, 29600]
    got, want, px, po, wv = device_sum(emel, kern, x, ne, nb)
    assert oracle_lib.oracle_sum(ctypes.byref(px.oview()), ctypes.byref(wv)) == 0
    assert abs(float(got) - float(want[0])) <= 1e-5 * abs(float(want[0]))


def test_sum_is_deterministic(emel, kern):
    rng = np.random.default_rng(4)
    x = rng.standard_normal(1 << 22).astype(np.float32)
    vals = {device_sum(emel, kern, x, [1 << 22, 1, 1, 1])[0].tobytes() for _ in range(5)}
    assert len(vals) == 1


def device_argmax(emel, kern, x, ne, nb=None, dtype=np.int64):
    ctx = kern.ctx
    px = gh.Pair(emel, ctx, x, ne, nb)
    po = scalar_out(emel, ctx, dtype)
    assert kern.process_event(emel.OpArgmax(px.dview(), po.dview())) == emel.Status.OK, ctx.last_error
    got = po.download()[0]
    idx = ctypes.c_int64()
    assert gh.oracle_call(kern_oracle(), px.oview(), ctypes.byref(idx), None) == 0
    px.free()
    po.free()
    return got, idx.value


_olib = None


def kern_oracle():
    return _olib.oracle_argmax_index


@pytest.fixture(autouse=True, scope="module")
def _bind(oracle_lib):
    global _olib
    _olib = oracle_lib


@pytest.mark.parametrize("n", [1, 2, 33, 4096, 999999, 1 << 24])
def test_argmax_exact_index(emel, kern, n):
    rng = np.random.default_rng(n + 1)
    x = rng.standard_normal(n).astype(np.float32)
    got, want = device_argmax(emel, kern, x, [n, 1, 1, 1])
    assert int(got) == want


def test_argmax_ties_nan_and_f32_encoding(emel, kern):
    x = np.zeros(1 << 20, np.float32)
    x[[1000, 500000, 700000]] = 3.0  # tie -> earliest
    got, want = device_argmax(emel, kern, x, [1 << 20, 1, 1, 1])
    assert int(got) == want == 1000
    x[0] = np.nan  # NaN at element 0 pins the answer to 0
    got, want = device_argmax(emel, kern, x, [1 << 20, 1, 1, 1])
    assert int(got) == want == 0
    x[0] = 0.0
    x[5] = np.nan  # other NaNs are never selected
    got, want = device_argmax(emel, kern, x, [1 << 20, 1, 1, 1])
    assert int(got) == want == 1000
    gotf, _ = device_argmax(emel, kern, x, [1 << 20, 1, 1, 1], dtype=np.float32)
    assert gotf == np.float32(1000.0)


@pytest.mark.parametrize("n", [4096, 1 << 22])
def test_argmax_lane_chain_edges(emel, kern, n):
    """The vector walk's per-lane chains: all NaN (and so a NaN at element 0,
    which pins the answer) and all -inf give 0; behind a -inf at element 0,
    a lone late comparable value among NaNs wins; -0 and +0 tie to the
    first; NaN runs in front of the maximum are skipped."""
    cases = []
    x = np.full(n, np.nan, np.float32)
    cases.append((x.copy(), 0))
    x[0] = -np.inf
    x[n - 7] = -3.0
    cases.append((x.copy(), n - 7))
    cases.append((np.full(n, -np.inf, np.float32), 0))
    z = np.zeros(n, np.float32)
    z[0] = -0.0
    cases.append((z, 0))
    y = np.full(n, -1.0, np.float32)
    y[1: n // 2] = np.nan
    y[0] = 2.0
    y[n // 2 + 5] = 2.0  # later equal value loses to element 0
    cases.append((y, 0))
    y2 = y.copy()
    y2[0] = -9.0
    cases.append((y2, n // 2 + 5))
    for arr, expect in cases:
        got, want = device_argmax(emel, kern, arr, [n, 1, 1, 1])
        assert int(got) == want == expect, (n, int(got), want, expect)


def test_argmax_strided(emel, kern):
    rng = np.random.default_rng(8)
    x = rng.standard_normal(64 * 50 * 3).astype(np.float32)
    got, want = device_argmax(emel, kern, x, [64, 50, 1, 1], [12, 768, 38400, 38400])
    assert int(got) == want


@pytest.mark.parametrize("ne0", [4, 8, 128])
def test_contiguous_rows_walk_ties_and_nans(emel, kern, oracle_lib, ne0):
    """Padded and permuted views whose rows stay contiguous and 16-byte
    aligned take the vectorised row walk: sums match, argmax ties keep the
    earliest logical index across rows, NaN at logical element 0 pins 0."""
    rng = np.random.default_rng(ne0)
    ne = [ne0, 37, 5, 3]
    row = ne0 + 8  # padded rows
    nb = [4, 4 * row, 4 * row * 37, 4 * row * 37 * 5]
    span = sum((ne[d] - 1) * nb[d] for d in range(4)) // 4 + 1
    x = rng.standard_normal(span).astype(np.float32)

    def at(i0, i1, i2, i3):
        return (i0 * nb[0] + i1 * nb[1] + i2 * nb[2] + i3 * nb[3]) // 4

    got, want, px, po, wv = device_sum(emel, kern, x, ne, nb)
    assert oracle_lib.oracle_sum(ctypes.byref(px.oview()), ctypes.byref(wv)) == 0
    assert abs(float(got) - float(want[0])) <= 1e-5 * max(abs(float(want[0])), 1.0), (got, want)
    px.free()
    po.free()
    x[at(ne0 - 1, 30, 4, 2)] = 50.0
    x[at(0, 2, 1, 1)] = 50.0  # same value, earlier logical index
    x[at(1 % ne0, 3, 0, 0)] = np.nan
    got, want = device_argmax(emel, kern, x, ne, nb)
    assert int(got) == want == ((1 * 5 + 1) * 37 + 2) * ne0
    x[at(0, 0, 0, 0)] = np.nan
    got, want = device_argmax(emel, kern, x, ne, nb)
    assert int(got) == want == 0


def test_cfg5_whole_tensor_sum_and_argmax_full_size(emel, kern, oracle_lib):
    """2^28 elements viewed through the dims-1/2-swapped layout."""
    from emel_rs_b200 import workloads
    src0, _ = workloads.cfg5()
    ne, nb = workloads.cfg5_src0_view()
    got, want, px, po, wv = device_sum(emel, kern, src0, ne, nb)
    assert oracle_lib.oracle_sum(ctypes.byref(px.oview()), ctypes.byref(wv)) == 0
    assert abs(float(got) - float(want[0])) <= 1e-5 * max(abs(float(want[0])), 1.0), (got, want)
    px.free()
    po.free()
    got, want = device_argmax(emel, kern, src0, ne, nb)
    assert int(got) == want


def test_sharded_partials_combine_to_the_whole_tensor_answer(emel, kern, oracle_lib):
    """Split a tensor along dim 3 into 4 shards; per-shard argmax partials and
    f64 sums, combined in shard order, equal the whole-tensor result."""
    rng = np.random.default_rng(12)
    ne = [256, 16, 8, 4]
    x = rng.standard_normal(int(np.prod(ne))).astype(np.float32)
    x[123] = 50.0
    x[3 * 256 * 16 * 8 + 7] = 50.0  # tie in a later shard loses
    ctx = kern.ctx
    shard = 256 * 16 * 8
    parts, sums = [], []
    for k in range(4):
        xs = x[k * shard:(k + 1) * shard]
        px = gh.Pair(emel, ctx, xs, [256, 16, 8, 1])
        part = emel.DeviceBuffer(ctx, ctypes.sizeof(emel.CArgmaxPartial))
        dsum = emel.DeviceBuffer(ctx, 8)
        lib = emel.lib()
        assert lib.emel_cuda_argmax_partial_compute(ctx.handle, None, ctypes.byref(px.dview().c()), k * shard,
                                                    part.ptr) == 0
        assert lib.emel_cuda_sum_f64(ctx.handle, None, ctypes.byref(px.dview().c()), dsum.ptr) == 0
        hp = emel.CArgmaxPartial()
        lib.emel_cuda_memcpy_d2h(ctx.handle, None, ctypes.addressof(hp), part.ptr, ctypes.sizeof(hp))
        hs = np.zeros(1, np.float64)
        dsum.download(hs)
        parts.append((hp.value, hp.has_value, hp.index, hp.first_is_nan))
        sums.append(float(hs[0]))
        px.free()
    idx, val = emel.argmax_combine(parts)
    want_idx = ctypes.c_int64()
    ov = gh.oracle.make_view(x.ctypes.data, x.nbytes, ne, gh.contiguous_nb(ne, 4), 0)
    assert oracle_lib.oracle_argmax_index(ctypes.byref(ov), ctypes.byref(want_idx), None) == 0
    assert idx == want_idx.value == 123
    want_sum = ctypes.c_double()
    assert oracle_lib.oracle_sum_f64(ctypes.byref(ov), ctypes.byref(want_sum)) == 0
    assert abs(np.float32(sum(sums)) - np.float32(want_sum.value)) <= 1e-5 * abs(want_sum.value)
