"""emel_cuda_diag / emel_cuda_diag_mask (diag.rs on the device) against the
oracle, through the C ABI: bit-exact (copies and constants only), on the
16-byte vector path (side % 4 == 0), the element path, in place, and with
NaN payloads; guards write nothing."""

import ctypes

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def kern(emel):
    return emel.Kernel(device=0, synchronize=True)


def dev(emel, ctx, host):
    b = emel.DeviceBuffer(ctx, max(host.nbytes, 16))
    b.upload(host)
    return b


@pytest.mark.parametrize("side", [1, 2, 3, 8, 37, 1024, 4096])
def test_diag(emel, kern, oracle_lib, side):
    rng = np.random.default_rng(side)
    x = rng.standard_normal(side).astype(np.float32)
    x.view(np.uint32)[0] = 0x7FA00003
    bi = dev(emel, kern.ctx, x)
    bo = dev(emel, kern.ctx, np.full(side * side, 5.0, np.float32))
    assert kern.process_event(emel.OpDiag(bi.ptr, side, bo.ptr, side * side)) == emel.Status.OK
    got = bo.download(np.empty(side * side, np.float32))
    want = np.full(side * side, 5.0, np.float32)
    assert oracle_lib.oracle_diag(x.ctypes.data, side, want.ctypes.data, side * side) == 0
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    bi.free(), bo.free()


@pytest.mark.parametrize("side,n_past", [(1, 0), (2, 0), (5, 1), (8, 0), (64, 3), (100, 7), (4096, 0),
                                         (4096, 3584), (3000, 5000)])
@pytest.mark.parametrize("mode", [0, 1])
def test_diag_mask(emel, kern, oracle_lib, side, n_past, mode):
    rng = np.random.default_rng(side * 31 + n_past)
    x = rng.standard_normal(side * side).astype(np.float32)
    x.view(np.uint32)[x.size // 2] = 0xFFC12345
    bi = dev(emel, kern.ctx, x)
    bo = dev(emel, kern.ctx, np.zeros(side * side, np.float32))
    cls = emel.OpDiagMaskInf if mode == 0 else emel.OpDiagMaskZero
    assert kern.process_event(cls(bi.ptr, side * side, bo.ptr, side * side, n_past)) == emel.Status.OK
    got = bo.download(np.empty_like(x))
    want = np.zeros_like(x)
    assert oracle_lib.oracle_diag_mask(mode, x.ctypes.data, x.size, want.ctypes.data, x.size, n_past) == 0
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    # in place
    assert kern.process_event(cls(bi.ptr, side * side, bi.ptr, side * side, n_past)) == emel.Status.OK
    assert np.array_equal(bi.download(np.empty_like(x)).view(np.uint32), want.view(np.uint32))
    bi.free(), bo.free()


def test_guards_write_nothing(emel, kern):
    x = np.arange(9, dtype=np.float32)
    bi = dev(emel, kern.ctx, x)
    bo = dev(emel, kern.ctx, np.full(9, 7.0, np.float32))
    S = emel.Status
    assert kern.process_event(emel.OpDiagMaskInf(bi.ptr, 9, bo.ptr, 9, -1)) == S.INVALID_SHAPE
    assert kern.process_event(emel.OpDiagMaskZero(bi.ptr, 8, bo.ptr, 8, 0)) == S.INVALID_SHAPE
    assert kern.process_event(emel.OpDiag(bi.ptr, 3, bo.ptr, 8)) == S.INVALID_SHAPE
    assert kern.process_event(emel.OpDiagMaskInf(bi.ptr, 9, bi.ptr + 4, 9, 0)) == S.INVALID_ARGUMENT
    assert kern.process_event(emel.OpDiag(bi.ptr, 3, bi.ptr, 9)) == S.INVALID_ARGUMENT
    assert bo.download(np.empty(9, np.float32)).tolist() == [7.0] * 9
    bi.free(), bo.free()


def causal_case(emel, kern, oracle_lib, x, side, n_past, in_place=False):
    bi = dev(emel, kern.ctx, x)
    bo = bi if in_place else dev(emel, kern.ctx, np.full(side * side, 7.0, np.float32))
    st = kern.process_event(emel.SoftMaxDiagMaskInf(bi.ptr, side * side, bo.ptr, side * side, n_past))
    got = bo.download(np.empty(side * side, np.float32))
    want = np.full(side * side, 7.0, np.float32)
    scratch = np.zeros(side * side, np.float32)
    ost = oracle_lib.oracle_soft_max_diag_mask_inf(x.ctypes.data, x.size, want.ctypes.data, want.size, n_past,
                                                   scratch.ctypes.data)
    bi.free()
    if not in_place:
        bo.free()
    return int(st), ost, got, want


def close_softmax(got, want):
    """soft_max bar: NaN positions identical, else within 1e-5 relative of
    the row's largest magnitude (binary64 sums, only their order differs)."""
    assert np.array_equal(np.isnan(got), np.isnan(want))
    ok = ~np.isnan(want)
    assert np.array_equal(got[ok] == 0, want[ok] == 0)
    assert np.max(np.abs(got[ok] - want[ok]), initial=0.0) <= 1e-5 * max(1.0, float(np.max(np.abs(want[ok]), initial=0)))


@pytest.mark.parametrize("side,n_past", [(1, 0), (2, 0), (7, 2), (64, 0), (300, 17), (4096, 0), (1000, 5000)])
def test_softmax_causal(emel, kern, oracle_lib, side, n_past):
    rng = np.random.default_rng(side + n_past)
    x = (rng.standard_normal(side * side) * 4).astype(np.float32)
    st, ost, got, want = causal_case(emel, kern, oracle_lib, x, side, n_past)
    assert st == 0 and ost == 0
    close_softmax(got, want)
    # bit-for-bit the masked columns, and in place
    st, ost, got2, _ = causal_case(emel, kern, oracle_lib, x, side, n_past, in_place=True)
    assert st == 0 and np.array_equal(got.view(np.uint32), got2.view(np.uint32))


def test_softmax_causal_special_rows(emel, kern, oracle_lib):
    side = 40
    rng = np.random.default_rng(3)
    x = rng.standard_normal(side * side).astype(np.float32)
    x[3 * side + 1] = np.nan              # NaN in a kept column
    x[5 * side + 0] = np.nan              # NaN at column 0 pins the maximum
    x[7 * side + 0] = -np.inf             # row 7: first kept value -inf, others finite
    x[8 * side:8 * side + 9] = -np.inf    # row 8: every kept value -inf
    x[9 * side + 2] = np.inf              # an infinite maximum
    x[10 * side + 20] = np.nan            # NaN in a masked column: masked to -inf, no effect
    st, ost, got, want = causal_case(emel, kern, oracle_lib, x, side, 0)
    assert st == 0 and ost == 0
    close_softmax(got, want)
    assert np.isnan(want[3 * side]) and not np.isnan(want[10 * side])
