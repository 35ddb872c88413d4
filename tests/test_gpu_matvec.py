"""emel_cuda_mul_mat_argmax (matmul.rs OpMulMatArgmax on the device)
against the oracle: the score and the row bit-exact (one sequential
binary32 sum per row, as the reference), on the bulk-copy tile path
(k % 4 == 0) and the plain path, with ties, NaN rows and a NaN at row 0."""

import ctypes

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu
B = ctypes.byref


@pytest.fixture(scope="module")
def kern(emel):
    return emel.Kernel(device=0, synchronize=True)


def nb_of(ne):
    nb = [4]
    for d in range(1, 4):
        nb.append(nb[-1] * ne[d - 1])
    return nb


def cview(emel, buf, nbytes, ne):
    v = emel.CView()
    v.data, v.storage_bytes, v.dtype = buf.ptr, nbytes, 0
    for d in range(4):
        v.ne[d], v.nb[d] = ne[d], nb_of(ne)[d]
    return v


def run_both(emel, kern, olib, lhs, rhs, k, m):
    ctx = kern.ctx
    bl, br = emel.DeviceBuffer(ctx, lhs.nbytes), emel.DeviceBuffer(ctx, rhs.nbytes)
    bd, bi = emel.DeviceBuffer(ctx, 16), emel.DeviceBuffer(ctx, 16)
    bl.upload(lhs)
    br.upload(rhs)
    bd.upload(np.full(4, 9.0, np.float32))
    st = emel.lib().emel_cuda_mul_mat_argmax(ctx.handle, None, B(cview(emel, bl, lhs.nbytes, [k, m, 1, 1])),
                                             B(cview(emel, br, rhs.nbytes, [1, k, 1, 1])),
                                             B(cview(emel, bd, 4, [1, 1, 1, 1])), ctypes.c_void_p(bi.ptr))
    sync = emel.lib().emel_cuda_stream_synchronize(ctx.handle, None)
    got_v = bd.download(np.empty(4, np.float32))[0]
    got_i = int(bi.download(np.empty(4, np.int32))[0])
    out = np.full(1, 9.0, np.float32)
    idx = ctypes.c_int32()
    ost = olib.oracle_mul_mat_argmax(
        B(oracle.make_view(lhs.ctypes.data, lhs.nbytes, [k, m, 1, 1], nb_of([k, m, 1, 1]), 0)),
        B(oracle.make_view(rhs.ctypes.data, rhs.nbytes, [1, k, 1, 1], nb_of([1, k, 1, 1]), 0)),
        B(oracle.make_view(out.ctypes.data, out.nbytes, [1, 1, 1, 1], nb_of([1, 1, 1, 1]), 0)), B(idx))
    for b in (bl, br, bd, bi):
        b.free()
    return int(st), int(sync), ost, np.float32(got_v), got_i, out[0], idx.value


@pytest.mark.parametrize("k,m", [(4096, 1000), (4096, 20000), (128, 129), (1000, 333), (1001, 257), (3, 2)])
def test_parity(emel, kern, oracle_lib, k, m):
    rng = np.random.default_rng(k + m)
    lhs = rng.standard_normal(k * m).astype(np.float32)
    rhs = rng.standard_normal(k).astype(np.float32)
    st, sync, ost, gv, gi, wv, wi = run_both(emel, kern, oracle_lib, lhs, rhs, k, m)
    assert st == sync == ost == 0
    assert gi == wi and gv.view(np.uint32) == wv.view(np.uint32), (gi, wi, gv, wv)


@pytest.mark.parametrize("k", [4096, 1001])
def test_ties_nan_rows_and_pinned_row_zero(emel, kern, oracle_lib, k):
    rng = np.random.default_rng(k)
    m = 700
    lhs = (rng.standard_normal((m, k)) * 0.01).astype(np.float32)
    rhs = np.ones(k, np.float32)
    lhs[[300, 450, 699], :] = 0.0
    lhs[[300, 450, 699], 0] = 1000.0  # three equal best scores: the first wins
    lhs[10, 5] = np.nan               # a NaN row never wins
    st, sync, ost, gv, gi, wv, wi = run_both(emel, kern, oracle_lib, lhs.ravel(), rhs, k, m)
    assert st == sync == ost == 0 and gi == wi == 300 and gv == wv == 1000.0
    lhs[0, 3] = np.uint32(0x7fa00005).view(np.float32)  # row 0 NaN: pinned
    st, sync, ost, gv, gi, wv, wi = run_both(emel, kern, oracle_lib, lhs.ravel(), rhs, k, m)
    assert st == sync == ost == 0 and gi == wi == 0
    assert gv.view(np.uint32) == wv.view(np.uint32), (hex(gv.view(np.uint32)), hex(wv.view(np.uint32)))
