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


# ---- Q8_0 rows (matmul.rs OpMulMatArgmaxQ8_0) ---------------------------------

def q8_rows(rng, k, rows, planted=None, scale_exp=(-12, -4)):
    """Random Q8_0 rows: binary16 scales 2^e * u, quants uniform in [-127, 127]."""
    blocks = k // 32
    d = (rng.uniform(0.5, 1.0, size=(rows, blocks)) * 2.0 ** rng.integers(*scale_exp, size=(rows, blocks)))
    d = d.astype(np.float16)
    q = rng.integers(-127, 128, size=(rows, blocks, 32), dtype=np.int8)
    if planted is not None:
        q[planted] = np.abs(q[planted])
        d[planted] = np.float16(0.5)
    blob = np.empty((rows, blocks, 34), np.uint8)
    blob[:, :, :2] = d.view(np.uint8).reshape(rows, blocks, 2)
    blob[:, :, 2:] = q.view(np.uint8)
    return blob.reshape(-1)


def run_q8_both(emel, kern, olib, blob, rhs, k, rows, offset=0):
    ctx = kern.ctx
    rb = k // 32 * 34
    store = np.zeros(blob.size + offset, np.uint8)
    store[offset:] = blob
    bl, br = emel.DeviceBuffer(ctx, store.nbytes + 16), emel.DeviceBuffer(ctx, rhs.nbytes)
    bd, bi = emel.DeviceBuffer(ctx, 16), emel.DeviceBuffer(ctx, 16)
    bl.upload(store)
    br.upload(rhs)
    v = emel.CView()
    v.data, v.storage_bytes, v.dtype = bl.ptr + offset, blob.nbytes, 8
    for dim, (n, s) in enumerate(zip([k, rows, 1, 1], [1, rb, rb * rows, rb * rows])):
        v.ne[dim], v.nb[dim] = n, s
    st = emel.lib().emel_cuda_mul_mat_argmax_q8_0(ctx.handle, None, B(v), B(cview(emel, br, rhs.nbytes, [1, k, 1, 1])),
                                                  B(cview(emel, bd, 4, [1, 1, 1, 1])), ctypes.c_void_p(bi.ptr))
    sync = emel.lib().emel_cuda_stream_synchronize(ctx.handle, None)
    got_v = bd.download(np.empty(4, np.float32))[0]
    got_i = int(bi.download(np.empty(4, np.int32))[0])
    out = np.full(1, 9.0, np.float32)
    idx = ctypes.c_int32()
    ost = olib.oracle_mul_mat_argmax_q8_0(
        B(oracle.make_view(blob.ctypes.data, blob.nbytes, [k, rows, 1, 1], [1, rb, rb * rows, rb * rows], 8)),
        B(oracle.make_view(rhs.ctypes.data, rhs.nbytes, [1, k, 1, 1], nb_of([1, k, 1, 1]), 0)),
        B(oracle.make_view(out.ctypes.data, out.nbytes, [1, 1, 1, 1], nb_of([1, 1, 1, 1]), 0)), B(idx))
    for b in (bl, br, bd, bi):
        b.free()
    return int(st), int(sync), ost, np.float32(got_v), got_i, out[0], idx.value


def test_q8_0_reference_golden_vector(emel, kern, oracle_lib):
    # snapshots/parity/kernel-argmax-parity/manifest.txt case=q8_0_success
    blob = np.zeros(544, np.uint8)
    for b in range(16):
        blob[b * 34:b * 34 + 2] = (0x00, 0x3C)
        if b >= 8:
            blob[b * 34 + 2:b * 34 + 34] = 1
    st, sync, ost, gv, gi, ov, oi = run_q8_both(emel, kern, oracle_lib, blob, np.ones(256, np.float32), 256, 2)
    assert st == 0 and sync == 0 and gi == 1 and int(np.array([gv]).view(np.uint32)[0]) == 0x437FFC00


@pytest.mark.parametrize("k,rows,offset", [(32, 1, 0), (64, 7, 0), (96, 33, 2), (4096, 1000, 0), (4096, 151936, 0),
                                           (32768, 64, 0), (288, 257, 2)])
def test_q8_0_parity(emel, kern, oracle_lib, k, rows, offset):
    rng = np.random.default_rng(k + rows)
    planted = int(rng.integers(0, rows))
    blob = q8_rows(rng, k, rows, planted)
    rhs = np.abs(rng.standard_normal(k)).astype(np.float32)
    if offset:
        offset = 4  # a 4-byte aligned base that is not 16-byte aligned
    st, sync, ost, gv, gi, ov, oi = run_q8_both(emel, kern, oracle_lib, blob, rhs, k, rows, offset)
    assert st == 0 and sync == 0 and ost == 0
    assert gi == oi and np.array([gv]).view(np.uint32)[0] == np.array([ov]).view(np.uint32)[0]


def test_q8_0_special_values(emel, kern, oracle_lib):
    rng = np.random.default_rng(8)
    k, rows = 128, 50
    blob = q8_rows(rng, k, rows)
    rhs = rng.standard_normal(k).astype(np.float32)
    rhs[5] = np.nan        # quantizes to 0
    rhs[40] = np.inf       # block scale inf: every quant of that block 0 or NaN -> 0
    rhs[70:102] = 0.0      # a zero block: scale 0
    st, sync, ost, gv, gi, ov, oi = run_q8_both(emel, kern, oracle_lib, blob, rhs, k, rows)
    assert st == 0 and sync == 0 and ost == 0
    assert gi == oi and (np.isnan(gv) and np.isnan(ov) or np.array([gv]).view(np.uint32)[0] == np.array([ov]).view(np.uint32)[0])
    # equal rows: the first wins
    one = q8_rows(rng, k, 1)
    blob = np.concatenate([one] * 5)
    st, sync, ost, gv, gi, ov, oi = run_q8_both(emel, kern, oracle_lib, blob, np.ones(k, np.float32), k, 5)
    assert gi == oi == 0


# ---- Q4_0 / Q4_1 / Q5_0 rows (matmul.rs OpMulMatArgmaxQ4_0 / Q4_1 / Q5_0) -------

PACKED = {2: ("q4_0", 18), 3: ("q4_1", 20), 6: ("q5_0", 22), 8: ("q8_0", 34)}


def packed_rows(rng, code, k, rows, planted=None):
    """Random rows of the format: binary16 scales (and Q4_1 mins) 2^e * u,
    random nibbles / high bits / quants."""
    blocks = k // 32
    bb = PACKED[code][1]
    blob = rng.integers(0, 256, size=(rows, blocks, bb), dtype=np.uint8)
    d = (rng.uniform(0.5, 1.0, size=(rows, blocks)) * 2.0 ** rng.integers(-10, -4, size=(rows, blocks)))
    blob[:, :, :2] = d.astype(np.float16).view(np.uint8).reshape(rows, blocks, 2)
    if code == 3:
        m = -(rng.uniform(0.5, 1.0, size=(rows, blocks)) * 2.0 ** -6)
        blob[:, :, 2:4] = m.astype(np.float16).view(np.uint8).reshape(rows, blocks, 2)
    if planted is not None:
        blob[planted, :, :2] = np.array([0.25], np.float16).view(np.uint8)
    return blob.reshape(-1)


def run_packed_both(emel, kern, olib, code, blob, rhs, k, rows):
    ctx = kern.ctx
    suffix, bb = PACKED[code]
    rb = k // 32 * bb
    bl, br = emel.DeviceBuffer(ctx, blob.nbytes + 16), emel.DeviceBuffer(ctx, rhs.nbytes)
    bd, bi = emel.DeviceBuffer(ctx, 16), emel.DeviceBuffer(ctx, 16)
    bl.upload(blob)
    br.upload(rhs)
    v = emel.CView()
    v.data, v.storage_bytes, v.dtype = bl.ptr, blob.nbytes, code
    for dim, (n, s) in enumerate(zip([k, rows, 1, 1], [1, rb, rb * rows, rb * rows])):
        v.ne[dim], v.nb[dim] = n, s
    fn = getattr(emel.lib(), f"emel_cuda_mul_mat_argmax_{suffix}")
    st = fn(ctx.handle, None, B(v), B(cview(emel, br, rhs.nbytes, [1, k, 1, 1])), B(cview(emel, bd, 4, [1, 1, 1, 1])),
            ctypes.c_void_p(bi.ptr))
    sync = emel.lib().emel_cuda_stream_synchronize(ctx.handle, None)
    got_v = bd.download(np.empty(4, np.float32))[0]
    got_i = int(bi.download(np.empty(4, np.int32))[0])
    out = np.full(1, 9.0, np.float32)
    idx = ctypes.c_int32()
    ost = getattr(olib, f"oracle_mul_mat_argmax_{suffix}")(
        B(oracle.make_view(blob.ctypes.data, blob.nbytes, [k, rows, 1, 1], [1, rb, rb * rows, rb * rows], code)),
        B(oracle.make_view(rhs.ctypes.data, rhs.nbytes, [1, k, 1, 1], nb_of([1, k, 1, 1]), 0)),
        B(oracle.make_view(out.ctypes.data, out.nbytes, [1, 1, 1, 1], nb_of([1, 1, 1, 1]), 0)), B(idx))
    for b in (bl, br, bd, bi):
        b.free()
    return int(st), int(sync), ost, np.float32(got_v), got_i, out[0], idx.value


def test_q5_0_reference_golden_vector(emel, kern, oracle_lib):
    # snapshots/parity/kernel-argmax-parity/manifest.txt case=q5_0_success
    blob = np.zeros(352, np.uint8)
    for b in range(16):
        blob[b * 22:b * 22 + 2] = (0x00, 0x3C)
        if b >= 8:
            blob[b * 22 + 2:b * 22 + 6] = 0xFF
            blob[b * 22 + 6:b * 22 + 22] = 0x0F
    st, sync, ost, gv, gi, ov, oi = run_packed_both(emel, kern, oracle_lib, 6, blob, np.ones(256, np.float32), 256, 2)
    assert st == 0 and sync == 0 and gi == 1 and int(np.array([gv]).view(np.uint32)[0]) == 0x44EFFC40


@pytest.mark.parametrize("code", [2, 3, 6])
@pytest.mark.parametrize("k,rows", [(32, 1), (64, 9), (96, 33), (4096, 2000), (32768, 40), (288, 257)])
def test_packed_parity(emel, kern, oracle_lib, code, k, rows):
    rng = np.random.default_rng(code * 1000 + k + rows)
    planted = int(rng.integers(0, rows))
    blob = packed_rows(rng, code, k, rows, planted)
    rhs = rng.standard_normal(k).astype(np.float32)
    st, sync, ost, gv, gi, ov, oi = run_packed_both(emel, kern, oracle_lib, code, blob, rhs, k, rows)
    assert st == 0 and sync == 0 and ost == 0
    assert gi == oi and np.array([gv]).view(np.uint32)[0] == np.array([ov]).view(np.uint32)[0]


# ---- Q4_K rows (matmul.rs OpMulMatArgmaxQ4K) -----------------------------------

def q4k_rows(rng, k, rows, planted=None):
    blocks = k // 256
    blob = rng.integers(0, 256, size=(rows, blocks, 144), dtype=np.uint8)
    d = rng.uniform(0.5, 1.0, size=(rows, blocks, 2)) * 2.0 ** -8
    blob[:, :, :4] = d.astype(np.float16).view(np.uint8).reshape(rows, blocks, 4)
    if planted is not None:
        blob[planted, :, :2] = np.array([0.02], np.float16).view(np.uint8)
    return blob.reshape(-1)


def run_q4k_both(emel, kern, olib, blob, rhs, k, rows, code=12, offset=0):
    """Device and oracle answers for K-quant rows; the device copy of the
    blob starts `offset` bytes into its buffer (4: a 4-byte aligned base that
    is not 16-byte aligned, so every row takes the word-staging path)."""
    ctx = kern.ctx
    suffix, bb = {10: ("q2_k", 84), 11: ("q3_k", 110), 12: ("q4_k", 144), 14: ("q6_k", 210)}[code]
    rb = k // 256 * bb
    store = np.zeros(blob.size + offset, np.uint8)
    store[offset:] = blob
    bl, br = emel.DeviceBuffer(ctx, store.nbytes + 16), emel.DeviceBuffer(ctx, rhs.nbytes)
    bd, bi = emel.DeviceBuffer(ctx, 16), emel.DeviceBuffer(ctx, 16)
    bl.upload(store)
    br.upload(rhs)
    v = emel.CView()
    v.data, v.storage_bytes, v.dtype = bl.ptr + offset, blob.nbytes, code
    for dim, (n, s) in enumerate(zip([k, rows, 1, 1], [1, rb, rb * rows, rb * rows])):
        v.ne[dim], v.nb[dim] = n, s
    fn = getattr(emel.lib(), f"emel_cuda_mul_mat_argmax_{suffix}")
    st = fn(ctx.handle, None, B(v), B(cview(emel, br, rhs.nbytes, [1, k, 1, 1])), B(cview(emel, bd, 4, [1, 1, 1, 1])),
            ctypes.c_void_p(bi.ptr))
    sync = emel.lib().emel_cuda_stream_synchronize(ctx.handle, None)
    got_v = bd.download(np.empty(4, np.float32))[0]
    got_i = int(bi.download(np.empty(4, np.int32))[0])
    out = np.full(1, 9.0, np.float32)
    idx = ctypes.c_int32()
    ost = getattr(olib, f"oracle_mul_mat_argmax_{suffix}")(
        B(oracle.make_view(blob.ctypes.data, blob.nbytes, [k, rows, 1, 1], [1, rb, rb * rows, rb * rows], code)),
        B(oracle.make_view(rhs.ctypes.data, rhs.nbytes, [1, k, 1, 1], nb_of([1, k, 1, 1]), 0)),
        B(oracle.make_view(out.ctypes.data, out.nbytes, [1, 1, 1, 1], nb_of([1, 1, 1, 1]), 0)), B(idx))
    for b in (bl, br, bd, bi):
        b.free()
    return int(st), int(sync), ost, np.float32(got_v), got_i, out[0], idx.value


def test_q4_k_reference_golden_vector(emel, kern, oracle_lib):
    # snapshots/parity/kernel-argmax-parity/manifest.txt case=q4_k_success
    blob = np.zeros(288, np.uint8)
    blob[144:146] = (0x00, 0x3C)
    blob[148:160] = 1
    blob[160:] = 0xFF
    st, sync, ost, gv, gi, ov, oi = run_q4k_both(emel, kern, oracle_lib, blob, np.ones(256, np.float32), 256, 2)
    assert st == 0 and sync == 0 and gi == 1 and int(np.array([gv]).view(np.uint32)[0]) == 0x45700000


@pytest.mark.parametrize("k,rows", [(256, 1), (256, 33), (512, 100), (4096, 3000), (32768, 40), (4352, 65)])
def test_q4_k_parity(emel, kern, oracle_lib, k, rows):
    rng = np.random.default_rng(k + 7 * rows)
    planted = int(rng.integers(0, rows))
    blob = q4k_rows(rng, k, rows, planted)
    rhs = rng.standard_normal(k).astype(np.float32)
    rhs[5] = -abs(rhs[5]) - 10.0  # a negative maximum magnitude in block 0
    if k >= 512:
        rhs[256:512] = 0.0  # a zero block
    st, sync, ost, gv, gi, ov, oi = run_q4k_both(emel, kern, oracle_lib, blob, rhs, k, rows)
    assert st == 0 and sync == 0 and ost == 0
    assert gi == oi and np.array([gv]).view(np.uint32)[0] == np.array([ov]).view(np.uint32)[0]


# ---- Q6_K rows (matmul.rs OpMulMatArgmaxQ6K) -----------------------------------

def q6k_rows(rng, k, rows, planted=None):
    blocks = k // 256
    blob = rng.integers(0, 256, size=(rows, blocks, 210), dtype=np.uint8)
    blob[:, :, 192:208] = rng.integers(-64, 64, size=(rows, blocks, 16), dtype=np.int8).view(np.uint8)
    d = rng.uniform(0.5, 1.0, size=(rows, blocks)) * 2.0 ** -10
    blob[:, :, 208:210] = d.astype(np.float16).view(np.uint8).reshape(rows, blocks, 2)
    if planted is not None:
        blob[planted, :, 208:210] = np.array([0.01], np.float16).view(np.uint8)
        blob[planted, :, 192:208] = 60
    return blob.reshape(-1)


def test_q6_k_reference_golden_vector(emel, kern, oracle_lib):
    # snapshots/parity/kernel-argmax-parity/manifest.txt case=q6_k_success
    blob = np.zeros(420, np.uint8)
    blob[210:338] = 0xFF
    blob[338:402] = 0xFF
    blob[402:418] = 1
    blob[418:420] = (0x00, 0x3C)
    st, sync, ost, gv, gi, ov, oi = run_q4k_both(emel, kern, oracle_lib, blob, np.ones(256, np.float32), 256, 2, 14)
    assert st == 0 and sync == 0 and gi == 1 and int(np.array([gv]).view(np.uint32)[0]) == 0x45F80000


@pytest.mark.parametrize("k,rows", [(256, 1), (256, 33), (512, 100), (4096, 3000), (32768, 40), (4352, 65)])
def test_q6_k_parity(emel, kern, oracle_lib, k, rows):
    rng = np.random.default_rng(k + 11 * rows)
    planted = int(rng.integers(0, rows))
    blob = q6k_rows(rng, k, rows, planted)
    rhs = rng.standard_normal(k).astype(np.float32)
    st, sync, ost, gv, gi, ov, oi = run_q4k_both(emel, kern, oracle_lib, blob, rhs, k, rows, 14)
    assert st == 0 and sync == 0 and ost == 0
    assert gi == oi and np.array([gv]).view(np.uint32)[0] == np.array([ov]).view(np.uint32)[0]


# ---- Q2_K / Q3_K rows (matmul.rs OpMulMatArgmaxQ2K / Q3K) ----------------------

def q23k_rows(rng, code, k, rows, planted=None):
    blocks = k // 256
    bb, dpos = (84, 80) if code == 10 else (110, 108)
    blob = rng.integers(0, 256, size=(rows, blocks, bb), dtype=np.uint8)
    nd = 2 if code == 10 else 1
    d = rng.uniform(0.5, 1.0, size=(rows, blocks, nd)) * 2.0 ** -9
    blob[:, :, dpos:dpos + 2 * nd] = d.astype(np.float16).view(np.uint8).reshape(rows, blocks, 2 * nd)
    if planted is not None:
        blob[planted, :, dpos:dpos + 2] = np.array([0.05], np.float16).view(np.uint8)
    return blob.reshape(-1)


def test_q2_k_q3_k_reference_golden_vectors(emel, kern, oracle_lib):
    # kernel-argmax-parity manifest: q2_k_success (row 1, 0x46340000),
    # q3_k_success (row 0, +0)
    q2 = np.zeros(168, np.uint8)
    q2[164:166] = (0x00, 0x3C)
    q2[84:164] = 0xFF
    st, sync, ost, gv, gi, ov, oi = run_q4k_both(emel, kern, oracle_lib, q2, np.ones(256, np.float32), 256, 2, 10)
    assert st == 0 and sync == 0 and gi == 1 and int(np.array([gv]).view(np.uint32)[0]) == 0x46340000
    q3 = np.zeros(220, np.uint8)
    q3[110:206] = 0xFF
    q3[206:218] = 0x21
    q3[218:220] = (0x00, 0x3C)
    st, sync, ost, gv, gi, ov, oi = run_q4k_both(emel, kern, oracle_lib, q3, np.ones(256, np.float32), 256, 2, 11)
    assert st == 0 and sync == 0 and gi == 0 and int(np.array([gv]).view(np.uint32)[0]) == 0


@pytest.mark.parametrize("code", [10, 11])
@pytest.mark.parametrize("k,rows", [(256, 1), (256, 33), (512, 100), (4096, 3000), (32768, 40), (4352, 65)])
def test_q2_k_q3_k_parity(emel, kern, oracle_lib, code, k, rows):
    rng = np.random.default_rng(code * 100 + k + rows)
    planted = int(rng.integers(0, rows))
    blob = q23k_rows(rng, code, k, rows, planted)
    rhs = rng.standard_normal(k).astype(np.float32)
    st, sync, ost, gv, gi, ov, oi = run_q4k_both(emel, kern, oracle_lib, blob, rhs, k, rows, code)
    assert st == 0 and sync == 0 and ost == 0
    assert gi == oi and np.array([gv]).view(np.uint32)[0] == np.array([ov]).view(np.uint32)[0]


# ---- K-quant staging paths and the grid-stride group loop ----------------------

KQ_ROWS = {10: lambda rng, k, rows, pl: q23k_rows(rng, 10, k, rows, pl),
           11: lambda rng, k, rows, pl: q23k_rows(rng, 11, k, rows, pl),
           12: q4k_rows, 14: q6k_rows}


@pytest.mark.parametrize("code", [10, 11, 12, 14])
@pytest.mark.parametrize("k,rows", [(256, 33), (4096, 700), (32768, 40)])
def test_k_quant_unaligned_base_parity(emel, kern, oracle_lib, code, k, rows):
    """A 4-byte aligned, not 16-byte aligned lhs: Q4_K (144-byte blocks) and
    Q6_K rows are otherwise always 16-byte aligned and would only take the
    16-byte chunk staging; here every format stages aligned words."""
    rng = np.random.default_rng(code * 31 + k + rows)
    planted = int(rng.integers(0, rows))
    blob = KQ_ROWS[code](rng, k, rows, planted)
    rhs = rng.standard_normal(k).astype(np.float32)
    st, sync, ost, gv, gi, ov, oi = run_q4k_both(emel, kern, oracle_lib, blob, rhs, k, rows, code, offset=4)
    assert st == 0 and sync == 0 and ost == 0
    assert gi == oi and np.array([gv]).view(np.uint32)[0] == np.array([ov]).view(np.uint32)[0]


@pytest.mark.parametrize("code", [10, 12])
@pytest.mark.parametrize("offset", [0, 4])
def test_k_quant_rows_beyond_one_wave(emel, kern, oracle_lib, code, offset):
    """500,000 rows: more than one resident wave can hold (148 SMs x at most
    2048 threads x one row per lane), so warps loop to a second group of 32
    rows and reuse both staging buffers.  The planted maximum sits in the
    last group."""
    k, rows = 256, 500_000
    rng = np.random.default_rng(4242 + code + offset)
    planted = rows - 17
    blob = KQ_ROWS[code](rng, k, rows, planted)
    rhs = np.abs(rng.standard_normal(k)).astype(np.float32)
    st, sync, ost, gv, gi, ov, oi = run_q4k_both(emel, kern, oracle_lib, blob, rhs, k, rows, code, offset=offset)
    assert st == 0 and sync == 0 and ost == 0
    assert gi == oi and np.array([gv]).view(np.uint32)[0] == np.array([ov]).view(np.uint32)[0]


@pytest.mark.parametrize("code", [10, 11, 12, 14])
@pytest.mark.parametrize("rows,planted", [(151936, 151935), (20001, 0), (20001, 10000)])
def test_k_quant_balanced_vocabulary_rows(emel, kern, oracle_lib, code, rows, planted):
    """k = 4096 on a 16-byte aligned base takes the two-rows-per-warp kernel
    (one bulk copy per two rows, sixteen lanes per row, the reference's fold
    as nine chains): the vocabulary's 151,936 rows with the maximum in the
    last row, an odd row count whose last unit holds one row, and maxima
    at row 0 and mid-tensor, bit-exact against the oracle."""
    k = 4096
    rng = np.random.default_rng(777 + code + rows + planted)
    blob = KQ_ROWS[code](rng, k, rows, planted)
    rhs = rng.standard_normal(k).astype(np.float32)
    st, sync, ost, gv, gi, ov, oi = run_q4k_both(emel, kern, oracle_lib, blob, rhs, k, rows, code, offset=0)
    assert st == 0 and sync == 0 and ost == 0
    assert gi == oi and np.array([gv]).view(np.uint32)[0] == np.array([ov]).view(np.uint32)[0]
