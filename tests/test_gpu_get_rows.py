"""emel_cuda_get_rows (get_rows.rs on the device) against the oracle,
through the C ABI: every source type (F32 with strided rows, F16 and BF16
with any strides, Q4_0 / Q8_0 / Q4_K blocks with random bytes -- NaN, inf
and subnormal scales included), strided indices, outer batches; bit-exact.
An index outside [0, rows) writes nothing and is reported by the next
stream synchronisation."""

import ctypes

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu
B = ctypes.byref
F32, F16, I32, Q4_0, Q8_0, Q4_K, BF16 = 0, 1, 26, 2, 8, 12, 30
FORMAT = {Q4_0: (32, 18), Q8_0: (32, 34), Q4_K: (256, 144)}


@pytest.fixture(scope="module")
def kern(emel):
    return emel.Kernel(device=0, synchronize=True)


def contiguous_nb(ne, size=4):
    nb = [size]
    for d in range(1, 4):
        nb.append(nb[-1] * ne[d - 1])
    return nb


class Dev:
    """A host array in a device buffer plus the matching C and oracle views."""

    def __init__(self, emel, ctx, host, ne, nb, code):
        self.emel, self.host = emel, np.ascontiguousarray(host)
        self.ne, self.nb, self.code = list(ne), list(nb), code
        self.buf = emel.DeviceBuffer(ctx, max(self.host.nbytes, 16))
        self.buf.upload(self.host)

    def c(self):
        v = self.emel.CView()
        v.data, v.storage_bytes, v.dtype = self.buf.ptr, self.host.nbytes, self.code
        for d in range(4):
            v.ne[d], v.nb[d] = self.ne[d], self.nb[d]
        return v

    def o(self, arr=None):
        a = self.host if arr is None else arr
        return oracle.make_view(a.ctypes.data, a.nbytes, self.ne, self.nb, self.code)

    def download(self):
        return self.buf.download(np.empty_like(self.host))

    def free(self):
        self.buf.free()


def run_both(emel, kern, olib, src, ne, nb, code, idx, idx_ne, idx_nb=None, fill=7.0):
    ctx = kern.ctx
    idx = np.asarray(idx, np.int32)
    ine = list(idx_ne) + [1]
    dne = [ne[0]] + list(idx_ne)
    ds = Dev(emel, ctx, src, ne, nb, code)
    di = Dev(emel, ctx, idx, ine, idx_nb or contiguous_nb(ine), I32)
    dd = Dev(emel, ctx, np.full(int(np.prod(dne)), fill, np.float32), dne, contiguous_nb(dne), F32)
    st = emel.lib().emel_cuda_get_rows(ctx.handle, None, B(ds.c()), B(di.c()), B(dd.c()))
    sync = emel.lib().emel_cuda_stream_synchronize(ctx.handle, None)
    got = dd.download()
    want = dd.host.copy()
    ost = olib.oracle_get_rows(B(ds.o()), B(di.o()), B(dd.o(want)))
    for d in (ds, di, dd):
        d.free()
    return int(st), int(sync), ost, got, want


def bits_equal(got, want, what):
    g, w = got.view(np.uint32), want.view(np.uint32)
    bad = np.flatnonzero(g != w)
    assert bad.size == 0, f"{what}: {bad.size} differ, first {bad[0]}: {g[bad[0]]:#x} vs {w[bad[0]]:#x}"


def test_reference_known_answers_on_the_device(emel, kern, oracle_lib):
    src = np.array([1, 2, 3, 4, 5, 6, 10, 20, 30, 40, 50, 60], np.float32)
    st, sync, ost, got, _ = run_both(emel, kern, oracle_lib, src, [3, 2, 2, 1], contiguous_nb([3, 2, 2, 1]), F32,
                                     [1, 0, 0, 1], [2, 2, 1])
    assert st == sync == ost == 0 and got.tolist() == [4, 5, 6, 1, 2, 3, 10, 20, 30, 40, 50, 60]
    q = np.frombuffer(np.uint16(0x3c00).tobytes() + bytes([0x98]) * 16 + np.uint16(0x3c00).tobytes() +
                      bytes([0xa7]) * 16, np.uint8)
    st, sync, ost, got, _ = run_both(emel, kern, oracle_lib, q, [32, 2, 1, 1], [1, 18, 36, 36], Q4_0, [1, 0],
                                     [2, 1, 1])
    assert st == sync == ost == 0
    assert got.tolist() == [-1.0] * 16 + [2.0] * 16 + [0.0] * 16 + [1.0] * 16


@pytest.mark.parametrize("case", ["contiguous", "padded_rows", "batches_strided_indices", "odd_cols"])
def test_f32_sources(emel, kern, oracle_lib, case):
    rng = np.random.default_rng(len(case))
    cols, rows = (4096, 300) if case != "odd_cols" else (1001, 77)
    outer = (2, 3) if case == "batches_strided_indices" else (1, 1)
    ne = [cols, rows, outer[0], outer[1]]
    pad = 12 if case == "padded_rows" else 0
    nb = [4, (cols + pad) * 4]
    nb += [nb[1] * rows, nb[1] * rows * outer[0]]
    span = sum((ne[d] - 1) * nb[d] for d in range(4)) // 4 + 1
    src = rng.standard_normal(span).astype(np.float32)
    src[:3] = np.array([0x7fa00001, 0xff800000, 0x00000001], np.uint32).view(np.float32)
    n_idx = 64 * outer[0] * outer[1]
    idx_ne = [64, outer[0], outer[1]]
    idx = rng.integers(0, rows, size=n_idx * 2).astype(np.int32)  # every other element used when strided
    idx_nb = [8, 8 * 64, 8 * 64 * outer[0]] if case == "batches_strided_indices" else None
    if idx_nb is None:
        idx = idx[:n_idx]
    st, sync, ost, got, want = run_both(emel, kern, oracle_lib, src, ne, nb, F32, idx, idx_ne,
                                        idx_nb and idx_nb + [idx_nb[-1] * outer[1]])
    assert st == sync == ost == 0
    bits_equal(got, want, f"f32 {case}")


@pytest.mark.parametrize("code", [F16, BF16])
@pytest.mark.parametrize("strided", [False, True])
def test_half_sources(emel, kern, oracle_lib, code, strided):
    rng = np.random.default_rng(code + strided)
    cols, rows = 2048, 129
    ne = [cols, rows, 2, 1]
    if strided:  # a transposed view: columns 2 * rows bytes apart
        nb = [2 * rows, 2, 2 * rows * cols, 2 * rows * cols * 2]
    else:
        nb = contiguous_nb(ne, 2)
    span = sum((ne[d] - 1) * nb[d] for d in range(4)) // 2 + 1
    src = rng.integers(0, 1 << 16, size=span, dtype=np.uint32).astype(np.uint16)  # every bit pattern class
    idx = rng.integers(0, rows, size=2 * 40).astype(np.int32)
    st, sync, ost, got, want = run_both(emel, kern, oracle_lib, src, ne, nb, code, idx, [40, 2, 1])
    assert st == sync == ost == 0
    bits_equal(got, want, f"half {code} strided={strided}")


@pytest.mark.parametrize("code", [Q4_0, Q8_0, Q4_K])
@pytest.mark.parametrize("cols", [64, 96, 256, 4096, 5120])
def test_quantized_sources(emel, kern, oracle_lib, code, cols):
    """Row sizes cover the 16-, 4- and 2-byte staging loads (e.g. Q4_0 rows
    of 36 and 54 bytes) and rows longer than one staged chunk."""
    if cols % FORMAT[code][0]:
        pytest.skip("not whole blocks")
    rng = np.random.default_rng(code * 7 + cols)
    bv, bb = FORMAT[code]
    rows, outer = 33, (2, 2)
    row_bytes = cols // bv * bb
    ne = [cols, rows, outer[0], outer[1]]
    nb = [1, row_bytes, row_bytes * rows, row_bytes * rows * outer[0]]
    src = rng.integers(0, 256, size=row_bytes * rows * outer[0] * outer[1], dtype=np.uint32).astype(np.uint8)
    # most scales ordinary (so the products are numbers), some random bits (NaN, inf, subnormal)
    blocks = src.reshape(-1, bb)
    ordinary = rng.random(blocks.shape[0]) < 0.9
    scales = np.where(ordinary, rng.integers(0x2000, 0x3c00, size=blocks.shape[0]), rng.integers(0, 1 << 16, size=blocks.shape[0]))
    blocks[:, 0] = scales & 0xff
    blocks[:, 1] = scales >> 8
    idx_ne = [50, outer[0], outer[1]]
    idx = rng.integers(0, rows, size=int(np.prod(idx_ne))).astype(np.int32)
    st, sync, ost, got, want = run_both(emel, kern, oracle_lib, src, ne, nb, code, idx, idx_ne)
    assert st == sync == ost == 0
    bits_equal(got, want, f"quant {code} cols={cols}")


@pytest.mark.parametrize("bad", [-1, 300])
def test_out_of_range_index_writes_nothing_and_reports_at_sync(emel, kern, oracle_lib, bad):
    rng = np.random.default_rng(1)
    src = rng.standard_normal(4096 * 300).astype(np.float32)
    idx = rng.integers(0, 300, size=64).astype(np.int32)
    idx[37] = bad
    st, sync, ost, got, want = run_both(emel, kern, oracle_lib, src, [4096, 300, 1, 1], contiguous_nb([4096, 300, 1, 1]),
                                        F32, idx, [64, 1, 1])
    assert st == 0 and sync == 9 and ost == 9
    assert np.all(got == 7.0)
    # reported once: the next synchronisation is clean
    assert emel.lib().emel_cuda_stream_synchronize(kern.ctx.handle, None) == 0


def test_rejected_views_return_synchronously(emel, kern, oracle_lib):
    src = np.ones(12, np.float32)
    # destination extents that do not match: ShapeMismatch
    ctx = kern.ctx
    ds = Dev(emel, ctx, src, [3, 4, 1, 1], contiguous_nb([3, 4, 1, 1]), F32)
    di = Dev(emel, ctx, np.zeros(2, np.int32), [2, 1, 1, 1], contiguous_nb([2, 1, 1, 1]), I32)
    dd = Dev(emel, ctx, np.full(6, 7.0, np.float32), [6, 1, 1, 1], contiguous_nb([6, 1, 1, 1]), F32)
    assert emel.lib().emel_cuda_get_rows(ctx.handle, None, B(ds.c()), B(di.c()), B(dd.c())) == 2
    # a Q8_0 view whose ne[0] is not whole blocks: InvalidView
    dq = Dev(emel, ctx, np.zeros(34, np.uint8), [31, 1, 1, 1], [1, 34, 34, 34], Q8_0)
    assert emel.lib().emel_cuda_get_rows(ctx.handle, None, B(dq.c()), B(di.c()), B(dd.c())) == 1
    assert np.all(dd.download() == 7.0)
    for d in (ds, di, dd, dq):
        d.free()


def run_bytes(emel, kern, olib, src, offset, ne, nb, idx, idx_ne, dst_offset=0, fill=7.0):
    """emel_cuda_get_rows_f32_bytes and oracle_get_rows_f32_bytes on the byte
    source `src[offset:]` (the device pointer is then `offset` bytes past a
    256-byte aligned allocation)."""
    ctx = kern.ctx
    src = np.ascontiguousarray(src, np.uint8)
    idx = np.asarray(idx, np.int32)
    ine = list(idx_ne) + [1]
    dne = [ne[0]] + list(idx_ne)
    ds = Dev(emel, ctx, src, ne, nb, F32)
    di = Dev(emel, ctx, idx, ine, contiguous_nb(ine), I32)
    n_out = int(np.prod(dne))
    dd = Dev(emel, ctx, np.full(n_out + 4, fill, np.float32), dne, contiguous_nb(dne), F32)
    sv = ds.c()
    sv.data, sv.storage_bytes = ds.buf.ptr + offset, src.nbytes - offset
    dv = dd.c()
    dv.data, dv.storage_bytes = dd.buf.ptr + 4 * dst_offset, 4 * n_out
    st = emel.lib().emel_cuda_get_rows_f32_bytes(ctx.handle, None, B(sv), B(di.c()), B(dv))
    sync = emel.lib().emel_cuda_stream_synchronize(ctx.handle, None)
    got = dd.download()[dst_offset:dst_offset + n_out]
    want = np.full(n_out, fill, np.float32)
    tail = src[offset:]
    ost = olib.oracle_get_rows_f32_bytes(B(oracle.make_view(tail.ctypes.data, tail.nbytes, ne, nb, F32)), B(di.o()),
                                         B(oracle.make_view(want.ctypes.data, want.nbytes, dne,
                                                            contiguous_nb(dne), F32)))
    for d in (ds, di, dd):
        d.free()
    return int(st), int(sync), ost, got, want


def test_f32_bytes_reference_known_answers_on_the_device(emel, kern, oracle_lib):
    src = np.zeros(17, np.uint8)
    src[0:8] = np.array([1.0, 2.0], np.float32).view(np.uint8)
    src[9:17] = np.array([3.0, 4.0], np.float32).view(np.uint8)
    st, sync, ost, got, _ = run_bytes(emel, kern, oracle_lib, src, 0, [2, 2, 1, 1], [4, 9, 18, 18], [1, 0],
                                      [2, 1, 1])
    assert st == sync == ost == 0 and got.tolist() == [3.0, 4.0, 1.0, 2.0]
    st, _, ost, got, _ = run_bytes(emel, kern, oracle_lib, src[:16], 0, [2, 2, 1, 1], [4, 9, 18, 18], [1, 0],
                                   [2, 1, 1], fill=9.0)
    assert st == ost == 1 and got.tolist() == [9.0] * 4


@pytest.mark.parametrize("offset", [0, 1, 2, 3, 5, 9, 14, 16])
@pytest.mark.parametrize("case", ["odd_row_stride", "aligned_rows", "batches", "padded_cols"])
def test_f32_bytes_sources(emel, kern, oracle_lib, offset, case):
    rng = np.random.default_rng(offset * 7 + len(case))
    if case == "odd_row_stride":
        ne, nb, idx_ne = [1001, 70, 1, 1], None, [90, 1, 1]
        nb = [4, 4 * 1001 + 3, (4 * 1001 + 3) * 70, (4 * 1001 + 3) * 70]
    elif case == "aligned_rows":
        ne, idx_ne = [4096, 40, 1, 1], [64, 1, 1]
        nb = [4, 4 * 4096 + 16, (4 * 4096 + 16) * 40, (4 * 4096 + 16) * 40]
    elif case == "batches":
        ne, idx_ne = [257, 9, 3, 2], [5, 3, 2]
        nb = [4, 4 * 257 + 1, (4 * 257 + 1) * 9 + 7, ((4 * 257 + 1) * 9 + 7) * 3 + 5]
    else:
        ne, idx_ne = [64, 33, 1, 1], [48, 1, 1]
        nb = [0, 0, 0, 0]  # implicit contiguous strides
    if nb[0] == 0:
        span = 4 * ne[0] * ne[1] * ne[2] * ne[3]
    else:
        span = sum((ne[d] - 1) * nb[d] for d in range(1, 4)) + 4 * ne[0]
    # random words, NaN payloads and signed zeros included, at any byte offset
    src = rng.integers(0, 256, size=offset + span, dtype=np.uint8)
    idx = rng.integers(0, ne[1], size=int(np.prod(idx_ne))).astype(np.int32)
    st, sync, ost, got, want = run_bytes(emel, kern, oracle_lib, src, offset, ne, nb, idx, idx_ne)
    assert st == sync == ost == 0
    bits_equal(got, want, f"f32 bytes {case} offset {offset}")


def test_f32_bytes_unaligned_destination_rows(emel, kern, oracle_lib):
    rng = np.random.default_rng(3)
    ne, nb = [512, 20, 1, 1], [4, 2051, 2051 * 20, 2051 * 20]
    src = rng.integers(0, 256, size=3 + 19 * 2051 + 2048, dtype=np.uint8)
    idx = rng.integers(0, 20, size=30).astype(np.int32)
    st, sync, ost, got, want = run_bytes(emel, kern, oracle_lib, src, 3, ne, nb, idx, [30, 1, 1], dst_offset=1)
    assert st == sync == ost == 0
    bits_equal(got, want, "f32 bytes, destination off a 16-byte boundary")


@pytest.mark.parametrize("bad", [-1, 20])
def test_f32_bytes_out_of_range_index_writes_nothing(emel, kern, oracle_lib, bad):
    rng = np.random.default_rng(9)
    ne, nb = [300, 20, 1, 1], [4, 1203, 1203 * 20, 1203 * 20]
    src = rng.integers(0, 256, size=1 + 19 * 1203 + 1200, dtype=np.uint8)
    idx = rng.integers(0, 20, size=16).astype(np.int32)
    idx[11] = bad
    st, sync, ost, got, _ = run_bytes(emel, kern, oracle_lib, src, 1, ne, nb, idx, [16, 1, 1])
    assert st == 0 and sync == 9 and ost == 9 and np.all(got == 7.0)
    assert emel.lib().emel_cuda_stream_synchronize(kern.ctx.handle, None) == 0
