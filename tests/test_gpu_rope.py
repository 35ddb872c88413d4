"""emel_cuda_rope (rope.rs OpRope on the device) against the oracle's
correctly-rounded build, through the C ABI.

cos / sin / exp are libm calls in the reference: both sides evaluate them in
binary64 and round once, so they agree except for rare double-rounding
ties; a differing cos or sin then moves the whole (position, pair) column of
rows by an ulp or two.  Bar: at least 99.99 % of elements bit-identical, the
rest within 2e-6 relative (of the row's largest magnitude), NaN positions
identical, copied columns bit-identical."""

import ctypes

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu
B = ctypes.byref
F32, I32 = 0, 26
NORM, NEOX, TIMESTEP = 0, 2, 4


@pytest.fixture(scope="module")
def kern(emel):
    return emel.Kernel(device=0, synchronize=True)


@pytest.fixture(scope="module")
def cr_lib():
    return oracle.load(cr=True)


def nb_of(ne, size=4):
    nb = [size]
    for d in range(1, 4):
        nb.append(nb[-1] * ne[d - 1])
    return nb


class Dev:
    def __init__(self, emel, ctx, host, ne, nb, code):
        self.emel, self.host, self.ne, self.nb, self.code = emel, np.ascontiguousarray(host), list(ne), list(nb), code
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


def run(emel, kern, olib, x, ne, pos, mode, n_dims, src_nb=None, dst_nb=None, dst_ne=None, fill=9.0, **kw):
    ctx = kern.ctx
    pr = dict(n_dims=n_dims, mode=mode, freq_base=10000.0, freq_scale=1.0, ext_factor=0.0, attn_factor=1.0)
    pr.update(kw)
    dne = dst_ne or ne
    dnb = dst_nb or nb_of(dne)
    dspan = sum((dne[d] - 1) * dnb[d] for d in range(4)) // 4 + 1
    ds = Dev(emel, ctx, np.asarray(x, np.float32), ne, src_nb or nb_of(ne), F32)
    pos = np.asarray(pos, np.int32)
    dp = Dev(emel, ctx, pos, [pos.size, 1, 1, 1], nb_of([pos.size, 1, 1, 1]), I32)
    dd = Dev(emel, ctx, np.full(dspan, fill, np.float32), dne, dnb, F32)
    st = kern.process_event(emel.OpRope(ds.c(), dp.c(), dd.c(), pr))
    got = dd.buf.download(np.empty_like(dd.host))
    want = dd.host.copy()
    ost = olib.oracle_rope(B(ds.o()), B(dp.o()), B(dd.o(want)), B(oracle.RopeParams(**pr)))
    for d in (ds, dp, dd):
        d.buf.free()
    return int(st), ost, got, want


def close(got, want, what, scale):
    nan = np.isnan(want)
    assert np.array_equal(np.isnan(got), nan), f"{what}: NaN positions"
    g, w = got[~nan], want[~nan]
    same = g.view(np.uint32) == w.view(np.uint32)
    assert same.mean() >= 0.9999, f"{what}: only {same.mean():.6f} bit-identical"
    err = np.abs(g.astype(np.float64) - w.astype(np.float64)).max(initial=0.0)
    assert err <= 2e-6 * scale, f"{what}: max difference {err}"


def test_reference_known_answers_on_the_device(emel, kern, cr_lib):
    x = np.arange(1, 13, dtype=np.float32)
    st, ost, got, want = run(emel, kern, cr_lib, x, [6, 1, 2, 1], [1, 2], NORM, 4)
    assert st == ost == 0
    close(got, want, "norm [6,1,2,1]", 12.0)
    st, ost, got, want = run(emel, kern, cr_lib, x[:4], [4, 1, 1, 1], [1], TIMESTEP, 4)
    assert st == ost == 0
    close(got, want, "timestep [4,1,1,1]", 4.0)


@pytest.mark.parametrize("mode,n_dims", [(NEOX, 128), (NORM, 128), (NORM, 64), (NEOX, 96)])
def test_llm_shapes(emel, kern, cr_lib, mode, n_dims):
    rng = np.random.default_rng(mode * 1000 + n_dims)
    cols, heads, npos = 128, 32, 257
    x = rng.standard_normal(cols * heads * npos * 2).astype(np.float32)
    x[5] = np.nan
    x[cols * 3 + 1] = np.uint32(0x7fa00003).view(np.float32)
    pos = rng.integers(0, 32768, size=npos).astype(np.int32)
    st, ost, got, want = run(emel, kern, cr_lib, x, [cols, heads, npos, 2], pos, mode, n_dims,
                             freq_scale=0.25, attn_factor=1.1)
    assert st == ost == 0
    close(got, want, f"mode {mode} n_dims {n_dims}", 8.0)
    tail = got.reshape(-1, cols)[:, n_dims:]
    assert np.array_equal(tail.view(np.uint32), want.reshape(-1, cols)[:, n_dims:].view(np.uint32))


def test_strided_views(emel, kern, cr_lib):
    """src stored [128, positions, heads] read as [128, heads, positions];
    dst rows padded by 8 floats."""
    rng = np.random.default_rng(4)
    cols, heads, npos = 128, 8, 33
    x = rng.standard_normal(cols * heads * npos).astype(np.float32)
    src_nb = [4, 4 * cols * npos, 4 * cols, 4 * cols * npos * heads]
    dst_nb = [4, 4 * (cols + 8)]
    dst_nb += [dst_nb[1] * heads, dst_nb[1] * heads * npos]
    pos = rng.integers(-100, 5000, size=npos).astype(np.int32)
    st, ost, got, want = run(emel, kern, cr_lib, x, [cols, heads, npos, 1], pos, NEOX, 128, src_nb=src_nb,
                             dst_nb=dst_nb)
    assert st == ost == 0
    close(got, want, "strided neox", 6.0)


def test_timestep_mode(emel, kern, cr_lib):
    rng = np.random.default_rng(5)
    x = rng.standard_normal(256 * 4 * 9).astype(np.float32)
    pos = rng.integers(0, 1000, size=9).astype(np.int32)
    st, ost, got, want = run(emel, kern, cr_lib, x, [256, 4, 9, 1], pos, TIMESTEP, 256, freq_scale=0.5)
    assert st == ost == 0
    close(got, want, "timestep", 6.0)


def test_more_pairs_than_one_table_chunk(emel, kern, cr_lib):
    """n_dims 8192: 4096 pairs, two shared-memory chunks, one theta chain."""
    rng = np.random.default_rng(6)
    x = rng.standard_normal(8192 * 2 * 3).astype(np.float32)
    st, ost, got, want = run(emel, kern, cr_lib, x, [8192, 2, 3, 1], [7, 300, 20000], NORM, 8192, freq_base=500000.0)
    assert st == ost == 0
    close(got, want, "long rows", 6.0)


@pytest.mark.parametrize("kw,ne_dst,status", [
    (dict(mode=99), None, 11), (dict(freq_base=0.0), None, 3), (dict(ext_factor=0.5), None, 3),
    (dict(n_dims=3), None, 3), (dict(), [4, 2, 1, 1], 2), (dict(mode=99), [4, 2, 1, 1], 2),
])
def test_rejections_write_nothing(emel, kern, cr_lib, kw, ne_dst, status):
    mode = kw.pop("mode", NORM)
    n_dims = kw.pop("n_dims", 4)
    x = np.arange(8, dtype=np.float32)
    st, ost, got, _ = run(emel, kern, cr_lib, x, [8, 1, 1, 1], [3], mode, n_dims, dst_ne=ne_dst, **kw)
    assert st == ost == status
    assert np.all(got == 9.0)
