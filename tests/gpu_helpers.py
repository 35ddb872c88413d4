"""Helpers shared by the GPU parity tests: device buffers through the C ABI,
oracle calls on host copies, and the comparison rules."""

import ctypes

import numpy as np

import oracle

CODE = {np.dtype(np.float32): 0, np.dtype(np.float16): 1, np.dtype(np.int32): 26, np.dtype(np.int64): 27}


def contiguous_nb(ne, itemsize):
    nb = [itemsize]
    for d in range(1, 4):
        nb.append(nb[-1] * ne[d - 1])
    return nb


def ne_of(arr):
    ne = list(arr.shape)[::-1]
    return (ne + [1] * 4)[:4]


class Pair:
    """One host array mirrored in a device buffer, with one layout used for
    both the device view and the oracle view."""

    def __init__(self, pkg, ctx, host, ne=None, nb=None, upload=True):
        self.pkg = pkg
        self.host = np.ascontiguousarray(host)
        self.ne = list(ne) if ne is not None else ne_of(self.host)
        self.nb = list(nb) if nb is not None else contiguous_nb(self.ne, self.host.itemsize)
        self.code = CODE[self.host.dtype]
        self.buf = pkg.DeviceBuffer(ctx, self.host.nbytes)
        if upload:
            self.buf.upload(self.host)

    def dview(self):
        return self.pkg.TensorView(self.buf.ptr, self.host.nbytes,
                                   self.pkg.Layout.new(self.code, self.ne, self.nb))

    def oview(self):
        return oracle.make_view(self.host.ctypes.data, self.host.nbytes, self.ne, self.nb, self.code)

    def download(self):
        return self.buf.download(np.empty_like(self.host))

    def free(self):
        self.buf.free()


def oracle_call(fn, *args):
    """Calls an oracle function, passing View structs by reference."""
    conv = [ctypes.byref(a) if isinstance(a, oracle.View) else a for a in args]
    return fn(*conv)


def ulp_diff_f32(a, b):
    ai = a.view(np.int32).astype(np.int64)
    bi = b.view(np.int32).astype(np.int64)
    ai = np.where(ai < 0, -(ai & 0x7FFFFFFF), ai)
    bi = np.where(bi < 0, -(bi & 0x7FFFFFFF), bi)
    return np.abs(ai - bi)


def ulp_diff_f16(a, b):
    ai = a.view(np.int16).astype(np.int64)
    bi = b.view(np.int16).astype(np.int64)
    ai = np.where(ai < 0, -(ai & 0x7FFF), ai)
    bi = np.where(bi < 0, -(bi & 0x7FFF), bi)
    return np.abs(ai - bi)


def assert_bits_equal(got, want, what):
    g = got.view(np.uint16 if got.dtype == np.float16 else np.uint32)
    w = want.view(np.uint16 if want.dtype == np.float16 else np.uint32)
    bad = np.flatnonzero(g.ravel() != w.ravel())
    assert bad.size == 0, (f"{what}: {bad.size} of {g.size} elements differ; first at {bad[0]}: "
                           f"got {g.ravel()[bad[0]]:#x} want {w.ravel()[bad[0]]:#x}")


def max_rel_err(got, want, floor):
    g = got.astype(np.float64).ravel()
    w = want.astype(np.float64).ravel()
    return float(np.max(np.abs(g - w) / np.maximum(np.abs(w), floor))) if g.size else 0.0
