"""Back-to-back elementwise launches on one stream with no host wait in
between.  Dense elementwise kernels start reading their inputs before the
previous kernel on the stream has finished when the host's stream record
shows that kernel wrote none of those bytes; these tests chain operations
whose inputs are, and are not, the previous operation's output (whole,
partly overlapping, offset by one vector, and a different buffer), eagerly
and inside a CUDA graph, and compare every result with numpy."""

import ctypes

import numpy as np
import pytest

import gpu_helpers as gh

pytestmark = pytest.mark.gpu

N = 1 << 24  # 64 MB per f32 buffer: kernels long enough to overlap
NEG, RELU, EXP, SQR = 2, 6, 13, 64


def _view(emel, ptr, n, dtype_code=0, itemsize=4):
    v = emel.CView()
    v.data = ptr
    v.storage_bytes = n * itemsize
    for d in range(4):
        v.ne[d] = n if d == 0 else 1
        v.nb[d] = itemsize if d == 0 else n * itemsize
    v.dtype = dtype_code
    return v


def _run_chain(emel, ctx, lib, s, bufs, x, y):
    """The chain of launches; returns the numpy answers in buffer order."""
    h = s.handle
    B = ctypes.byref

    def unary(op, src, dst, n=N, so=0, do=0):
        vs = _view(emel, bufs[src].ptr + so * 4, n)
        vd = _view(emel, bufs[dst].ptr + do * 4, n)
        assert lib.emel_cuda_unary(ctx.handle, h, op, B(vs), B(vd)) == 0, ctx.last_error

    def binary(op, a, b, dst):
        va, vb, vd = (_view(emel, bufs[i].ptr, N) for i in (a, b, dst))
        assert lib.emel_cuda_binary(ctx.handle, h, op, B(va), B(vb), B(vd)) == 0, ctx.last_error

    # buffers: 0 = x, 1 = y, 2..6 results
    unary(NEG, 0, 2)            # b2 = -x
    unary(SQR, 2, 3)            # b3 = b2^2: reads the previous output
    unary(NEG, 1, 4)            # b4 = -y: independent of the previous launch
    binary(0, 3, 4, 5)          # b5 = b3 + b4: reads the previous output (b4)
    unary(RELU, 0, 6)           # b6 = relu(x): independent
    # a view that starts 4 elements into the previous output, written to b2
    # (overlaps the previous launch's output by all but 4 elements)
    unary(NEG, 6, 2, n=N - 4, so=4, do=0)
    unary(EXP, 2, 3, n=N - 4)   # b3[:N-4] = exp(b2[:N-4]): the previous output
    binary(2, 5, 0, 4)          # b4 = b5 * x: independent of b3

    def rows(buf, ne0):
        v = _view(emel, bufs[buf].ptr, N)
        v.ne[0], v.ne[1] = ne0, N // ne0
        v.nb[1] = ne0 * 4
        v.nb[2] = v.nb[3] = N * 4
        return v

    def row_vec(buf, ne0):
        return _view(emel, bufs[buf].ptr, ne0)

    # b6 = b4 + y[:4096] per row (row broadcast): reads the previous output
    assert lib.emel_cuda_broadcast_row(ctx.handle, h, 0, B(rows(4, 4096)), B(row_vec(1, 4096)),
                                       B(rows(6, 4096))) == 0, ctx.last_error
    # b2 = x * b6[:4096] per row (repeat broadcast, src1 [4096, 1]): its
    # broadcast operand is the previous output
    one = row_vec(6, 4096)
    assert lib.emel_cuda_binary_repeat(ctx.handle, h, 2, B(rows(0, 4096)), B(one), B(rows(2, 4096))) == 0, \
        ctx.last_error
    # b5 = y - b3 per row broadcast of y's first row: independent of b2
    assert lib.emel_cuda_broadcast_row(ctx.handle, h, 1, B(rows(3, 4096)), B(row_vec(1, 4096)),
                                       B(rows(5, 4096))) == 0, ctx.last_error

    # whole-tensor sum of b5, the previous launch's output (small[0]); argmax
    # of x, independent (small[1], i64)
    sv = _view(emel, bufs[7].ptr, 1)
    assert lib.emel_cuda_sum(ctx.handle, h, B(_view(emel, bufs[5].ptr, N)), B(sv)) == 0, ctx.last_error
    av = _view(emel, bufs[7].ptr + 8, 1, dtype_code=27, itemsize=8)
    assert lib.emel_cuda_argmax(ctx.handle, h, B(_view(emel, bufs[0].ptr, N)), B(av)) == 0, ctx.last_error
    # rms_norm rows of b6 (written three launches ago) into b8, then soft_max
    # rows of b8 (the previous output) into b4
    assert lib.emel_cuda_rms_norm(ctx.handle, h, B(rows(6, 4096)), B(rows(8, 4096)), ctypes.c_float(1e-6)) == 0, \
        ctx.last_error
    assert lib.emel_cuda_soft_max(ctx.handle, h, B(rows(8, 4096)), B(rows(4, 4096))) == 0, ctx.last_error

    b2 = np.empty(N, np.float32)
    b2[:N - 4] = -np.maximum(x, 0)[4:]
    b2[N - 4:] = -x[N - 4:]
    b5 = (x * x) + (-y)
    b3 = (x * x).astype(np.float32)
    b3[:N - 4] = np.exp(b2[:N - 4].astype(np.float64)).astype(np.float32)
    b4 = (b5 * x).astype(np.float32)
    b6 = (b4.reshape(-1, 4096) + y[:4096]).reshape(-1)
    b2 = (x.reshape(-1, 4096) * b6[:4096]).reshape(-1)
    b5 = (b3.reshape(-1, 4096) - y[:4096]).reshape(-1)
    r6 = b6.reshape(-1, 4096).astype(np.float64)
    b8 = r6 / np.sqrt((r6 * r6).mean(axis=1, keepdims=True) + 1e-6)
    e8 = np.exp(b8 - b8.max(axis=1, keepdims=True))
    b4 = (e8 / e8.sum(axis=1, keepdims=True)).reshape(-1)
    return {2: b2, 3: b3, 4: b4, 5: b5, 6: b6, 8: b8.reshape(-1), "argmax": int(np.argmax(x))}


@pytest.mark.parametrize("graph", [False, True])
def test_chained_launches_respect_their_inputs(emel, graph):
    ctx = emel.Context(0)
    lib = emel.lib()
    s = emel.Stream(ctx)
    rng = np.random.default_rng(41)
    x = (rng.standard_normal(N) * 2).astype(np.float32)
    y = (rng.standard_normal(N) * 2).astype(np.float32)
    bufs = [emel.DeviceBuffer(ctx, N * 4) for _ in range(9)]
    bufs[0].upload(x)
    bufs[1].upload(y)
    for r in range(3):
        # scramble the result buffers so a read that came too early shows
        for i in range(2, 9):
            bufs[i].upload(np.full(N, np.float32(1e30 + r)))
        if graph:
            g = emel.Graph(ctx, s)
            with g:
                want = _run_chain(emel, ctx, lib, s, bufs, x, y)
            g.launch()
            s.synchronize()
            g.close()
        else:
            want = _run_chain(emel, ctx, lib, s, bufs, x, y)
            s.synchronize()
        got = {i: bufs[i].download(np.empty(N, np.float32)) for i in want if i != "argmax"}
        small = bufs[7].download(np.empty(4, np.float32))
        # b3 holds exp results (within 2 ulp of the correctly rounded exp);
        # b5 = b3 - y per row is then checked bit for bit on the device's b3
        d = gh.ulp_diff_f32(got[3], want[3])
        assert int(d.max()) <= 2, f"buffer 3: {int(d.max())} ulp"
        want[5] = (got[3].reshape(-1, 4096) - y[:4096]).reshape(-1)
        for i in (2, 5, 6):
            gh.assert_bits_equal(got[i], want[i], f"buffer {i} (graph={graph}, round {r})")
        total = float(np.sum(got[5].astype(np.float64)))
        assert abs(float(small[0]) - total) <= 1e-5 * abs(total), (float(small[0]), total)
        assert int(small[2:4].view(np.int64)[0]) == want["argmax"]
        for i in (8, 4):  # rms_norm rows, then soft_max of them
            err = np.abs(got[i].astype(np.float64) - want[i]) / np.maximum(np.abs(want[i]), 1e-30)
            assert float(err[np.abs(want[i]) > 1e-30].max()) <= 1e-5, (i, float(err.max()))
    for b in bufs:
        b.free()
    s.close()


def test_eager_launch_after_a_capture_waits_for_the_kernel_before_it(emel):
    """Launches captured into a graph do not run on the stream, so the kernel
    an eager launch follows is the one before the capture: c = -x runs
    eagerly, b = relu(x) is only captured, then y = c * c must see all of c."""
    ctx = emel.Context(0)
    lib = emel.lib()
    s = emel.Stream(ctx)
    rng = np.random.default_rng(43)
    x = (rng.standard_normal(N) * 2).astype(np.float32)
    bufs = [emel.DeviceBuffer(ctx, N * 4) for _ in range(4)]
    bufs[0].upload(x)
    B = ctypes.byref
    v = [_view(emel, b.ptr, N) for b in bufs]
    for r in range(3):
        for i in (1, 2, 3):
            bufs[i].upload(np.full(N, np.float32(7e20 + r)))
        assert lib.emel_cuda_unary(ctx.handle, s.handle, NEG, B(v[0]), B(v[1])) == 0, ctx.last_error
        g = emel.Graph(ctx, s)
        with g:
            assert lib.emel_cuda_unary(ctx.handle, s.handle, RELU, B(v[0]), B(v[2])) == 0, ctx.last_error
        assert lib.emel_cuda_unary(ctx.handle, s.handle, SQR, B(v[1]), B(v[3])) == 0, ctx.last_error
        s.synchronize()
        gh.assert_bits_equal(bufs[3].download(np.empty(N, np.float32)), (-x) * (-x), f"round {r}")
        g.close()
    for b in bufs:
        b.free()
    s.close()
