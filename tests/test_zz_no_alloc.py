"""emel_cuda_sum_noalloc: the whole-tensor sum for callers that cannot
allocate device memory (a host application that owns all of it, or code
that must not let cudaMalloc/cudaFree synchronise the device).  It takes no
context and keeps its scratch in a static device array, so this test checks
that two calls in a row -- which reuse that array -- each return exactly the
bits the context-based emel_cuda_sum returns for the same input (both launch
the same kernel on the same grid), and that both are within the 1e-5
relative tolerance of the oracle's OpSum (reductions.rs:671-681).  The file
name sorts last so a run that stops at the first failure has already run
every other test."""

import ctypes

import numpy as np
import pytest

import gpu_helpers as gh

pytestmark = pytest.mark.gpu


def test_noalloc_sum_matches_context_sum_on_consecutive_calls(emel, oracle_lib):
    lib = emel.lib()
    ctx = emel.Context(0)  # the test allocates its buffers; the entry point does not
    rng = np.random.default_rng(2024)
    dense = rng.standard_normal(1 << 22).astype(np.float32)
    strided = rng.standard_normal(300 * 97 * 2).astype(np.float32)
    cases = [(dense, [1 << 22, 1, 1, 1], None), (strided, [300, 97, 1, 1], [8, 2400, 232800, 232800])]
    for x, ne, nb in cases:  # two consecutive calls on different inputs share the scratch
        px = gh.Pair(emel, ctx, x, ne, nb)
        want_buf = gh.Pair(emel, ctx, np.zeros(1, np.float32), [1, 1, 1, 1])
        got_buf = gh.Pair(emel, ctx, np.full(1, np.nan, np.float32), [1, 1, 1, 1])
        src, want_v, got_v = px.dview().c(), want_buf.dview().c(), got_buf.dview().c()
        assert lib.emel_cuda_sum(ctx.handle, None, ctypes.byref(src), ctypes.byref(want_v)) == 0, ctx.last_error
        assert lib.emel_cuda_sum_noalloc(None, ctypes.byref(src), ctypes.byref(got_v)) == 0
        ctx.synchronize()
        want = want_buf.download()
        got = got_buf.download()
        # same kernel, same grid, same fold order: identical bits
        gh.assert_bits_equal(got, want, f"noalloc vs context sum {ne}")
        # and the oracle's f64 accumulation rounded once to f32
        ref = np.zeros(1, np.float32)
        ov = gh.Pair(emel, ctx, ref, [1, 1, 1, 1], upload=False)
        assert oracle_lib.oracle_sum(ctypes.byref(px.oview()), ctypes.byref(ov.oview())) == 0
        r = float(ov.host[0])
        assert abs(float(got[0]) - r) <= 1e-5 * max(abs(r), 1e-3), (ne, float(got[0]), r)
        for p in (px, want_buf, got_buf, ov):
            p.free()


def test_noalloc_sum_rejects_like_the_context_sum(emel):
    lib = emel.lib()
    ctx = emel.Context(0)
    px = gh.Pair(emel, ctx, np.ones(8, np.float32))
    bad = gh.Pair(emel, ctx, np.full(2, 7.0, np.float32), [2, 1, 1, 1])
    src, dst = px.dview().c(), bad.dview().c()
    assert lib.emel_cuda_sum_noalloc(None, ctypes.byref(src), ctypes.byref(dst)) == 2  # SHAPE_MISMATCH
    ctx.synchronize()
    assert bad.download().tolist() == [7.0, 7.0]
