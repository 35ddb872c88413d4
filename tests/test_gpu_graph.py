"""Launch capture: a sequence of entry points captured into a CUDA graph
(including forked branches joined through events) replays to the same bits
as eager dispatch, and the launch counter counts replayed kernels."""

import ctypes

import numpy as np
import pytest

import gpu_helpers as gh

pytestmark = pytest.mark.gpu


def test_graph_replay_matches_eager_with_branches(emel):
    ctx = emel.Context(0)
    lib = emel.lib()
    main, side = emel.Stream(ctx), emel.Stream(ctx)
    rng = np.random.default_rng(3)
    x = (rng.standard_normal(1 << 16) * 3).astype(np.float32)
    px = gh.Pair(emel, ctx, x)
    outs = [gh.Pair(emel, ctx, np.zeros_like(x)) for _ in range(4)]
    ops = [10, 8, 13, 65]
    xv = px.dview().c()

    def launch(stream, i):
        ov = outs[i].dview().c()
        src = np.abs(x) if ops[i] == 65 else x
        assert lib.emel_cuda_unary(ctx.handle, stream.handle, ops[i], ctypes.byref(xv), ctypes.byref(ov)) == 0

    # eager reference results
    for i in range(4):
        launch(main, i)
    main.synchronize()
    eager = [o.download() for o in outs]
    for o in outs:
        o.buf.upload(np.zeros_like(x))

    g = emel.Graph(ctx, main)
    fork, join = emel.CudaEvent(ctx), emel.CudaEvent(ctx)
    with g:
        fork.record(main.handle)
        side.wait(fork)
        launch(main, 0)
        launch(side, 1)
        launch(main, 2)
        launch(side, 3)
        join.record(side.handle)
        main.wait(join)
    before = ctx.launches
    for _ in range(3):
        g.launch()
    main.synchronize()
    assert ctx.launches - before == 12
    for o, e in zip(outs, eager):
        gh.assert_bits_equal(o.download(), e, "graph replay")
    g.close()


def test_timed_event_nodes_measure_kernels_inside_a_graph(emel):
    ctx = emel.Context(0)
    lib = emel.lib()
    s = emel.Stream(ctx)
    x = np.ones(1 << 22, np.float32)
    px, po = gh.Pair(emel, ctx, x), gh.Pair(emel, ctx, np.zeros_like(x))
    xv, ov = px.dview().c(), po.dview().c()
    e0, e1 = emel.CudaEvent(ctx), emel.CudaEvent(ctx)
    g = emel.Graph(ctx, s)
    with g:
        e0.record_timed(s.handle)
        for _ in range(4):
            assert lib.emel_cuda_unary(ctx.handle, s.handle, 6, ctypes.byref(xv), ctypes.byref(ov)) == 0
        e1.record_timed(s.handle)
    g.launch()
    s.synchronize()
    ms = e0.elapsed_ms(e1)
    assert 0.0 < ms < 50.0
