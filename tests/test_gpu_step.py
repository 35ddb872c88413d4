"""The graph seam on the device: one emel-graph processor step -- rms_norm,
a repeat of the weight row, the multiply, and soft_max, as op-coded generic
requests (generic.rs:580-766) -- run through the RunKernelFn callback
emel_cuda_run_kernel (emel-graph processor/kernel_step/sm.rs:125-126), both
request by request and replayed as one captured CUDA graph, against the
oracle's restatement of the same generic loops run in the same order.
Bar: 1e-5 relative (rms_norm and soft_max accumulate in f64 / binary32 in
the generic loops' order; the soft_max exponential is the binary32 core).
A failing request stops the step with its own status and nothing after it
runs."""

import ctypes
import struct

import numpy as np
import pytest

import gpu_helpers as gh
import oracle

pytestmark = pytest.mark.gpu

RMS_NORM, REPEAT, MUL, SOFT_MAX = 24, 19, 6, 46


def build(emel, ctx, rng, width=4096, rows=96):
    x = (rng.standard_normal(width * rows) * 2.0).astype(np.float32)
    w = rng.uniform(0.5, 1.5, width).astype(np.float32)
    ne, wne = [width, rows, 1, 1], [width, 1, 1, 1]
    bufs = {k: gh.Pair(emel, ctx, a, n) for k, a, n in (("x", x, ne), ("w", w, wne))}
    for k in ("a", "W", "b", "y"):
        bufs[k] = gh.Pair(emel, ctx, np.full(width * rows, 5.0, np.float32), ne)
    eps = struct.pack("=f", 1e-6)
    spec = [(RMS_NORM, "x", None, "a", eps), (REPEAT, "w", None, "W", b""), (MUL, "a", "W", "b", b""),
            (SOFT_MAX, "b", None, "y", b"")]
    return bufs, spec


def device_events(emel, bufs, spec):
    return [emel.GenericEvent(op, src0=bufs[s0].dview(), src1=bufs[s1].dview() if s1 else None,
                              dst=bufs[d].dview(), params=prm) for op, s0, s1, d, prm in spec]


def oracle_chain(olib, bufs, spec):
    host = {k: p.host.copy() for k, p in bufs.items()}
    for op, s0, s1, d, prm in spec:
        vs = {k: oracle.make_view(host[k].ctypes.data, host[k].nbytes, bufs[k].ne, bufs[k].nb, 0)
              for k in (s0, s1, d) if k}
        r = oracle.generic_request(op, vs[s0], vs[s1] if s1 else None, None, vs[d], prm)
        assert olib.oracle_generic(ctypes.byref(r)) == 0
    return host["y"]


@pytest.mark.parametrize("capture", [False, True])
def test_step_through_run_kernel_matches_the_oracle(emel, oracle_lib, capture):
    ctx = emel.Context(0)
    stream = emel.Stream(ctx)
    bufs, spec = build(emel, ctx, np.random.default_rng(31))
    want = oracle_chain(oracle_lib, bufs, spec)
    step = emel.KernelStep(ctx, stream.handle, device_events(emel, bufs, spec), capture=capture)
    for k in range(3):  # capture: the first run records, the others replay
        bufs["y"].buf.upload(np.full_like(want, 5.0))
        ok, st = step.run(step_index=k)
        assert ok and st == emel.Status.OK, (st, ctx.last_error)
        got = bufs["y"].download()
        assert gh.max_rel_err(got, want, 1e-30) <= 1e-5, k
    assert step.runs == 3
    step.close()
    stream.close()


def test_failing_request_stops_the_step(emel):
    ctx = emel.Context(0)
    stream = emel.Stream(ctx)
    bufs, spec = build(emel, ctx, np.random.default_rng(5), width=256, rows=8)
    bad = list(spec)
    # Mul with operands of different element counts: the generic route
    # does not fit (INVALID_SHAPE), so the soft_max after it must not run
    bad[2] = (MUL, "a", "w", "b", b"")
    step = emel.KernelStep(ctx, stream.handle, device_events(emel, bufs, bad))
    ok, st = step.run()
    assert not ok and st == emel.Status.INVALID_SHAPE
    ctx.synchronize(stream.handle)
    assert np.all(bufs["y"].download() == 5.0)
    assert step.runs == 0
    step.close()
    stream.close()
