"""World-size-2 tests of the multi-GPU host logic on CPU (gloo): dim-3
sharding, the all-gather of per-shard partials and their rank-ordered
combination.  Per-shard partials come from the oracle here (the GPU ranks
compute them with emel_cuda_sum_f64 / emel_cuda_argmax_partial_compute);
the gather and combine code is the product's."""

import ctypes
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


CASES = {
    "plain": dict(ne=[64, 8, 16, 6], plant=None, nan0=False),
    "uneven_split_tie_across_shards": dict(ne=[32, 4, 8, 5], plant=[(3, 40.0), (-7, 40.0)], nan0=False),
    "nan_at_element_zero": dict(ne=[32, 4, 8, 4], plant=[(100, 9.0)], nan0=True),
}


def make_tensor(case):
    ne = case["ne"]
    rng = np.random.default_rng(sum(ne))
    x = rng.standard_normal(int(np.prod(ne))).astype(np.float32)
    for idx, val in case["plant"] or []:
        x[idx] = val
    if case["nan0"]:
        x[0] = np.nan
    return x


def worker(rank, world, port, case_name, q):
    try:
        sys.path.insert(0, str(ROOT))
        sys.path.insert(0, str(ROOT / "oracle"))
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        import torch
        import torch.distributed as dist
        from datetime import timedelta

        import oracle
        from __graft_entry__ import load_package

        pkg = load_package()
        from emel_rs_b200 import distributed as D

        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
        case = CASES[case_name]
        ne = case["ne"]
        x = make_tensor(case)
        b, e = D.shard_bounds(ne[3], world, rank)
        plane = ne[0] * ne[1] * ne[2]
        shard = np.ascontiguousarray(x[b * plane:e * plane])
        sne = [ne[0], ne[1], ne[2], e - b]
        olib = oracle.load()
        v = oracle.host_view(shard, sne)
        s = ctypes.c_double()
        assert olib.oracle_sum_f64(ctypes.byref(v), ctypes.byref(s)) == 0
        idx, val = ctypes.c_int64(), ctypes.c_float()
        assert olib.oracle_argmax_index(ctypes.byref(v), ctypes.byref(idx), ctypes.byref(val)) == 0
        # the device partial skips NaN; emulate its (has, value, index) with the
        # first-non-NaN scan the kernel performs
        finite = ~np.isnan(shard)
        if finite.any():
            m = np.max(shard[finite])
            first = int(np.flatnonzero(shard == m)[0])
            part = (float(m), 1, b * plane + first, int(np.isnan(shard[0])))
        else:
            part = (0.0, 0, b * plane, int(np.isnan(shard[0])))
        total32, total64 = D.global_sum(torch, dist, s.value)
        gidx, gval = D.global_argmax(pkg, torch, dist, part)
        dist.destroy_process_group()
        q.put((rank, float(total32), total64, gidx))
    except Exception as exc:  # report to the parent instead of hanging it
        q.put((rank, "error", repr(exc), None))


@pytest.mark.parametrize("case_name", list(CASES))
def test_two_rank_sum_and_argmax_match_whole_tensor(case_name):
    import torch.multiprocessing as mp

    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=worker, args=(r, 2, port, case_name, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=180) for _ in procs]
    for p in procs:
        p.join(timeout=60)
    assert all(r[1] != "error" for r in results), results
    case = CASES[case_name]
    x = make_tensor(case)
    olib = oracle.load()
    v = oracle.host_view(x, case["ne"])
    out = np.zeros(1, np.float32)
    ov = oracle.host_view(out, [1, 1, 1, 1])
    assert olib.oracle_sum(ctypes.byref(v), ctypes.byref(ov)) == 0
    idx = ctypes.c_int64()
    assert olib.oracle_argmax_index(ctypes.byref(v), ctypes.byref(idx), None) == 0
    for rank, total32, total64, gidx in results:
        if not np.isnan(out[0]):
            assert abs(total32 - float(out[0])) <= 1e-5 * max(1.0, abs(float(out[0]))), (rank, total32, out[0])
        assert gidx == idx.value, (rank, gidx, idx.value)


def test_shard_bounds_cover_the_dimension_exactly():
    sys.path.insert(0, str(ROOT))
    from __graft_entry__ import load_package
    load_package()
    from emel_rs_b200 import distributed as D
    for extent in (1, 5, 8, 13):
        for world in (1, 2, 4, 8):
            spans = [D.shard_bounds(extent, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == extent
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            assert max(e - b for b, e in spans) - min(e - b for b, e in spans) <= 1
