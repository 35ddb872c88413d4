"""Multi-GPU sharded path on real devices: one process per GPU, NCCL.

Each rank holds the dim-3 slices [b, e) of the tensor (config 5's permuted
view, or a small contiguous case), runs the repeat broadcast on its shard
(checked bit-exactly against the oracle for that shard), computes its sum
and argmax partials on the device (emel_cuda_sum_f64,
emel_cuda_argmax_partial_compute), all-gathers them over NCCL and combines
them in rank order.  The parent checks every rank's combined answer against
the oracle's whole-tensor OpSum / OpArgmax.  Skipped unless the process
sees at least `world` GPUs."""

import ctypes
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent

pytestmark = pytest.mark.gpu

SMALL = {
    "uneven_split_tie_across_shards": dict(ne=[32, 4, 8, 5], plant=[(3, 40.0), (-7, 40.0)], nan0=False),
    "nan_at_element_zero": dict(ne=[32, 4, 8, 4], plant=[(100, 9.0)], nan0=True),
    # one slice per rank at 8 GPUs; the tie's later copy sits in the last slice
    "eight_slices_tie_first_and_last": dict(ne=[32, 4, 8, 8], plant=[(5, 50.0), (-3, 50.0), (6000, 49.0)],
                                            nan0=False),
}


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def gpu_count():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def small_tensor(case):
    ne = case["ne"]
    rng = np.random.default_rng(sum(ne))
    x = rng.standard_normal(int(np.prod(ne))).astype(np.float32)
    for idx, val in case["plant"]:
        x[idx] = val
    if case["nan0"]:
        x[0] = np.nan
    return x


def cfg5_slices(W, begin, end):
    """Storage of dim-3 slices [begin, end) of config 5's src0, and src1."""
    parts = []
    src1 = None
    for j in range(begin, end):
        s0, src1 = W.cfg5(ne3=1, shard=j)
        parts.append(s0)
    return np.concatenate(parts, axis=0), src1


def worker(rank, world, port, case_name, q):
    try:
        sys.path.insert(0, str(ROOT))
        sys.path.insert(0, str(ROOT / "oracle"))
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        from datetime import timedelta

        import torch
        import torch.distributed as dist

        import oracle
        from __graft_entry__ import load_package

        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                                device_id=dev)
        pkg = load_package()
        from emel_rs_b200 import distributed as D
        from emel_rs_b200 import workloads as W

        lib = pkg.lib()
        ctx = pkg.Context(rank)
        olib = oracle.load()
        repeat_ok = None
        if case_name == "cfg5":
            b, e = D.shard_bounds(W.CFG5_NE[3], world, rank)
            s0, s1 = cfg5_slices(W, b, e)
            ne, nb = W.cfg5_src0_view(ne3=e - b)
            plane = ne[0] * ne[1] * ne[2]
            t0 = torch.from_numpy(s0).to(dev)
            t1 = torch.from_numpy(s1).to(dev)
            td = torch.empty_like(t0)
            v0, v1, vd = pkg.CView(), pkg.CView(), pkg.CView()
            for v, t, vne, vnb in ((v0, t0, ne, nb), (v1, t1, [128, 1, 8192, 1], None),
                                   (vd, td, ne, None)):
                v.data = t.data_ptr()
                v.storage_bytes = t.numel() * 4
                vnb = vnb or pkg.contiguous_nb(vne)
                for d in range(4):
                    v.ne[d], v.nb[d] = vne[d], vnb[d]
                v.dtype = 0
            torch.cuda.synchronize()
            st = lib.emel_cuda_binary_repeat(ctx.handle, None, 2, ctypes.byref(v0), ctypes.byref(v1), ctypes.byref(vd))
            assert st == 0, ctx.last_error
            ctx.synchronize()
            got = td.cpu().numpy()
            want = np.empty_like(s0)
            o0 = oracle.host_view(s0, ne, nb)
            o1 = oracle.host_view(s1, [128, 1, 8192, 1])
            od = oracle.host_view(want, ne)
            assert olib.oracle_binary_repeat(2, ctypes.byref(o0), ctypes.byref(o1), ctypes.byref(od)) == 0
            repeat_ok = bool(np.array_equal(got.view(np.uint32), want.view(np.uint32)))
            src_view = v0
        else:
            case = SMALL[case_name]
            ne = case["ne"]
            x = small_tensor(case)
            b, e = D.shard_bounds(ne[3], world, rank)
            plane = ne[0] * ne[1] * ne[2]
            shard = np.ascontiguousarray(x[b * plane:e * plane])
            t0 = torch.from_numpy(shard).to(dev)
            src_view = pkg.CView()
            src_view.data = t0.data_ptr()
            src_view.storage_bytes = t0.numel() * 4
            sne = [ne[0], ne[1], ne[2], e - b]
            snb = pkg.contiguous_nb(sne)
            for d in range(4):
                src_view.ne[d], src_view.nb[d] = sne[d], snb[d]
            src_view.dtype = 0
            torch.cuda.synchronize()
        acc = torch.empty(1, dtype=torch.float64, device=dev)
        part = torch.empty(24, dtype=torch.uint8, device=dev)
        st = lib.emel_cuda_sum_f64(ctx.handle, None, ctypes.byref(src_view), ctypes.c_void_p(acc.data_ptr()))
        assert st == 0, ctx.last_error
        st = lib.emel_cuda_argmax_partial_compute(ctx.handle, None, ctypes.byref(src_view), b * plane,
                                                  ctypes.c_void_p(part.data_ptr()))
        assert st == 0, ctx.last_error
        ctx.synchronize()
        local_sum = float(acc.cpu().item())
        local_part = D.read_partial(pkg, ctx, part.data_ptr())
        total32, total64 = D.global_sum(torch, dist, local_sum, device=dev)
        gidx, gval = D.global_argmax(pkg, torch, dist, local_part, device=dev)
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, float(total32), total64, gidx, repeat_ok))
    except Exception as exc:  # report to the parent instead of hanging it
        q.put((rank, "error", repr(exc), None, None))


def run_ranks(world, case_name, target=None):
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=target or worker, args=(r, world, port, case_name, q)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        results = [q.get(timeout=600) for _ in procs]
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    assert all(r[1] != "error" for r in results), results
    return results


def whole_tensor_answers(x, ne, nb=None):
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle
    olib = oracle.load()
    v = oracle.host_view(x, ne, nb)
    out = np.zeros(1, np.float32)
    ov = oracle.host_view(out, [1, 1, 1, 1])
    assert olib.oracle_sum(ctypes.byref(v), ctypes.byref(ov)) == 0
    idx = ctypes.c_int64()
    assert olib.oracle_argmax_index(ctypes.byref(v), ctypes.byref(idx), None) == 0
    return float(out[0]), idx.value


def check(results, want_sum, want_idx):
    for rank, total32, total64, gidx, repeat_ok in results:
        if not np.isnan(want_sum):
            assert abs(total32 - want_sum) <= 1e-5 * max(1.0, abs(want_sum)), (rank, total32, want_sum)
        assert gidx == want_idx, (rank, gidx, want_idx)
        assert repeat_ok in (None, True), rank


@pytest.mark.parametrize("case_name", list(SMALL))
def test_two_gpu_partials_match_whole_tensor(case_name):
    if gpu_count() < 2:
        pytest.skip("needs 2 GPUs")
    results = run_ranks(2, case_name)
    case = SMALL[case_name]
    want_sum, want_idx = whole_tensor_answers(small_tensor(case), case["ne"])
    check(results, want_sum, want_idx)


def test_cfg5_sharded_over_all_gpus():
    world = gpu_count()
    if world < 2:
        pytest.skip("needs 2 GPUs")
    world = min(world, 8)
    results = run_ranks(world, "cfg5")
    sys.path.insert(0, str(ROOT))
    from __graft_entry__ import load_package
    load_package()
    from emel_rs_b200 import workloads as W
    x, _ = cfg5_slices(W, 0, W.CFG5_NE[3])
    ne, nb = W.cfg5_src0_view()
    want_sum, want_idx = whole_tensor_answers(x, ne, nb)
    check(results, want_sum, want_idx)


# ---- NVLink peer exchange (emel_cuda_exchange_*) -----------------------------
def pattern(rank, step):
    return bytes((rank * 37 + step * 11 + i) % 256 for i in range(32))


def exchange_worker(rank, world, port, mode, q):
    """Publishes a per-rank, per-step 32-byte pattern and checks every rank's
    gathered array: eager steps, then replays of a captured graph (the step
    counter lives on the device).  mode "timeout": afterwards rank 0 alone
    publishes and waits on a second exchange with a 300 ms limit; its wait
    must expire, report EMEL_CUDA_TIMEOUT and leave the context usable."""
    try:
        sys.path.insert(0, str(ROOT))
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        from datetime import timedelta

        import torch
        import torch.distributed as dist

        from __graft_entry__ import load_package

        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                                device_id=dev)
        pkg = load_package()
        from emel_rs_b200 import distributed as D

        lib = pkg.lib()
        ctx = pkg.Context(rank)
        stream = pkg.Stream(ctx)
        sh = stream.handle
        ex = D.PeerExchange(pkg, ctx, dist, world, rank, timeout_ms=10000)
        payload = torch.zeros(32, dtype=torch.uint8, device=dev)
        gathered = torch.zeros(world * 32, dtype=torch.uint8, device=dev)

        def set_payload(step):
            payload.copy_(torch.frombuffer(bytearray(pattern(rank, step)), dtype=torch.uint8))
            torch.cuda.synchronize()

        def gathered_ok(step):
            return gathered.cpu().numpy().tobytes() == b"".join(pattern(r, step) for r in range(world))

        eager_ok = True
        for step in range(12):
            set_payload(step)
            ex.publish(sh, payload.data_ptr())
            ex.wait(sh, gathered.data_ptr())
            stream.synchronize()
            eager_ok = eager_ok and gathered_ok(step)
        graph = pkg.Graph(ctx, stream)
        with graph:
            ex.publish(sh, payload.data_ptr())
            ex.wait(sh, gathered.data_ptr())
        graph_ok = True
        for step in range(12, 20):
            set_payload(step)
            graph.launch()
            stream.synchronize()
            graph_ok = graph_ok and gathered_ok(step)
        graph.close()
        timeout_status = usable = None
        short = None
        if mode == "timeout":
            short = D.PeerExchange(pkg, ctx, dist, world, rank, timeout_ms=300)
            dist.barrier()
            if rank == 0:
                set_payload(99)
                short.publish(sh, payload.data_ptr())
                short.wait(sh, gathered.data_ptr())
                timeout_status = lib.emel_cuda_stream_synchronize(ctx.handle, sh)
                x = torch.full((4096,), -2.0, device=dev)
                y = torch.empty_like(x)
                v, w = pkg.CView(), pkg.CView()
                for t, cv in ((x, v), (y, w)):
                    cv.data, cv.storage_bytes, cv.dtype = t.data_ptr(), t.numel() * 4, 0
                    for d, (n, b) in enumerate(zip([4096, 1, 1, 1], pkg.contiguous_nb([4096, 1, 1, 1]))):
                        cv.ne[d], cv.nb[d] = n, b
                st = lib.emel_cuda_unary(ctx.handle, sh, 6, ctypes.byref(v), ctypes.byref(w))  # relu
                st2 = lib.emel_cuda_stream_synchronize(ctx.handle, sh)
                usable = st == 0 and st2 == 0 and bool((y.cpu() == 0).all())
        dist.barrier()
        ex.close()
        if short is not None:
            short.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, eager_ok, graph_ok, timeout_status, usable))
    except Exception as exc:  # report to the parent instead of hanging it
        q.put((rank, "error", repr(exc), None, None))


def test_peer_exchange_eager_and_graph_replays():
    world = gpu_count()
    if world < 2:
        pytest.skip("needs 2 GPUs")
    results = run_ranks(min(world, 8), "steps", target=exchange_worker)
    for rank, eager_ok, graph_ok, _, _ in results:
        assert eager_ok and graph_ok, rank


def test_peer_exchange_wait_expires_without_a_publisher():
    if gpu_count() < 2:
        pytest.skip("needs 2 GPUs")
    sys.path.insert(0, str(ROOT))
    results = run_ranks(2, "timeout", target=exchange_worker)
    by_rank = {r[0]: r for r in results}
    assert by_rank[0][1] and by_rank[0][2] and by_rank[1][1] and by_rank[1][2]
    assert by_rank[0][3] == 17, by_rank[0]  # EMEL_CUDA_TIMEOUT
    assert by_rank[0][4] is True, by_rank[0]


# ---- device-side combine (emel_cuda_exchange_wait_sum_argmax) ----------------
def shard_of(pkg, torch, dev, W, D, case_name, world, rank):
    """(device tensor, view, first ordinal) of this rank's dim-3 slices."""
    if case_name == "cfg5":
        b, e = D.shard_bounds(W.CFG5_NE[3], world, rank)
        s0, _ = cfg5_slices(W, b, e)
        ne, nb = W.cfg5_src0_view(ne3=e - b)
        t = torch.from_numpy(s0).to(dev)
    else:
        case = SMALL[case_name]
        full = case["ne"]
        x = small_tensor(case)
        b, e = D.shard_bounds(full[3], world, rank)
        plane = full[0] * full[1] * full[2]
        t = torch.from_numpy(np.ascontiguousarray(x[b * plane:e * plane])).to(dev)
        ne = [full[0], full[1], full[2], e - b]
        nb = pkg.contiguous_nb(ne)
    v = pkg.CView()
    v.data, v.storage_bytes, v.dtype = t.data_ptr(), t.numel() * 4, 0
    for d in range(4):
        v.ne[d], v.nb[d] = ne[d], nb[d]
    return t, v, b * ne[0] * ne[1] * ne[2]


def combine_worker(rank, world, port, case_name, q):
    """Per step: the shard's f64 sum and argmax partial, published over
    NVLink, then one wait that gathers and combines on the device into an
    F32 sum and an I64 index.  Two eager steps, then three replays of the
    step captured as a graph; every step's answers are reported."""
    try:
        sys.path.insert(0, str(ROOT))
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        from datetime import timedelta

        import torch
        import torch.distributed as dist

        from __graft_entry__ import load_package

        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120),
                                device_id=dev)
        pkg = load_package()
        from emel_rs_b200 import distributed as D
        from emel_rs_b200 import workloads as W

        lib = pkg.lib()
        ctx = pkg.Context(rank)
        stream = pkg.Stream(ctx)
        sh = stream.handle
        t, v, base = shard_of(pkg, torch, dev, W, D, case_name, world, rank)
        payload = torch.zeros(32, dtype=torch.uint8, device=dev)
        gathered = torch.zeros(world * 32, dtype=torch.uint8, device=dev)
        sum_out = torch.full((1,), 7.0, dtype=torch.float32, device=dev)
        idx_out = torch.full((1,), -1, dtype=torch.int64, device=dev)
        vs, vi = pkg.CView(), pkg.CView()
        for cv, tt, code in ((vs, sum_out, 0), (vi, idx_out, 27)):
            cv.data, cv.storage_bytes, cv.dtype = tt.data_ptr(), tt.numel() * tt.element_size(), code
            for d, (n, b) in enumerate(zip([1, 1, 1, 1], pkg.contiguous_nb([1, 1, 1, 1], code))):
                cv.ne[d], cv.nb[d] = n, b
        torch.cuda.synchronize()
        ex = D.PeerExchange(pkg, ctx, dist, world, rank, timeout_ms=10000)
        B = ctypes.byref

        def step():
            p = payload.data_ptr()
            assert lib.emel_cuda_sum_f64(ctx.handle, sh, B(v), ctypes.c_void_p(p)) == 0, ctx.last_error
            assert lib.emel_cuda_argmax_partial_compute(ctx.handle, sh, B(v), base, ctypes.c_void_p(p + 8)) == 0
            ex.publish(sh, p)
            st = lib.emel_cuda_exchange_wait_sum_argmax(ctx.handle, sh, ex.handle, ctypes.c_void_p(gathered.data_ptr()),
                                                        B(vs), B(vi))
            assert st == 0, ctx.last_error

        answers = []
        for _ in range(2):
            step()
            assert lib.emel_cuda_stream_synchronize(ctx.handle, sh) == 0
            answers.append((float(sum_out.cpu()[0]), int(idx_out.cpu()[0])))
            sum_out.fill_(7.0)
            idx_out.fill_(-1)
            torch.cuda.synchronize()
        graph = pkg.Graph(ctx, stream)
        with graph:
            step()
        for _ in range(3):
            graph.launch()
            assert lib.emel_cuda_stream_synchronize(ctx.handle, sh) == 0
            answers.append((float(sum_out.cpu()[0]), int(idx_out.cpu()[0])))
            sum_out.fill_(7.0)
            idx_out.fill_(-1)
            torch.cuda.synchronize()
        graph.close()
        dist.barrier()
        ex.close()
        dist.barrier()
        dist.destroy_process_group()
        q.put((rank, answers, None, None, None))
    except Exception as exc:  # report to the parent instead of hanging it
        q.put((rank, "error", repr(exc), None, None))


def check_combined(results, want_sum, want_idx):
    for rank, answers, _, _, _ in results:
        assert len(answers) == 5, rank
        for total32, gidx in answers:
            if np.isnan(want_sum):
                assert np.isnan(total32), (rank, total32)
            else:
                assert abs(total32 - want_sum) <= 1e-5 * max(1.0, abs(want_sum)), (rank, total32, want_sum)
            assert gidx == want_idx, (rank, gidx, want_idx)


@pytest.mark.parametrize("case_name", list(SMALL))
def test_device_combine_matches_whole_tensor(case_name):
    """The combined whole-tensor sum (f64 partials added in rank order, one
    rounding) and argmax (strict >, first index; a NaN at element 0 pins 0)
    against the oracle's OpSum / OpArgmax on the whole tensor.  Cases with
    eight slices run on up to 8 GPUs, the others on 2."""
    gpus = gpu_count()
    if gpus < 2:
        pytest.skip("needs 2 GPUs")
    case = SMALL[case_name]
    world = min(gpus, 8) if case["ne"][3] >= 8 else 2
    results = run_ranks(world, case_name, target=combine_worker)
    want_sum, want_idx = whole_tensor_answers(small_tensor(case), case["ne"])
    check_combined(results, want_sum, want_idx)


def test_device_combine_cfg5_over_all_gpus():
    gpus = gpu_count()
    if gpus < 2:
        pytest.skip("needs 2 GPUs")
    results = run_ranks(min(gpus, 8), "cfg5", target=combine_worker)
    sys.path.insert(0, str(ROOT))
    from __graft_entry__ import load_package
    load_package()
    from emel_rs_b200 import workloads as W
    x, _ = cfg5_slices(W, 0, W.CFG5_NE[3])
    ne, nb = W.cfg5_src0_view()
    want_sum, want_idx = whole_tensor_answers(x, ne, nb)
    check_combined(results, want_sum, want_idx)
