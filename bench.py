"""Benchmark of the emel-kernels hot path on B200.

Default workload (configuration 5 of the benchmark set): src0 f32
ne = [128, 32, 8192, 8] (1.07 GB) stored as a view with dims 1 and 2
swapped, split along dim 3 across the GPUs (strong scaling: the tensor is
fixed, each of N GPUs holds 8/N slices); src1 ne = [128, 1, 8192, 1]
replicated.  One step = whole-tensor sum and argmax, repeat-broadcast mul
and add; with N > 1 the per-shard sum / argmax partials are exchanged over
NVLink and combined on the device.  Metric: achieved HBM GB/s (algorithmic
bytes: every input element read once, every output element written once,
per op; ops run one after another on one stream).

    python bench.py [--gpus N --steps K --warmup W]       # B200 device table
    python bench.py --impl reference ...                   # CPU reference lane
    python bench.py --suite                                # per-op lines, all configs
    python bench.py --workload cfg2 [--gpus N]             # configuration 2 sweep, weak scaling

Multi-GPU (torchrun, one process per GPU): the timed region is bracketed by
barriers and the max over ranks is reported.
"""

import argparse
import ctypes
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from __graft_entry__ import load_package  # noqa: E402

METRIC = "per-op achieved HBM GB/s (fraction of ~8 TB/s) at 1/2/4/8 B200 vs host CPU"
UNIT = "GB/s"
OPS = [("silu", 10), ("gelu", 8), ("relu", 6), ("exp", 13), ("neg", 2), ("sqr", 64), ("sqrt", 65), ("pow2", 64)]
FALLBACK_HBM_GBS = 6650.0


# ---------------------------------------------------------------------------
# environment
# ---------------------------------------------------------------------------
def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["hbm_gbs"]), "measured"
    return FALLBACK_HBM_GBS, "fallback"


def profile_traffic(name):
    """Per-launch DRAM bytes of the dominant kernel from a committed ncu
    summary (a line `dram_bytes_per_launch: <int>`), or None."""
    p = ROOT / "profiles" / name
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.strip().startswith("dram_bytes_per_launch:"):
            return int(line.split(":", 1)[1].strip().split()[0])
    return None


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while the timed
    region runs."""

    REASONS = {0x8: "hw_slowdown", 0x40: "hw_thermal_slowdown", 0x20: "sw_thermal_slowdown", 0x4: "sw_power_cap"}

    def __init__(self, device):
        self.device = device
        self.samples = []
        self.reasons = set()
        self.stop = threading.Event()
        self.max_mhz = None
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(self._physical_index(device))
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.nv = None

    @staticmethod
    def _physical_index(device):
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        if vis:
            ids = [v.strip() for v in vis.split(",") if v.strip()]
            if device < len(ids) and ids[device].isdigit():
                return int(ids[device])
        return device

    def _run(self):
        while not self.stop.is_set():
            try:
                self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
                get = getattr(self.nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                    self.nv.nvmlDeviceGetCurrentClocksThrottleReasons
                r = get(self.h)
                for bit, name in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            self.stop.wait(0.01)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *exc):
        if self.ok:
            self.stop.set()
            self.t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# B200 arm
# ---------------------------------------------------------------------------
class Cfg2Step:
    """The 16-op sweep over device buffers.  Each op reads its own copy of
    its input so one step touches ~705 MB (5.6x the 126 MB L2): no input is
    still in L2 when it is read again a step later."""

    def __init__(self, pkg, ctx, torch, device, seed, only=None):
        from emel_rs_b200 import workloads
        self.pkg, self.ctx = pkg, ctx
        x, xa = workloads.cfg2(seed)
        self.host = {"f32": (x, xa), "f16": (x.astype(np.float16), xa.astype(np.float16))}
        self.ne = [workloads.CFG2_NE[0], workloads.CFG2_NE[1], 1, 1]
        self.n = x.size
        self.tensors = []
        self.launches = []  # (name, bytes, fn, args)
        lib = pkg.lib()
        for dt_name, code, tdt in (("f32", 0, torch.float32), ("f16", 1, torch.float16)):
            base, base_abs = (torch.from_numpy(a).to(device) for a in self.host[dt_name])
            for name, op in OPS:
                if only and f"{name}_{dt_name}" not in only:
                    continue
                src = (base_abs if name in ("sqrt", "pow2") else base).clone()
                dst = torch.empty_like(src)
                self.tensors += [src, dst]
                sv = self._view(src, code)
                dv = self._view(dst, code)
                nbytes = 2 * self.n * src.element_size()
                self.launches.append((f"{name}_{dt_name}", nbytes, lib.emel_cuda_unary,
                                      [op, ctypes.byref(sv), ctypes.byref(dv)], (sv, dv)))
        self.step_bytes = sum(l[1] for l in self.launches)

    def _view(self, t, code):
        v = self.pkg.CView()
        v.data = t.data_ptr()
        v.storage_bytes = t.numel() * t.element_size()
        nb = self.pkg.contiguous_nb(self.ne, code)
        for d in range(4):
            v.ne[d] = self.ne[d]
            v.nb[d] = nb[d]
        v.dtype = code
        return v

    def run(self, stream, events=None):
        """Issues the 16 launches on `stream`; with `events` (17 of them),
        an event before each launch and one after the last."""
        h = self.ctx.handle
        for i, (_, _, fn, args, _) in enumerate(self.launches):
            if events is not None:
                events[i].record_timed(stream)
            st = fn(h, stream, *args)
            if st != 0:
                raise RuntimeError(f"launch {self.launches[i][0]} failed: {st} {self.ctx.last_error}")
        if events is not None:
            events[-1].record_timed(stream)

    def capture(self, stream, events=None, branches=1):
        """One step as a CUDA graph.  The 16 ops are independent (each reads
        its own input, writes its own output), so with branches > 1 they are
        spread round-robin over parallel graph branches (fork/join through
        events) and neighbouring kernels overlap instead of each paying its
        own ramp-up and tail."""
        g = self.pkg.Graph(self.ctx, stream)
        h = self.ctx.handle
        with g:
            if branches <= 1:
                self.run(stream.handle, events)
            else:
                if not hasattr(self, "side"):
                    self.side = [self.pkg.Stream(self.ctx) for _ in range(branches - 1)]
                lanes = [stream] + self.side[:branches - 1]
                fork = self.pkg.CudaEvent(self.ctx)
                fork.record(stream.handle)
                for s in lanes[1:]:
                    s.wait(fork)
                for i, (name, _, fn, args, _) in enumerate(self.launches):
                    st = fn(h, lanes[i % branches].handle, *args)
                    if st != 0:
                        raise RuntimeError(f"launch {name} failed: {st} {self.ctx.last_error}")
                self._joins = []
                for s in lanes[1:]:
                    e = self.pkg.CudaEvent(self.ctx)
                    e.record(s.handle)
                    stream.wait(e)
                    self._joins.append(e)
                self._fork = fork
        return g

    def calibration_graphs(self, stream):
        """One graph per op: the op over every buffer pair of its dtype, back
        to back, between two events.  Returns (name, bytes, reps, graph, e0, e1)."""
        out = []
        h = self.ctx.handle
        for name, nbytes, fn, args, (sv, dv) in self.launches:
            dt = name.rsplit("_", 1)[1]
            pairs = [views for nm, _, _, _, views in self.launches if nm.rsplit("_", 1)[1] == dt]
            e0, e1 = self.pkg.CudaEvent(self.ctx), self.pkg.CudaEvent(self.ctx)
            g = self.pkg.Graph(self.ctx, stream)
            with g:
                e0.record_timed(stream.handle)
                for psv, pdv in pairs:
                    st = fn(h, stream.handle, args[0], ctypes.byref(psv), ctypes.byref(pdv))
                    if st != 0:
                        raise RuntimeError(self.ctx.last_error)
                e1.record_timed(stream.handle)
            out.append((name, nbytes, len(pairs), g, e0, e1))
        return out


def run_b200(args, world, rank, local):
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    pkg = load_package()
    ctx = pkg.Context(local)
    only = set(args.only.split(",")) if args.only else None
    step = Cfg2Step(pkg, ctx, torch, device, seed=2 + 1000 * rank, only=only)
    torch.cuda.synchronize()
    stream = pkg.Stream(ctx)
    sh = stream.handle

    # The step is captured once as a CUDA graph and replayed K times.
    plain = step.capture(stream, branches=args.branches)
    calib = step.calibration_graphs(stream)

    for _ in range(args.warmup):
        plain.launch()
    stream.synchronize()
    t0, t1 = pkg.CudaEvent(ctx), pkg.CudaEvent(ctx)
    launches_before = ctx.launches
    if world > 1:
        dist.barrier()
    stream.synchronize()
    with ClockSampler(local) as clocks:
        t0.record(sh)
        for s in range(args.steps):
            plain.launch()
        t1.record(sh)
        stream.synchronize()
        gpu_launches = ctx.launches - launches_before
        # Per-kernel durations, right after the timed region on the same
        # stream: each op runs 8 times back to back over 8 distinct buffer
        # pairs of its dtype (117-235 MB, no L2 reuse) between one event pair.
        # An event pair costs ~5 us inside a graph, so bracketing single
        # launches would overstate short kernels; over 8 launches the bias is
        # under 0.7 us per launch.
        per_op = {}
        for name, nbytes, reps, g, e0, e1 in calib:
            d = []
            for _ in range(3):
                g.launch()
                stream.synchronize()
                d.append(e0.elapsed_ms(e1) / reps)
            per_op[name] = (nbytes, statistics.median(d))
    if world > 1:
        dist.barrier()
    ms = t0.elapsed_ms(t1)
    ms_t = torch.tensor([ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_max = float(ms_t.item())

    # the dominant kernel: the op with the largest share of the step's kernel
    # time (all 16 launches are instantiations of the ew_flat streaming kernel)
    dom_name, (dom_bytes, dom_ms) = max(per_op.items(), key=lambda kv: kv[1][1])
    kernel_ms = sum(t for _, t in per_op.values())

    e2e = None if args.no_e2e else run_e2e(args, pkg, ctx, torch, step, stream, world)

    if rank != 0:
        if world > 1:
            dist.destroy_process_group()
        return
    peak, peak_kind = peaks()
    value = world * args.steps * step.step_bytes / (ms_max / 1e3) / 1e9
    achieved = dom_bytes / (dom_ms / 1e3) / 1e9
    traffic = profile_traffic("unary_cfg2_ncu.md")
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_max / args.steps, 5), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32+f16", "data": "synthetic (seeded, per rank)",
        "config": {
            "workload": "cfg2 unary/activation sweep: silu, gelu(tanh), relu, exp, neg, sqr, sqrt, pow(x,2) "
                        "on f32 and f16 ne=[14336,512]; N(0,2) clamped to [-10,10]; sqrt/pow on |x|+1e-3",
            "ops_per_step": len(step.launches), "bytes_per_step": step.step_bytes,
            "l2": "inputs larger than L2: 16 distinct input/output buffer pairs, 705 MB touched per step",
            "parallelism": f"dp{world} (independent per-GPU batches)", "graph_branches": args.branches,
        },
        "roofline": {"bound": "hbm", "kernel": f"ew_flat ({dom_name})", "achieved": round(achieved, 1),
                     "peak": peak, "peak_source": f"{peak_kind} hbm_gbs", "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "traffic": traffic,
                     "algorithmic_bytes_per_launch": dom_bytes, "launch_ms": round(dom_ms, 5),
                     "share_of_step": round(dom_ms / kernel_ms, 4)},
        "per_op_gbs": {k: round(b / (t / 1e3) / 1e9, 1) for k, (b, t) in per_op.items()},
        "e2e": e2e,
        "gpu_launches": gpu_launches,
        "clocks": clocks.summary(),
    }
    if world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_single(args)
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_e2e(args, pkg, ctx, torch, step, stream, world):
    """The same metric through the C ABI with host buffers: every step copies
    the four source tensors from pinned host memory, runs the 16 ops and
    reads all 16 outputs back (captured once, replayed per step)."""
    lib = pkg.lib()
    sh = stream.handle
    device = torch.device("cuda", ctx.device)
    srcs = []  # (pinned host, device tensor)
    for dt_name in ("f32", "f16"):
        for arr in step.host[dt_name]:
            h = torch.from_numpy(arr.copy()).pin_memory()
            d = torch.empty_like(h, device=device)
            srcs.append((h, d))
    f32x, f32a, f16x, f16a = (d for _, d in srcs)
    outs = []
    launches = []
    for dt_name, code, (x, xa) in (("f32", 0, (f32x, f32a)), ("f16", 1, (f16x, f16a))):
        for name, op in OPS:
            src = xa if name in ("sqrt", "pow2") else x
            dst = torch.empty_like(src)
            hout = torch.empty(dst.shape, dtype=dst.dtype, pin_memory=True)
            outs.append((hout, dst))
            sv, dv = step._view(src, code), step._view(dst, code)
            launches.append((op, sv, dv))
    h2d = sum(h.numel() * h.element_size() for h, _ in srcs)
    d2h = sum(h.numel() * h.element_size() for h, _ in outs)

    def one():
        for h, d in srcs:
            lib.emel_cuda_memcpy_h2d(ctx.handle, sh, d.data_ptr(), h.data_ptr(), h.numel() * h.element_size())
        for op, sv, dv in launches:
            st = lib.emel_cuda_unary(ctx.handle, sh, op, ctypes.byref(sv), ctypes.byref(dv))
            if st != 0:
                raise RuntimeError(ctx.last_error)
        for h, d in outs:
            lib.emel_cuda_memcpy_d2h(ctx.handle, sh, h.data_ptr(), d.data_ptr(), h.numel() * h.element_size())

    torch.cuda.synchronize()
    g = pkg.Graph(ctx, stream)
    with g:
        one()
    steps = max(3, min(args.steps, 20))
    for _ in range(2):
        g.launch()
    stream.synchronize()
    t0, t1 = pkg.CudaEvent(ctx), pkg.CudaEvent(ctx)
    t0.record(sh)
    for _ in range(steps):
        g.launch()
    t1.record(sh)
    stream.synchronize()
    ms = t0.elapsed_ms(t1)
    if world > 1:
        import torch.distributed as dist
        m = torch.tensor([ms], dtype=torch.float64, device=device)
        dist.all_reduce(m, op=dist.ReduceOp.MAX)
        ms = float(m.item())
    value = world * steps * step.step_bytes / (ms / 1e3) / 1e9
    return {"value": round(value, 2), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "steps": steps,
            "path": "graph of emel_cuda_memcpy_h2d x4 + emel_cuda_unary x16 + emel_cuda_memcpy_d2h x16 (pinned host)"}


# ---------------------------------------------------------------------------
# Per-op suite over all five configurations (BASELINE table; 1 GPU)
# ---------------------------------------------------------------------------
L2_BYTES = 126 * 1024 * 1024


def run_suite(args):
    """Times every operator of every configuration: each op is captured R
    times back to back over enough rotating buffer sets that a set is
    evicted from L2 before it is read again, and the graph is timed with
    events.  Prints one JSON line per op and returns them."""
    import torch

    pkg = load_package()
    from emel_rs_b200 import workloads as W

    lib = pkg.lib()
    ctx = pkg.Context(0)
    stream = pkg.Stream(ctx)
    sh = stream.handle
    dev = torch.device("cuda", 0)
    peak, peak_kind = peaks()
    out = []

    def view(t, ne, nb=None, code=0):
        v = pkg.CView()
        v.data = t.data_ptr()
        v.storage_bytes = t.numel() * t.element_size()
        nb = nb or pkg.contiguous_nb(ne, code)
        for d in range(4):
            v.ne[d] = ne[d]
            v.nb[d] = nb[d]
        v.dtype = code
        return v

    def sets_for(nbytes):
        return max(1, min(8, -(-3 * L2_BYTES // max(1, nbytes))))

    only = set(args.only.split(",")) if args.only else None

    def measure(cfg, name, nbytes, elems, make_launch, sets, extra=None):
        if only and name not in only and cfg not in only:
            return
        torch.cuda.synchronize()  # inputs were uploaded on torch's stream
        launches = [make_launch(k) for k in range(sets)]
        # 32 back-to-back launches per graph (a whole number of passes over
        # the buffer sets): the graph's own launch and drain are spread thin,
        # as in a model step of many operators
        reps = -(-32 // sets) * sets
        for L in launches:
            L()
        stream.synchronize()
        g = pkg.Graph(ctx, stream)
        e0, e1 = pkg.CudaEvent(ctx), pkg.CudaEvent(ctx)
        with g:
            e0.record_timed(sh)
            for r in range(reps):
                launches[r % sets]()
            e1.record_timed(sh)
        times = []
        for _ in range(5):
            g.launch()
            stream.synchronize()
            times.append(e0.elapsed_ms(e1) / reps)
        g.close()
        ms = statistics.median(times)
        gbs = nbytes / (ms / 1e3) / 1e9
        line = {"suite": cfg, "op": name, "gbs": round(gbs, 1), "frac_of_peak": round(gbs / peak, 4),
                "gelems": round(elems / (ms / 1e3) / 1e9, 2), "us_per_launch": round(ms * 1e3, 2),
                "algorithmic_bytes": nbytes, "buffer_sets": sets, "peak": f"{peak} GB/s ({peak_kind})"}
        if extra is not None:
            line.update(extra(ms))
        print(json.dumps(line), flush=True)
        out.append(line)

    def chk(st):
        if st != 0:
            raise RuntimeError(f"status {st}: {ctx.last_error}")

    # with --only, a configuration's data is built only when one of its ops
    # is selected (keys: suite names, or the op names themselves)
    suite_ops = {"cfg1": [f"broadcast_row_{o}" for o in ("add", "sub", "mul", "div")],
                 "cfg2": [f"{o}_{dt}" for o, _ in OPS for dt in ("f32", "f16")],
                 "cfg3": ["rms_norm", "rms_norm_mul_fused", "rms_norm_then_mul_two_ops", "norm", "sum_rows"],
                 "cfg5": ["repeat_mul_permuted", "repeat_add_permuted", "sum_whole_permuted",
                          "argmax_whole_permuted", "cont_permuted"],
                 "cfg5_shard": ["repeat_mul_slice", "repeat_add_slice", "sum_slice", "argmax_slice"],
                 "glu": list(W.GLU_OPS), "get_rows": [f"get_rows_{f}" for f in W.EMB_FORMATS],
                 "rope": ["rope_neox", "rope_norm"],
                 "matvec": ["mul_mat_argmax_vocab", "mul_mat_argmax_q8_0_vocab", "mul_mat_argmax_q2_k_vocab",
                            "mul_mat_argmax_q3_k_vocab", "mul_mat_argmax_q4_k_vocab", "mul_mat_argmax_q6_k_vocab"],
                 "attention": [o.name for o in W.fa_spec().ops], "diag": [o.name for o in W.diag_spec().ops]}

    def wants(*keys):
        if not only:
            return True
        return any(key in only or any(name in only for name in suite_ops.get(key, [])) for key in keys)

    B = ctypes.byref
    # cfg1: row-broadcast binary ops
    if wants("cfg1",):
        src0, src1 = W.cfg1()
        spec = W.cfg1_spec()
        nb_ = spec.ops[0].bytes
        S = sets_for(nb_)
        a = [torch.from_numpy(src0).to(dev) for _ in range(S)]
        b = torch.from_numpy(src1).to(dev)
        d = [torch.empty_like(a[0]) for _ in range(S)]
        ne = [W.CFG1_NE[0], W.CFG1_NE[1], 1, 1]
        va = [view(t, ne) for t in a]
        vb = view(b, [W.CFG1_NE[0], 1, 1, 1])
        vd = [view(t, ne) for t in d]
        for op, opname in enumerate(("add", "sub", "mul", "div")):
            measure("cfg1", f"broadcast_row_{opname}", nb_, spec.ops[0].elements,
                    lambda k, op=op: (lambda: chk(lib.emel_cuda_broadcast_row(ctx.handle, sh, op, B(va[k]), B(vb), B(vd[k])))),
                    S)
        del a, d
    # cfg2: unary sweep
    if wants("cfg2",):
        x, xa = W.cfg2()
        ne = [W.CFG2_NE[0], W.CFG2_NE[1], 1, 1]
        for dt, code, tdt in (("f32", 0, torch.float32), ("f16", 1, torch.float16)):
            n = x.size * (4 if dt == "f32" else 2) * 2
            S = sets_for(n)
            for opname, opc in OPS:
                base = torch.from_numpy(xa if opname in ("sqrt", "pow2") else x).to(dev).to(tdt)
                srcs = [base.clone() for _ in range(S)]
                dsts = [torch.empty_like(base) for _ in range(S)]
                vs = [view(t, ne, code=code) for t in srcs]
                vo = [view(t, ne, code=code) for t in dsts]
                measure("cfg2", f"{opname}_{dt}", n, x.size,
                        lambda k, opc=opc: (lambda: chk(lib.emel_cuda_unary(ctx.handle, sh, opc, B(vs[k]), B(vo[k])))), S)
                del srcs, dsts
    # cfg3: row normalisation
    if wants("cfg3",):
        x3, w3 = W.cfg3()
        ne = [W.CFG3_NE[0], W.CFG3_NE[1], 1, 1]
        spec = W.cfg3_spec()
        xs = torch.from_numpy(x3).to(dev)
        ws = torch.from_numpy(w3).to(dev)
        ys = torch.empty_like(xs)
        ys2 = torch.empty_like(xs)
        rows = torch.empty(W.CFG3_NE[1], device=dev)
        vx, vw, vy, vy2 = view(xs, ne), view(ws, [W.CFG3_NE[0], 1, 1, 1]), view(ys, ne), view(ys2, ne)
        vr = view(rows, [1, W.CFG3_NE[1], 1, 1])
        measure("cfg3", "rms_norm", spec.ops[0].bytes, spec.ops[0].elements,
                lambda k: (lambda: chk(lib.emel_cuda_rms_norm(ctx.handle, sh, B(vx), B(vy), 1e-6))), 1)
        measure("cfg3", "rms_norm_mul_fused", spec.ops[1].bytes, spec.ops[1].elements,
                lambda k: (lambda: chk(lib.emel_cuda_rms_norm_mul(ctx.handle, sh, B(vx), B(vw), B(vy), 1e-6))), 1)
        measure("cfg3", "rms_norm_then_mul_two_ops", spec.ops[0].bytes + spec.ops[1].bytes, spec.ops[0].elements,
                lambda k: (lambda: (chk(lib.emel_cuda_rms_norm(ctx.handle, sh, B(vx), B(vy), 1e-6)),
                                    chk(lib.emel_cuda_broadcast_row(ctx.handle, sh, 2, B(vy), B(vw), B(vy2))))), 1)
        measure("cfg3", "norm", spec.ops[2].bytes, spec.ops[2].elements,
                lambda k: (lambda: chk(lib.emel_cuda_norm(ctx.handle, sh, B(vx), B(vy), 1e-5))), 1)
        measure("cfg3", "sum_rows", spec.ops[3].bytes, spec.ops[3].elements,
                lambda k: (lambda: chk(lib.emel_cuda_sum_rows(ctx.handle, sh, B(vx), B(vr)))), 1)
        del xs, ys, ys2
    # cfg4a: masked, scaled softmax
    if wants("soft_max_ext_scale_mask", "cfg4"):
        scores, mask = W.cfg4a()
        kv, q, h = W.CFG4A_NE
        spec = W.cfg4_spec()
        ts = torch.from_numpy(scores).to(dev)
        tm = torch.from_numpy(mask).to(dev)
        to = torch.empty_like(ts)
        vs_, vm, vo_ = view(ts, [kv, q, h, 1]), view(tm, [kv, q, 1, 1], code=1), view(to, [kv, q, h, 1])
        measure("cfg4", "soft_max_ext_scale_mask", spec.ops[0].bytes, spec.ops[0].elements,
                lambda k: (lambda: chk(lib.emel_cuda_soft_max_ext(ctx.handle, sh, B(vs_), B(vm), B(vo_),
                                                                    float(W.CFG4A_SCALE)))), 1)
        del ts, to
    # cfg4b: vocab softmax and per-row argmax
    if wants("soft_max_vocab", "argmax_rows_vocab", "cfg4"):
        logits, _ = W.cfg4b()
        v, rws = W.CFG4B_NE
        spec = W.cfg4_spec()
        S = sets_for(spec.ops[1].bytes)
        tl = [torch.from_numpy(logits).to(dev) for _ in range(S)]
        tlo = [torch.empty_like(tl[0]) for _ in range(S)]
        ti = torch.empty(rws, dtype=torch.int64, device=dev)
        vl = [view(t, [v, rws, 1, 1]) for t in tl]
        vlo = [view(t, [v, rws, 1, 1]) for t in tlo]
        vi = view(ti, [1, rws, 1, 1], code=27)
        measure("cfg4", "soft_max_vocab", spec.ops[1].bytes, spec.ops[1].elements,
                lambda k: (lambda: chk(lib.emel_cuda_soft_max(ctx.handle, sh, B(vl[k]), B(vlo[k])))), S)
        measure("cfg4", "argmax_rows_vocab", spec.ops[2].bytes, spec.ops[2].elements,
                lambda k: (lambda: chk(lib.emel_cuda_argmax_rows(ctx.handle, sh, B(vl[k]), B(vi)))), S)
        del tl, tlo
    # cfg5: permuted repeat broadcast, whole-tensor sum and argmax
    if wants("cfg5",):
        s0, s1 = W.cfg5()
        ne5, nb5 = W.cfg5_src0_view()
        spec = W.cfg5_spec()
        t0 = torch.from_numpy(s0).to(dev)
        t1 = torch.from_numpy(s1).to(dev)
        td = torch.empty_like(t0)
        tsum = torch.empty(1, device=dev)
        targ = torch.empty(1, dtype=torch.int64, device=dev)
        v0 = view(t0, ne5, nb5)
        v1 = view(t1, [128, 1, 8192, 1])
        vd5 = view(td, ne5)
        one = [1, 1, 1, 1]
        vsum, varg = view(tsum, one), view(targ, one, code=27)
        for op, opname in ((2, "mul"), (0, "add")):
            measure("cfg5", f"repeat_{opname}_permuted", spec.ops[0].bytes, spec.ops[0].elements,
                    lambda k, op=op: (lambda: chk(lib.emel_cuda_binary_repeat(ctx.handle, sh, op, B(v0), B(v1), B(vd5)))), 1)
        measure("cfg5", "sum_whole_permuted", spec.ops[2].bytes, spec.ops[2].elements,
                lambda k: (lambda: chk(lib.emel_cuda_sum(ctx.handle, sh, B(v0), B(vsum)))), 1)
        measure("cfg5", "argmax_whole_permuted", spec.ops[3].bytes, spec.ops[3].elements,
                lambda k: (lambda: chk(lib.emel_cuda_argmax(ctx.handle, sh, B(v0), B(varg)))), 1)
        # shape.rs OpCont of the permuted view (a strided gather into dense rows)
        measure("cfg5", "cont_permuted", 2 * spec.ops[2].bytes, spec.ops[2].elements,
                lambda k: (lambda: chk(lib.emel_cuda_cont(ctx.handle, sh, B(v0), B(vd5)))), 1)
        del t0, t1, td
    # configuration 5 on one dim-3 slice: what each GPU holds at N=8 (134 MB
    # of src0); two shard copies alternate so no launch finds its input in L2
    if wants("cfg5_shard",):
        spec = W.cfg5_spec(ne3=1)
        ne1s, nb1s = W.cfg5_src0_view(ne3=1)
        sh0 = [torch.from_numpy(W.cfg5(ne3=1, shard=j)[0]).to(dev) for j in range(2)]
        t1 = torch.from_numpy(W.cfg5(ne3=1, shard=0)[1]).to(dev)
        outs = [torch.empty_like(sh0[0]) for _ in range(2)]
        v0s = [view(t, ne1s, nb1s) for t in sh0]
        vds = [view(t, ne1s) for t in outs]
        v1 = view(t1, [128, 1, 8192, 1])
        one = [1, 1, 1, 1]
        tsum, targ = torch.empty(1, device=dev), torch.empty(1, dtype=torch.int64, device=dev)
        vsum, varg = view(tsum, one), view(targ, one, code=27)
        for op, opname in ((2, "mul"), (0, "add")):
            measure("cfg5_shard", f"repeat_{opname}_slice", spec.ops[0].bytes, spec.ops[0].elements,
                    lambda k, op=op: (lambda: chk(lib.emel_cuda_binary_repeat(ctx.handle, sh, op, B(v0s[k]), B(v1),
                                                                               B(vds[k])))), 2)
        measure("cfg5_shard", "sum_slice", spec.ops[2].bytes, spec.ops[2].elements,
                lambda k: (lambda: chk(lib.emel_cuda_sum(ctx.handle, sh, B(v0s[k]), B(vsum)))), 2)
        measure("cfg5_shard", "argmax_slice", spec.ops[3].bytes, spec.ops[3].elements,
                lambda k: (lambda: chk(lib.emel_cuda_argmax(ctx.handle, sh, B(v0s[k]), B(varg)))), 2)
        del sh0, t1, outs
    # gated linear units (glu.rs) on configuration 2's feed-forward shape
    if wants("glu",):
        spec = W.glu_spec()
        xg = W.glu_ffn()
        sets = sets_for(spec.ops[0].bytes)
        tin = [torch.from_numpy(xg).to(dev) for _ in range(sets)]
        tout = [torch.empty(W.GLU_N, device=dev) for _ in range(sets)]
        for subop, o in enumerate(spec.ops):
            measure("glu", o.name, o.bytes, o.elements,
                    lambda k, subop=subop: (lambda: chk(lib.emel_cuda_glu(
                        ctx.handle, sh, subop, ctypes.c_void_p(tin[k].data_ptr()), 2 * W.GLU_N,
                        ctypes.c_void_p(tout[k].data_ptr()), W.GLU_N))), sets)
        del tin, tout
    # row gather (get_rows.rs): 8192 token rows of a [4096, 32000] table
    if wants("get_rows",):
        spec = W.emb_spec()
        tok = torch.from_numpy(W.emb_tokens()).to(dev)
        vidx = view(tok, [W.EMB_TOKENS, 1, 1, 1], code=26)
        for fmt, o in zip(W.EMB_FORMATS, spec.ops):
            if only and o.name not in only:
                continue
            data, ne, nb, code = W.emb_table(fmt)
            gather = lib.emel_cuda_get_rows_f32_bytes if fmt == "f32_bytes" else lib.emel_cuda_get_rows
            ttab = torch.from_numpy(data).to(dev)
            vtab = pkg.CView()
            vtab.data, vtab.storage_bytes, vtab.dtype = ttab.data_ptr(), ttab.numel(), code
            for d in range(4):
                vtab.ne[d], vtab.nb[d] = ne[d], nb[d]
            sets = sets_for(o.bytes)
            touts = [torch.empty(W.EMB_TOKENS * W.EMB_COLS, device=dev) for _ in range(sets)]
            vouts = [view(t, [W.EMB_COLS, W.EMB_TOKENS, 1, 1]) for t in touts]
            measure("get_rows", o.name, o.bytes, o.elements,
                    lambda k, vtab=vtab, vouts=vouts, fn=gather: (lambda: chk(fn(
                        ctx.handle, sh, B(vtab), B(vidx), B(vouts[k])))), sets)
            chk(lib.emel_cuda_stream_synchronize(ctx.handle, sh))
            del ttab, touts
    # rotary position embedding (rope.rs) of query rows
    if wants("rope",):
        spec = W.rope_spec()
        xr, pr_pos = W.rope_inputs()
        ne_r = list(W.ROPE_NE)
        sets = sets_for(spec.ops[0].bytes)
        txr = [torch.from_numpy(xr).to(dev) for _ in range(sets)]
        tyr = [torch.empty_like(t) for t in txr]
        tpos = torch.from_numpy(pr_pos).to(dev)
        vpos = view(tpos, [ne_r[2], 1, 1, 1], code=26)
        vxr = [view(t, ne_r) for t in txr]
        vyr = [view(t, ne_r) for t in tyr]
        for o, mode in zip(spec.ops, (2, 0)):
            prm = pkg.CRopeParams(n_dims=128, mode=mode, freq_base=10000.0, freq_scale=1.0, ext_factor=0.0,
                                  attn_factor=1.0)
            measure("rope", o.name, o.bytes, o.elements,
                    lambda k, prm=prm: (lambda: chk(lib.emel_cuda_rope(ctx.handle, sh, B(vxr[k]), B(vpos), B(vyr[k]),
                                                                         B(prm)))), sets)
        del txr, tyr
    # vocabulary matvec + argmax (matmul.rs OpMulMatArgmax)
    if not only or "matvec" in only or "mul_mat_argmax_vocab" in only:
        spec = W.mv_spec()
        lm, rv = W.mv_inputs()
        tl, tr = torch.from_numpy(lm).to(dev), torch.from_numpy(rv).to(dev)
        del lm
        tv = torch.empty(1, device=dev)
        ti = torch.empty(1, dtype=torch.int32, device=dev)
        vl, vr, vv = view(tl, [W.MV_K, W.MV_ROWS, 1, 1]), view(tr, [1, W.MV_K, 1, 1]), view(tv, [1, 1, 1, 1])
        o = spec.ops[0]
        measure("matvec", o.name, o.bytes, o.elements,
                lambda k: (lambda: chk(lib.emel_cuda_mul_mat_argmax(ctx.handle, sh, B(vl), B(vr), B(vv),
                                                                    ctypes.c_void_p(ti.data_ptr())))), 1)
        del tl, tr
    if not only or "matvec" in only or "mul_mat_argmax_q8_0_vocab" in only:
        o = W.mvq8_spec().ops[0]
        blob, rv = W.mvq8_inputs()
        tq, tr = torch.from_numpy(blob).to(dev), torch.from_numpy(rv).to(dev)
        del blob
        tv = torch.empty(1, device=dev)
        ti = torch.empty(1, dtype=torch.int32, device=dev)
        rb = W.MV_K // 32 * 34
        vq = view(tq, [W.MV_K, W.MV_ROWS, 1, 1], [1, rb, rb * W.MV_ROWS, rb * W.MV_ROWS], code=8)
        vr, vv = view(tr, [1, W.MV_K, 1, 1]), view(tv, [1, 1, 1, 1])
        measure("matvec", o.name, o.bytes, o.elements,
                lambda k: (lambda: chk(lib.emel_cuda_mul_mat_argmax_q8_0(ctx.handle, sh, B(vq), B(vr), B(vv),
                                                                         ctypes.c_void_p(ti.data_ptr())))), 1)
        del tq, tr
    for fmt, code in (("q2_k", 10), ("q3_k", 11), ("q4_k", 12), ("q6_k", 14)):
        o = W.mvk_spec(fmt)
        if only and "matvec" not in only and o.name not in only:
            continue
        blob, rv = W.mvk_inputs(fmt)
        tq, tr = torch.from_numpy(blob).to(dev), torch.from_numpy(rv).to(dev)
        del blob
        tv = torch.empty(1, device=dev)
        ti = torch.empty(1, dtype=torch.int32, device=dev)
        rb = W.MV_K // 256 * W.K_BLOCK_BYTES[fmt]
        vq = view(tq, [W.MV_K, W.MV_ROWS, 1, 1], [1, rb, rb * W.MV_ROWS, rb * W.MV_ROWS], code=code)
        vr, vv = view(tr, [1, W.MV_K, 1, 1]), view(tv, [1, 1, 1, 1])
        fn = getattr(lib, f"emel_cuda_mul_mat_argmax_{fmt}")
        measure("matvec", o.name, o.bytes, o.elements,
                lambda k, fn=fn, vq=vq, vr=vr, vv=vv, ti=ti: (lambda: chk(fn(ctx.handle, sh, B(vq), B(vr), B(vv),
                                                                           ctypes.c_void_p(ti.data_ptr())))), 1)
        del tq, tr
    # causal masks (diag.rs OpDiagMaskInf / OpDiagMaskZero) over a score matrix
    if wants("diag",):
        x = W.diag_inputs()
        n = x.size
        sets = sets_for(n * 8)
        tx = [torch.from_numpy(x).to(dev) for _ in range(sets)]
        ty = [torch.empty_like(t) for t in tx]
        del x
        ops = W.diag_spec().ops
        for o, mode in zip(ops[:2], (0, 1)):
            measure("diag", o.name, o.bytes, o.elements,
                    lambda k, mode=mode: (lambda: chk(lib.emel_cuda_diag_mask(
                        ctx.handle, sh, mode, ctypes.c_void_p(tx[k].data_ptr()), n,
                        ctypes.c_void_p(ty[k].data_ptr()), n, 0))), sets)
        # the mask fused with soft_max: one read of the kept triangle
        measure("diag", ops[2].name, ops[2].bytes, ops[2].elements,
                lambda k: (lambda: chk(lib.emel_cuda_soft_max_diag_mask_inf(
                    ctx.handle, sh, ctypes.c_void_p(tx[k].data_ptr()), n, ctypes.c_void_p(ty[k].data_ptr()), n, 0))),
                sets)
        del tx, ty
    # single-query attention (flash_attn.rs OpFlashAttnExt): one CTA per query
    # head runs the reference's per-token binary16 recurrence, so the time is
    # tokens x the recurrence's latency; ns_per_token reports that bound
    if wants("attention",):
        for o, tokens in zip(W.fa_spec().ops, W.FA_TOKENS):
            if not wants(o.name) and only:
                continue
            q, kh, vh = W.fa_inputs(tokens)
            sets = sets_for(o.bytes)
            tq = torch.from_numpy(q).to(dev)
            tk = [torch.from_numpy(kh.view(np.int16)).to(dev) for _ in range(sets)]
            tvv = [torch.from_numpy(vh.view(np.int16)).to(dev) for _ in range(sets)]
            to = torch.empty_like(tq)
            del kh, vh
            qne, kne = [W.FA_D, 1, W.FA_HEADS, 1], [W.FA_D, tokens, W.FA_KV_HEADS, 1]
            vq, vo = view(tq, qne), view(to, qne)
            vk = [view(t, kne, code=1) for t in tk]
            vv = [view(t, kne, code=1) for t in tvv]
            measure("attention", o.name, o.bytes, o.elements,
                    lambda k, vk=vk, vv=vv: (lambda: chk(lib.emel_cuda_flash_attn_ext(
                        ctx.handle, sh, B(vq), B(vk[k]), B(vv[k]), B(vo), None))), sets,
                    extra=lambda ms, tokens=tokens: {"ns_per_token": round(ms * 1e6 / tokens, 2),
                                                     "heads": W.FA_HEADS, "kv_heads": W.FA_KV_HEADS,
                                                     "head_dim": W.FA_D, "tokens": tokens})
            chk(lib.emel_cuda_stream_synchronize(ctx.handle, sh))
            del tk, tvv
    return out


# ---------------------------------------------------------------------------
# Configuration 5 sharded over the GPUs (strong scaling)
# ---------------------------------------------------------------------------
class Cfg5Shard:
    """This rank's dim-3 slices [b, e) of configuration 5's src0 (the
    dims-1/2-swapped view of contiguous [128, 8192, 32, 8]), the replicated
    src1 [128, 1, 8192, 1], the two repeat-broadcast outputs and the
    whole-tensor answers, all in device memory."""

    def __init__(self, pkg, ctx, torch, device, world, rank):
        from emel_rs_b200 import distributed as D
        from emel_rs_b200 import workloads as W

        self.pkg, self.ctx, self.torch, self.world, self.rank = pkg, ctx, torch, world, rank
        self.lib = pkg.lib()
        self.b, self.e = D.shard_bounds(W.CFG5_NE[3], world, rank)
        parts, s1 = [], None
        for j in range(self.b, self.e):
            s0, s1 = W.cfg5(ne3=1, shard=j)
            parts.append(s0)
        if s1 is None:  # more ranks than slices: this rank holds nothing
            _, s1 = W.cfg5(ne3=1, shard=0)
        self.host0 = np.concatenate(parts) if parts else np.empty(0, np.float32)
        self.host1 = s1
        self.src0 = torch.from_numpy(self.host0).to(device)
        self.src1 = torch.from_numpy(s1).to(device)
        self.ne, self.nb = W.cfg5_src0_view(ne3=self.e - self.b)
        self.mul_out = torch.empty_like(self.src0)
        self.add_out = torch.empty_like(self.src0)
        # exchange payload: the shard's f64 sum, then its argmax partial
        self.partial = torch.zeros(32, dtype=torch.uint8, device=device)
        self.gathered = torch.zeros(max(1, world) * 32, dtype=torch.uint8, device=device)
        self.sum_out = torch.zeros(1, dtype=torch.float32, device=device)
        self.idx_out = torch.zeros(1, dtype=torch.int64, device=device)
        self.v0 = self.view(self.src0, self.ne, self.nb)
        self.v1 = self.view(self.src1, [128, 1, 8192, 1])
        self.vm = self.view(self.mul_out, self.ne)
        self.va = self.view(self.add_out, self.ne)
        self.vsum = self.view(self.sum_out, [1, 1, 1, 1])
        self.vidx = self.view(self.idx_out, [1, 1, 1, 1], code=27)
        self.plane = self.ne[0] * self.ne[1] * self.ne[2]
        self.exchange = None
        n = 128 * 32 * 8192 * 8
        # algorithmic bytes of one step over the whole tensor (every rank's
        # shard): repeat mul and repeat add read src0 and src1 and write dst;
        # sum and argmax read src0
        self.op_bytes = {"repeat_mul": 2 * n * 4 + 128 * 8192 * 4, "repeat_add": 2 * n * 4 + 128 * 8192 * 4,
                         "sum": n * 4, "argmax": n * 4}
        self.step_bytes = sum(self.op_bytes.values())
        self.elements = n

    def view(self, t, vne, vnb=None, code=0):
        v = self.pkg.CView()
        v.data = t.data_ptr()
        v.storage_bytes = t.numel() * t.element_size()
        vnb = vnb or self.pkg.contiguous_nb(vne, code)
        for d in range(4):
            v.ne[d], v.nb[d] = vne[d], vnb[d]
        v.dtype = code
        return v

    def connect(self, dist):
        from emel_rs_b200 import distributed as D
        if self.world > 1:
            self.exchange = D.PeerExchange(self.pkg, self.ctx, dist, self.world, self.rank)
            # the publish runs on a side branch, beside the two broadcasts
            self.side = self.pkg.Stream(self.ctx)
            self.ev_fork, self.ev_join = self.pkg.CudaEvent(self.ctx), self.pkg.CudaEvent(self.ctx)

    def _ok(self, st, what):
        if st != 0:
            raise RuntimeError(f"{what}: status {st}: {self.ctx.last_error}")

    def step(self, sh):
        """One step on stream `sh`.  One GPU: OpSum, OpArgmax (exact i64
        index), repeat mul, repeat add.  N GPUs: the shard's f64 sum and
        argmax partial, published to every rank over NVLink on a side branch
        (forked after the partials, joined before the wait) while the two
        repeat broadcasts stream, then one wait that gathers every rank's
        partials and combines them on the device."""
        lib, h, B = self.lib, self.ctx.handle, ctypes.byref
        if self.exchange is None:
            self._ok(lib.emel_cuda_sum(h, sh, B(self.v0), B(self.vsum)), "sum")
            self._ok(lib.emel_cuda_argmax(h, sh, B(self.v0), B(self.vidx)), "argmax")
        else:
            p = self.partial.data_ptr()
            self._ok(lib.emel_cuda_sum_f64(h, sh, B(self.v0), ctypes.c_void_p(p)), "sum_f64")
            self._ok(lib.emel_cuda_argmax_partial_compute(h, sh, B(self.v0), self.b * self.plane,
                                                          ctypes.c_void_p(p + 8)), "argmax partial")
            self.ev_fork.record(sh)
            self.side.wait(self.ev_fork)
            self.exchange.publish(self.side.handle, p)
            self.ev_join.record(self.side.handle)
        self._ok(lib.emel_cuda_binary_repeat(h, sh, 2, B(self.v0), B(self.v1), B(self.vm)), "repeat mul")
        self._ok(lib.emel_cuda_binary_repeat(h, sh, 0, B(self.v0), B(self.v1), B(self.va)), "repeat add")
        if self.exchange is not None:
            self._ok(lib.emel_cuda_stream_wait_event(h, sh, self.ev_join.handle), "join")
            self._ok(lib.emel_cuda_exchange_wait_sum_argmax(h, sh, self.exchange.handle,
                                                            ctypes.c_void_p(self.gathered.data_ptr()),
                                                            B(self.vsum), B(self.vidx)), "exchange wait")

    def align(self, sh):
        """One untimed exchange round (publish + wait) on stream `sh`: every
        rank's stream leaves it within the exchange latency of the others, so
        a timed region that starts right after begins together on every GPU
        instead of when each host returns from its barrier."""
        if self.exchange is not None:
            self.exchange.publish(sh, self.partial.data_ptr())
            self.exchange.wait(sh, self.gathered.data_ptr())

    def answers(self):
        return float(self.sum_out.cpu()[0]), int(self.idx_out.cpu()[0])

    def calibration(self, stream, reps):
        """Per-op graphs: each op `reps` times back to back between two timed
        events, alternating between two copies of the shard so no launch
        finds its input in L2.  Returns (op, shard bytes, reps, graph, e0, e1)."""
        torch, pkg, lib, h, B = self.torch, self.pkg, self.lib, self.ctx.handle, ctypes.byref
        self.src0b = self.src0.clone()
        v0b = self.view(self.src0b, self.ne, self.nb)
        self._idx_scratch = torch.zeros(1, dtype=torch.int64, device=self.src0.device)
        sidx = self.view(self._idx_scratch, [1, 1, 1, 1], code=27)
        srcs, outs_m, outs_a = (self.v0, v0b), (self.vm, self.va), (self.va, self.vm)
        shard_bytes = {k: v * (self.e - self.b) // 8 for k, v in self.op_bytes.items()}
        ops = {
            "repeat_mul": lambda k: lib.emel_cuda_binary_repeat(h, stream.handle, 2, B(srcs[k % 2]), B(self.v1),
                                                                B(outs_m[k % 2])),
            "repeat_add": lambda k: lib.emel_cuda_binary_repeat(h, stream.handle, 0, B(srcs[k % 2]), B(self.v1),
                                                                B(outs_a[k % 2])),
            "sum": lambda k: lib.emel_cuda_sum(h, stream.handle, B(srcs[k % 2]), B(self.vsum)),
            "argmax": lambda k: lib.emel_cuda_argmax(h, stream.handle, B(srcs[k % 2]), B(sidx)),
        }
        out = []
        for name, fn in ops.items():
            e0, e1 = pkg.CudaEvent(self.ctx), pkg.CudaEvent(self.ctx)
            g = pkg.Graph(self.ctx, stream)
            with g:
                e0.record_timed(stream.handle)
                for k in range(reps):
                    self._ok(fn(k), name)
                e1.record_timed(stream.handle)
            out.append((name, shard_bytes[name], reps, g, e0, e1))
        return out

    def close(self):
        if self.exchange is not None:
            self.side.synchronize()
            self.exchange.close()
            self.exchange = None


def run_cfg5(args, world, rank, local):
    """Configuration 5, the default workload: the 1.07 GB permuted tensor
    split along dim 3 across the ranks (total work fixed: strong scaling).
    One step = whole-tensor sum and argmax, repeat mul and repeat add with
    the replicated src1, captured as one CUDA graph; with N GPUs the per-shard
    partials cross NVLink through the library's peer exchange and are
    combined on the device."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    pkg = load_package()
    ctx = pkg.Context(local)
    stream = pkg.Stream(ctx)
    sh = stream.handle
    shard = Cfg5Shard(pkg, ctx, torch, device, world, rank)
    shard.connect(dist)
    torch.cuda.synchronize()

    for _ in range(args.warmup):
        shard.step(sh)
    stream.synchronize()
    graph = pkg.Graph(ctx, stream)
    with graph:
        shard.step(sh)
    for _ in range(3):
        graph.launch()
    stream.synchronize()
    # The timed region: one graph holding an exchange round that aligns the
    # ranks (N > 1), the start event, the K steps back to back and the end
    # event, launched with one host call.  The device never waits on the
    # host inside it, and every rank's start event fires right after the
    # alignment, however late its host launched the graph (a host loop of K
    # launches, or host time between the alignment and the start event,
    # left GPUs idle and folded host skew into the max over ranks).
    t0, t1 = pkg.CudaEvent(ctx), pkg.CudaEvent(ctx)
    steps_graph = pkg.Graph(ctx, stream)
    with steps_graph:
        shard.align(sh)
        t0.record_timed(sh)
        for _ in range(args.steps):
            shard.step(sh)
        t1.record_timed(sh)
    steps_graph.launch()  # untimed: first replay of the new graph
    stream.synchronize()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    launches_before = ctx.launches
    with ClockSampler(local) as clocks:
        steps_graph.launch()
        stream.synchronize()
    steps_graph.close()
    # the alignment's two exchange kernels sit before the start event
    gpu_launches = ctx.launches - launches_before - (2 if shard.exchange is not None else 0)
    ms = t0.elapsed_ms(t1) / args.steps
    ms_t = torch.tensor([ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms = float(ms_t.item())
    total32, index = shard.answers()

    # per-op kernel time on this rank's shard, right after the timed region
    reps = 8
    per_op = {}
    for name, nbytes, r, g, e0, e1 in shard.calibration(stream, reps):
        d = []
        for _ in range(3):
            g.launch()
            stream.synchronize()
            d.append(e0.elapsed_ms(e1) / r)
        g.close()
        per_op[name] = (nbytes, statistics.median(d))
    e2e = None if args.no_e2e else run_cfg5_e2e(args, pkg, ctx, torch, shard, stream, world)
    graph.close()
    cfg2_ops = None
    if world == 1 and not args.no_cfg2:
        cfg2_ops = cfg2_per_op(pkg, ctx, torch, device, stream)

    if rank == 0:
        peak, peak_kind = peaks()
        dom_name, (dom_bytes, dom_ms) = max(per_op.items(), key=lambda kv: kv[1][1])
        kernel_ms = sum(t for _, t in per_op.values())
        achieved = dom_bytes / (dom_ms / 1e3) / 1e9
        traffic = profile_traffic("ew_rows_vec_cfg5_repeat_ncu.md")
        if traffic is not None:
            traffic = traffic * (shard.e - shard.b) // 8  # the profile covers the whole 8-slice tensor
        value = shard.step_bytes / (ms / 1e3) / 1e9
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 5), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded per dim-3 slice, N(0,1))",
            "config": {"workload": "cfg5: src0 f32 ne=[128,32,8192,8] stored as a view with dims 1 and 2 swapped "
                                   "(1.07 GB), split along dim 3 across the GPUs; src1 ne=[128,1,8192,1] "
                                   "replicated; one step = whole-tensor sum + argmax (exact i64 index), repeat "
                                   "mul, repeat add, one CUDA graph, ops serial on one stream; with N>1 the "
                                   "per-shard partials cross NVLink by peer stores (library kernels) and are "
                                   "combined on the device",
                       "bytes_per_step": shard.step_bytes, "elements": shard.elements,
                       "l2": "inputs larger than L2: the shard (1.07 GB / N) plus its two outputs exceed the "
                             "126 MB L2 at every N up to 8",
                       "parallelism": f"dim-3 shards over {world} GPU(s)",
                       "slices_per_gpu": shard.e - shard.b},
            "result": {"sum": total32, "argmax": index},
            "roofline": {"bound": "hbm", "kernel": f"ew_rows_vec ({dom_name})" if dom_name.startswith("repeat")
                         else dom_name, "achieved": round(achieved, 1), "peak": peak,
                         "peak_source": f"{peak_kind} hbm_gbs (burst copy)", "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic,
                         "algorithmic_bytes_per_launch": dom_bytes, "launch_ms": round(dom_ms, 5),
                         "share_of_step": round(dom_ms / kernel_ms, 4)},
            "per_op_gbs": {k: round(b / (t / 1e3) / 1e9, 1) for k, (b, t) in per_op.items()},
            "per_op_us": {k: round(t * 1e3, 2) for k, (_, t) in per_op.items()},
            "e2e": e2e,
            "gpu_launches": gpu_launches,
            "clocks": clocks.summary(),
        }
        if cfg2_ops is not None:
            line["cfg2_per_op_gbs"] = cfg2_ops
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline_cfg5(args)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()  # every rank's last wait is done: the peer buffers may go
        shard.close()
        dist.barrier()
        dist.destroy_process_group()


def run_cfg5_breakdown(args, world, rank, local):
    """Where one rank's configuration-5 step goes (`--breakdown`): the step,
    the step without the exchange, the exchange alone, one kernel alone, each
    captured as a CUDA graph and replayed K times (device time per replay),
    and one replay with an event node between consecutive kernels (the
    parts; the nodes stop the programmatic overlap, so they add up to more
    than the step).  Every rank prints one JSON line."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    pkg = load_package()
    ctx = pkg.Context(local)
    stream = pkg.Stream(ctx)
    sh = stream.handle
    shard = Cfg5Shard(pkg, ctx, torch, device, world, rank)
    shard.connect(dist)
    torch.cuda.synchronize()
    lib, h, B = shard.lib, ctx.handle, ctypes.byref

    def partials():
        p = shard.partial.data_ptr()
        shard._ok(lib.emel_cuda_sum_f64(h, sh, B(shard.v0), ctypes.c_void_p(p)), "sum_f64")
        shard._ok(lib.emel_cuda_argmax_partial_compute(h, sh, B(shard.v0), shard.b * shard.plane,
                                                       ctypes.c_void_p(p + 8)), "argmax partial")

    def broadcasts():
        mul_only()
        shard._ok(lib.emel_cuda_binary_repeat(h, sh, 0, B(shard.v0), B(shard.v1), B(shard.va)), "repeat add")

    def exchange():
        if shard.exchange is not None:
            shard.align(sh)

    def no_exchange():
        partials()
        broadcasts()

    evs = [pkg.CudaEvent(ctx) for _ in range(7)]

    def parts():
        p = shard.partial.data_ptr()
        evs[0].record_timed(sh)
        shard._ok(lib.emel_cuda_sum_f64(h, sh, B(shard.v0), ctypes.c_void_p(p)), "sum_f64")
        evs[1].record_timed(sh)
        shard._ok(lib.emel_cuda_argmax_partial_compute(h, sh, B(shard.v0), shard.b * shard.plane,
                                                       ctypes.c_void_p(p + 8)), "argmax partial")
        evs[2].record_timed(sh)
        if shard.exchange is not None:
            shard.exchange.publish(sh, p)
        evs[3].record_timed(sh)
        shard._ok(lib.emel_cuda_binary_repeat(h, sh, 2, B(shard.v0), B(shard.v1), B(shard.vm)), "repeat mul")
        evs[4].record_timed(sh)
        shard._ok(lib.emel_cuda_binary_repeat(h, sh, 0, B(shard.v0), B(shard.v1), B(shard.va)), "repeat add")
        evs[5].record_timed(sh)
        if shard.exchange is not None:
            shard._ok(lib.emel_cuda_exchange_wait_sum_argmax(h, sh, shard.exchange.handle,
                                                            ctypes.c_void_p(shard.gathered.data_ptr()),
                                                            B(shard.vsum), B(shard.vidx)), "exchange wait")
        evs[6].record_timed(sh)

    res = {"rank": rank, "world": world, "replays": args.steps}
    def mul_only():
        shard._ok(lib.emel_cuda_binary_repeat(h, sh, 2, B(shard.v0), B(shard.v1), B(shard.vm)), "repeat mul")

    variants = (("step", lambda: shard.step(sh)), ("no_exchange", no_exchange), ("exchange_only", exchange),
                ("repeat_mul_only", mul_only), ("parts", parts))
    for name, fn in variants:
        for _ in range(3):
            fn()
        stream.synchronize()
        g = pkg.Graph(ctx, stream)
        with g:
            fn()
        t0, t1 = pkg.CudaEvent(ctx), pkg.CudaEvent(ctx)
        for _ in range(3):
            g.launch()
        stream.synchronize()
        if world > 1:
            dist.barrier()
        shard.align(sh)
        t0.record(sh)
        for _ in range(args.steps):
            g.launch()
        t1.record(sh)
        stream.synchronize()
        res[f"{name}_us"] = round(t0.elapsed_ms(t1) / args.steps * 1e3, 2)
        if name == "parts":
            g.launch()
            stream.synchronize()
            res["parts_us"] = dict(zip(("sum", "argmax", "publish", "repeat_mul", "repeat_add", "wait"),
                                       (round(evs[i].elapsed_ms(evs[i + 1]) * 1e3, 2) for i in range(6))))
        g.close()
        if world > 1:
            dist.barrier()
    print(json.dumps(res), flush=True)
    if world > 1:
        dist.barrier()
        shard.close()
        dist.barrier()
        dist.destroy_process_group()


def run_cfg5_e2e(args, pkg, ctx, torch, shard, stream, world):
    """The same step through the C ABI with host buffers: every step copies
    this rank's src0 shard and src1 from pinned host memory, runs the step,
    and reads both outputs and the two whole-tensor answers back into pinned
    host memory.  Copies in and out run on their own streams so one step's
    upload overlaps the previous step's download (PCIe is full duplex);
    the step's kernels wait for its upload and for the previous download
    of the outputs they overwrite."""
    lib, h = pkg.lib(), ctx.handle
    up, down = pkg.Stream(ctx), pkg.Stream(ctx)
    sh = stream.handle
    hs0 = torch.from_numpy(shard.host0).pin_memory()
    hs1 = torch.from_numpy(shard.host1).pin_memory()
    hm = torch.empty(shard.mul_out.shape, dtype=torch.float32, pin_memory=True)
    ha = torch.empty(shard.add_out.shape, dtype=torch.float32, pin_memory=True)
    hsum = torch.empty(1, dtype=torch.float32, pin_memory=True)
    hidx = torch.empty(1, dtype=torch.int64, pin_memory=True)
    ins = [(shard.src0, hs0), (shard.src1, hs1)]
    outs = [(hm, shard.mul_out), (ha, shard.add_out), (hsum, shard.sum_out), (hidx, shard.idx_out)]
    h2d = sum(t.numel() * t.element_size() for _, t in ins)
    d2h = sum(t.numel() * t.element_size() for t, _ in outs)
    uploaded, computed, downloaded = pkg.CudaEvent(ctx), pkg.CudaEvent(ctx), pkg.CudaEvent(ctx)
    first = [True]

    def one():
        if not first[0]:
            up.wait(computed)  # the previous step has read src0
        for d, hh in ins:
            st = lib.emel_cuda_memcpy_h2d(h, up.handle, d.data_ptr(), hh.data_ptr(), hh.numel() * hh.element_size())
            if st != 0:
                raise RuntimeError(ctx.last_error)
        uploaded.record(up.handle)
        stream.wait(uploaded)
        if not first[0]:
            stream.wait(downloaded)  # the previous step's outputs are home
        shard.step(sh)
        computed.record(sh)
        down.wait(computed)
        for hh, d in outs:
            st = lib.emel_cuda_memcpy_d2h(h, down.handle, hh.data_ptr(), d.data_ptr(), hh.numel() * hh.element_size())
            if st != 0:
                raise RuntimeError(ctx.last_error)
        downloaded.record(down.handle)
        first[0] = False

    steps = max(3, min(args.steps, 10))
    for _ in range(2):
        one()
    up.synchronize()
    down.synchronize()
    stream.synchronize()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    t0, t1 = pkg.CudaEvent(ctx), pkg.CudaEvent(ctx)
    shard.align(sh)
    t0.record(sh)
    up.wait(t0)
    for _ in range(steps):
        one()
    stream.wait(downloaded)
    t1.record(sh)
    stream.synchronize()
    ms = t0.elapsed_ms(t1)
    if world > 1:
        import torch.distributed as dist
        m = torch.tensor([ms], dtype=torch.float64, device=shard.src0.device)
        dist.all_reduce(m, op=dist.ReduceOp.MAX)
        ms = float(m.item())
    got = (float(hsum[0]), int(hidx[0]))
    up.close()
    down.close()
    value = steps * shard.step_bytes / (ms / 1e3) / 1e9
    return {"value": round(value, 2), "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "steps": steps, "result": {"sum": got[0], "argmax": got[1]},
            "path": "per step: emel_cuda_memcpy_h2d of the src0 shard and src1 (pinned host) on an upload stream, "
                    "the step's entry points, emel_cuda_memcpy_d2h of both outputs, the sum and the argmax on a "
                    "download stream (per-rank bytes; upload of step s+1 overlaps download of step s)"}


def cfg2_per_op(pkg, ctx, torch, device, stream):
    """Configuration 2's 16 unary ops, one GB/s figure each (every op over
    eight distinct buffer pairs of its dtype, back to back, between two
    events)."""
    step = Cfg2Step(pkg, ctx, torch, device, seed=2)
    torch.cuda.synchronize()
    out = {}
    for name, nbytes, reps, g, e0, e1 in step.calibration_graphs(stream):
        d = []
        for _ in range(3):
            g.launch()
            stream.synchronize()
            d.append(e0.elapsed_ms(e1) / reps)
        g.close()
        out[name] = round(nbytes / (statistics.median(d) / 1e3) / 1e9, 1)
    return out


# ---------------------------------------------------------------------------
# CPU lanes (the oracle: C restatement of the reference loops)
# ---------------------------------------------------------------------------
class Cfg5Sample:
    """A bounded CPU sample of configuration 5: dim-2 rows [0, rows) of
    dim-3 slice 0 of src0 (the same permuted view), the matching rows of
    src1, and dense outputs; each part [r0, r1) of the rows is one
    independent unit of the four ops (repeat mul, repeat add, f64 sum,
    argmax with its ordinal base)."""

    def __init__(self, rows):
        sys.path.insert(0, str(ROOT / "oracle"))
        import oracle
        load_package()  # the seeded input generator lives in the package
        from emel_rs_b200 import workloads as W
        self.oracle = oracle
        self.lib = oracle.load()
        self.rows = rows
        s0, s1 = W.cfg5(ne3=1, shard=0)
        self.s0 = np.ascontiguousarray(s0)
        self.s1 = np.ascontiguousarray(s1)
        self.mul = np.empty((rows, 32, 128), np.float32)
        self.add = np.empty((rows, 32, 128), np.float32)

    def bytes_of(self, rows):
        n = rows * 32 * 128
        return 2 * (2 * n * 4 + rows * 128 * 4) + 2 * n * 4

    def run(self, r0, r1):
        """The four ops on rows [r0, r1); returns (f64 sum, (value, index, has))."""
        o, L, B = self.oracle, self.lib, ctypes.byref
        s = r1 - r0
        nb0 = [4, 4 * 128 * 8192, 512, 4 * 128 * 8192 * 32]
        base0 = self.s0.ctypes.data + r0 * 512
        span0 = self.s0.nbytes - r0 * 512
        v0 = o.make_view(base0, span0, [128, 32, s, 1], nb0, 0)
        v1 = o.make_view(self.s1.ctypes.data + r0 * 512, (8192 - r0) * 512, [128, 1, s, 1], [4, 512, 512, 512 * s], 0)
        out_nb = [4, 512, 512 * 32, 512 * 32 * s]
        vm = o.make_view(self.mul.ctypes.data + r0 * 32 * 512, s * 32 * 512, [128, 32, s, 1], out_nb, 0)
        va = o.make_view(self.add.ctypes.data + r0 * 32 * 512, s * 32 * 512, [128, 32, s, 1], out_nb, 0)
        assert L.oracle_binary_repeat(2, B(v0), B(v1), B(vm)) == 0
        assert L.oracle_binary_repeat(0, B(v0), B(v1), B(va)) == 0
        acc = ctypes.c_double()
        assert L.oracle_sum_f64(B(v0), B(acc)) == 0
        idx, val = ctypes.c_int64(), ctypes.c_float()
        assert L.oracle_argmax_index(B(v0), B(idx), B(val)) == 0
        return acc.value, (val.value, idx.value + r0 * 32 * 128)


def cpu_baseline_cfg5(args):
    """Single-thread oracle (the reference's kernels are single-threaded) on
    a time-bounded sample of configuration 5: repeated passes of the four
    ops over the first 512 dim-2 rows of dim-3 slice 0."""
    rows = 512
    sample = Cfg5Sample(rows)
    done, passes, t0 = 0, 0, time.perf_counter()
    while True:
        sample.run(0, rows)
        done += sample.bytes_of(rows)
        passes += 1
        if time.perf_counter() - t0 >= args.cpu_seconds:
            break
    dt = time.perf_counter() - t0
    return {"value": round(done / dt / 1e9, 3), "unit": UNIT, "cores": 1, "kind": "port",
            "sample": f"{passes} pass(es) of repeat mul + repeat add + sum + argmax over dim-2 rows [0, {rows}) of "
                      f"dim-3 slice 0 (1/{8 * 8192 // rows} of the cfg5 tensor) in {dt:.1f} s, single thread, "
                      f"C restatement of the emel-kernels loops (reference Rust not buildable offline)",
            "cpu_model": cpu_model()}


def run_reference_cfg5(args, world, rank):
    """CPU reference lane for configuration 5: the oracle (the C restatement
    of the emel-kernels loops; the reference's Rust is not buildable offline)
    on every host thread.  Each step is a bounded sample: the four ops over
    the first `rows` dim-2 rows of slice 0, the rows split across threads
    (ctypes releases the GIL), partial sums added and argmax partials folded
    in row order -- the same metric, unit and direction as the B200 arm."""
    if rank != 0:
        return
    from concurrent.futures import ThreadPoolExecutor
    threads = host_threads()
    pool = ThreadPoolExecutor(max_workers=threads)
    probe = Cfg5Sample(8192)

    def step(rows):
        chunk = max(1, -(-rows // threads))
        futs = [pool.submit(probe.run, r0, min(rows, r0 + chunk)) for r0 in range(0, rows, chunk)]
        total, best = 0.0, None
        for f in futs:
            s, (v, i) = f.result()
            total += s
            if best is None or v > best[0]:
                best = (v, i)
        return probe.bytes_of(rows)

    rows = max(threads, 256)
    t = time.perf_counter()
    step(rows)
    per_row = (time.perf_counter() - t) / rows
    # size each step so warmup + steps stay within the time budget
    rows = int(min(8192, max(threads, args.ref_seconds / max(1e-9, per_row * (args.steps + args.warmup)))))
    for _ in range(args.warmup):
        step(rows)
    t = time.perf_counter()
    done = 0
    for _ in range(args.steps):
        done += step(rows)
    dt = time.perf_counter() - t
    value = done / dt / 1e9
    frac = rows / (8 * 8192)
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3 / args.steps, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded per dim-3 slice, N(0,1))",
        "config": {"workload": "cfg5 (same ops, tensors and view as the B200 arm): whole-tensor sum + argmax, "
                               "repeat mul, repeat add on the dims-1/2-swapped view of [128,32,8192,8]",
                   "sample_rows_per_step": rows, "sample_fraction_per_step": round(frac, 6)},
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"dim-2 rows [0, {rows}) of dim-3 slice 0 per step ({frac:.5f} of the tensor), "
                                   f"{threads} threads", "cpu_model": cpu_model()},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def cpu_workload():
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle
    pkg = load_package()
    from emel_rs_b200 import workloads
    x, xa = workloads.cfg2(2)
    bufs = []
    items = []
    ne = [workloads.CFG2_NE[0], workloads.CFG2_NE[1], 1, 1]
    for dt, code in ((np.float32, 0), (np.float16, 1)):
        xs, xas = x.astype(dt), xa.astype(dt)
        for name, op in OPS:
            src = xas if name in ("sqrt", "pow2") else xs
            dst = np.empty_like(src)
            bufs += [src, dst]
            nb = pkg.contiguous_nb(ne, code)
            sv = oracle.make_view(src.ctypes.data, src.nbytes, ne, nb, code)
            dv = oracle.make_view(dst.ctypes.data, dst.nbytes, ne, nb, code)
            items.append((op, sv, dv, 2 * src.nbytes))
    return oracle.load(), items, bufs, x.size


def cpu_baseline_single(args):
    """Single-thread oracle (the reference's kernels are single-threaded) on a
    time-bounded sample: whole 16-op passes over the cfg2 tensors."""
    lib, items, bufs, n = cpu_workload()
    done_bytes, t0 = 0, time.perf_counter()
    passes = 0
    while True:
        for op, sv, dv, nbytes in items:
            lib.oracle_unary_range(op, ctypes.byref(sv), ctypes.byref(dv), 0, n)
            done_bytes += nbytes
        passes += 1
        if time.perf_counter() - t0 >= args.cpu_seconds:
            break
    dt = time.perf_counter() - t0
    return {"value": round(done_bytes / dt / 1e9, 3), "unit": UNIT, "cores": 1, "kind": "port",
            "sample": f"{passes} full cfg2 step(s) (16 ops x 7340032 elements) in {dt:.1f} s, single thread, "
                      f"C restatement of the emel-kernels loops (reference Rust not buildable offline)",
            "cpu_model": cpu_model()}


def cpu_model():
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except Exception:
        pass
    return "unknown"


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def run_reference(args, world, rank):
    """CPU reference lane: the oracle on all host threads (rows split across
    threads; ctypes releases the GIL), same metric and workload."""
    if rank != 0:
        return
    from concurrent.futures import ThreadPoolExecutor
    lib, items, bufs, n = cpu_workload()
    threads = host_threads()
    pool = ThreadPoolExecutor(max_workers=threads)

    def step(frac):
        count = max(threads, int(n * frac))
        chunk = (count + threads - 1) // threads
        done = 0
        for op, sv, dv, nbytes in items:
            futs = [pool.submit(lib.oracle_unary_range, op, ctypes.byref(sv), ctypes.byref(dv), b,
                                min(b + chunk, count)) for b in range(0, count, chunk)]
            for f in futs:
                f.result()
            done += nbytes * count // n
        return done

    t = time.perf_counter()
    step(1.0)
    full = time.perf_counter() - t
    # size each step so warmup + steps stay within the time budget
    frac = min(1.0, args.ref_seconds / max(1e-9, full * (args.steps + args.warmup)))
    for _ in range(args.warmup):
        step(frac)
    t = time.perf_counter()
    done = 0
    for _ in range(args.steps):
        done += step(frac)
    dt = time.perf_counter() - t
    value = done / dt / 1e9
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3 / args.steps, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32+f16",
        "data": "synthetic (seeded)",
        "config": {"workload": "cfg2 unary/activation sweep (same ops and tensors as the B200 arm)",
                   "sample_fraction_per_step": round(frac, 5)},
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{frac:.4f} of the cfg2 elements per op per step, {threads} threads",
                         "cpu_model": cpu_model()},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--ref-seconds", type=float, default=60.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true", help="skip the host-buffer end-to-end measurement")
    ap.add_argument("--only", default="", help="comma list of ops to run, e.g. gelu_f32,relu_f16 (profiling; with --suite: suite op names)")
    ap.add_argument("--branches", type=int, default=4, help="parallel graph branches for the 16 independent ops")
    ap.add_argument("--suite", action="store_true", help="per-op lines for every configuration (1 GPU)")
    ap.add_argument("--workload", choices=["cfg2", "cfg5"], default="cfg5",
                    help="cfg5 (default): the 4-D broadcast + whole-tensor reductions sharded along dim 3 "
                         "(strong scaling); cfg2: the 16-op unary sweep on independent per-GPU batches")
    ap.add_argument("--no-cfg2", action="store_true", help="cfg5 at N=1: skip the extra cfg2 per-op figures")
    ap.add_argument("--breakdown", action="store_true",
                    help="cfg5: per-rank step breakdown (step, without exchange, exchange alone, parts), K replays")
    args = ap.parse_args()
    world, rank, local = dist_env()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        if args.workload == "cfg5":
            run_reference_cfg5(args, world, rank)
        else:
            run_reference(args, world, rank)
        return
    if args.suite:
        run_suite(args)
        return
    if args.breakdown:
        run_cfg5_breakdown(args, world, rank, local)
        return
    if args.workload == "cfg5":
        run_cfg5(args, world, rank, local)
        return
    run_b200(args, world, rank, local)


if __name__ == "__main__":
    main()
