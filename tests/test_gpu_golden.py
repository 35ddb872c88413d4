"""The reference's golden parity cases, run through the CUDA path (C ABI ->
sm_100a kernels) and compared with the reference manifests' bits."""

import numpy as np
import pytest

import golden_runner as gr

pytestmark = pytest.mark.gpu

CASES = gr.load_cases()


@pytest.fixture(scope="module")
def kern(emel):
    return emel.Kernel(device=0, synchronize=True)


def run_cuda(pkg, kern, case):
    ctx = kern.ctx
    bufs = []

    def dev_view(spec, arr):
        b = pkg.DeviceBuffer(ctx, max(arr.nbytes, 4))
        if arr.nbytes:
            b.upload(arr)
        bufs.append(b)
        return pkg.TensorView(b.ptr, arr.nbytes, pkg.Layout.new(pkg.DType.F32, spec["ne"], spec["nb"]))

    views = {name: dev_view(spec, gr.host_array(spec)) for name, spec in case["inputs"].items()}
    o = case["output"]
    out_host = gr.host_array(o)
    dst = dev_view(o, out_host)
    p = case["params"]
    op = case["op"]
    if op == "binary":
        ev = [pkg.OpAdd, pkg.OpSub, pkg.OpMul, pkg.OpDiv][p["op"]](views["lhs"], views["rhs"], dst)
    elif op == "broadcast_row":
        ev = [pkg.OpAddBroadcastRow, pkg.OpSubBroadcastRow, pkg.OpMulBroadcastRow, pkg.OpDivBroadcastRow][p["op"]](
            views["src0"], views["src1"], dst)
    elif op == "unary":
        ev = pkg.OpUnaryTyped(pkg.UnaryOp(p["op"]), views["src"], dst)
    elif op == "op_unary":
        ev = pkg.OpUnary(pkg.UnaryOp(p["op"]), views["src"], dst)
    elif op == "copy":
        ev = pkg.CopyTensor(views["src"], dst)
    elif op == "scale":
        ev = pkg.OpScale(views["src"], dst, p["scale"])
    elif op == "clamp":
        ev = pkg.OpClamp(views["src"], dst, p["min"], p["max"])
    elif op == "leaky_relu":
        ev = pkg.OpLeakyRelu(views["src"], dst, p["slope"])
    elif op == "silu_back":
        ev = pkg.OpSiluBack(views["src"], views["grad"], dst)
    elif op == "norm":
        ev = pkg.OpNorm(views["src"], dst, p["eps"])
    elif op == "rms_norm":
        ev = pkg.OpRmsNorm(views["src"], dst, p["eps"])
    elif op == "soft_max":
        ev = pkg.OpSoftMax(views["src"], dst)
    elif op in ("sum", "mean", "sum_rows", "argmax"):
        ev = {"sum": pkg.OpSum, "mean": pkg.OpMean, "sum_rows": pkg.OpSumRows, "argmax": pkg.OpArgmax}[op](
            views["src"], dst)
    else:
        raise AssertionError(op)
    st = kern.process_event(ev)
    got = np.empty_like(out_host)
    if out_host.nbytes:
        bufs[-1].download(got)
    for b in bufs:
        b.free()
    return int(st), got


@pytest.mark.parametrize("case", CASES, ids=[f"{c['suite']}::{c['case']}" for c in CASES])
def test_cuda_reproduces_reference_golden(emel, kern, case):
    st, out = run_cuda(emel, kern, case)
    problems = gr.check_case(case, st, out)
    assert not problems, f"{case['source']}: {problems} ({kern.ctx.last_error})"
