"""Pins the CPU oracle to the reference's golden parity manifests and known-answer
unit tests (no GPU needed)."""

import ctypes

import numpy as np
import pytest

import golden_runner as gr
import oracle

CASES = gr.load_cases()


def run_oracle(lib, case):
    bufs, views = {}, {}
    for name, spec in case["inputs"].items():
        arr = gr.host_array(spec)
        bufs[name] = arr
        views[name] = oracle.make_view(arr.ctypes.data, arr.nbytes, spec["ne"], spec["nb"], 0)
    o = case["output"]
    out = gr.host_array(o)
    dst = oracle.make_view(out.ctypes.data, out.nbytes, o["ne"], o["nb"], 0)
    p = case["params"]
    op = case["op"]
    r = ctypes.byref
    if op == "binary":
        st = lib.oracle_binary(p["op"], r(views["lhs"]), r(views["rhs"]), r(dst))
    elif op == "broadcast_row":
        st = lib.oracle_broadcast_row(p["op"], r(views["src0"]), r(views["src1"]), r(dst))
    elif op == "unary":
        st = lib.oracle_unary(p["op"], r(views["src"]), r(dst))
    elif op == "op_unary":
        st = lib.oracle_op_unary(p["op"], r(views["src"]), r(dst))
    elif op == "copy":
        st = lib.oracle_copy(r(views["src"]), r(dst))
    elif op == "scale":
        st = lib.oracle_scale(r(views["src"]), r(dst), p["scale"])
    elif op == "clamp":
        st = lib.oracle_clamp(r(views["src"]), r(dst), p["min"], p["max"])
    elif op == "leaky_relu":
        st = lib.oracle_leaky_relu(r(views["src"]), r(dst), p["slope"])
    elif op == "silu_back":
        st = lib.oracle_silu_back(r(views["src"]), r(views["grad"]), r(dst))
    elif op == "norm":
        st = lib.oracle_norm(r(views["src"]), r(dst), p["eps"])
    elif op == "rms_norm":
        st = lib.oracle_rms_norm(r(views["src"]), r(dst), p["eps"])
    elif op == "soft_max":
        st = lib.oracle_soft_max(r(views["src"]), r(dst))
    elif op == "sum":
        st = lib.oracle_sum(r(views["src"]), r(dst))
    elif op == "mean":
        st = lib.oracle_mean(r(views["src"]), r(dst))
    elif op == "sum_rows":
        st = lib.oracle_sum_rows(r(views["src"]), r(dst))
    elif op == "argmax":
        st = lib.oracle_argmax(r(views["src"]), r(dst))
    else:
        raise AssertionError(f"unknown op {op}")
    return st, out


@pytest.mark.parametrize("case", CASES, ids=[f"{c['suite']}::{c['case']}" for c in CASES])
def test_oracle_reproduces_reference_golden(oracle_lib, case):
    st, out = run_oracle(oracle_lib, case)
    problems = gr.check_case(case, st, out)
    assert not problems, f"{case['source']}: {problems}"


def test_oracle_libm_cases_are_bit_exact_where_the_host_libm_allows(oracle_lib):
    """The reference tolerates 4 ulp on libm-backed unary ops; record how close
    glibc gets (informational bound: at most 1 ulp here)."""
    worst = 0
    for case in CASES:
        if case["compare"] != "ulp4" or case["expect_status"] != "ok":
            continue
        st, out = run_oracle(oracle_lib, case)
        assert st == 0
        bits = [int(b) for b in out.view(np.uint32)] if case["readout"] == "storage" else gr.logical_bits(
            out, case["output"]["ne"], case["output"]["nb"])
        worst = max(worst, int(gr.ulp_distance(bits, case["expect_bits"]).max()))
    assert worst <= 1


def test_fp16_conversions_match_ieee_round_to_nearest_even(oracle_lib):
    """The reference's binary16 helpers (unary.rs:546-586) are IEEE RNE for
    every non-NaN f32; check them against numpy's conversion on a sweep."""
    rng = np.random.default_rng(0)
    bits = np.concatenate([rng.integers(0, 2**32, 20000, dtype=np.uint64).astype(np.uint32),
                           np.arange(0x33000000, 0x33000000 + 4096, dtype=np.uint32),
                           np.arange(0x477fe000, 0x47800100, dtype=np.uint32)])
    vals = bits.view(np.float32)
    vals = vals[~np.isnan(vals)]
    with np.errstate(over="ignore"):
        want = vals.astype(np.float16).view(np.uint16)
    got = np.array([oracle_lib.oracle_fp32_to_fp16(float(v)) for v in vals], dtype=np.uint16)
    assert np.array_equal(got, want)
    halves = np.arange(0, 65536, dtype=np.uint32).astype(np.uint16)
    hv = halves.view(np.float16)
    keep = ~np.isnan(hv)
    back = np.array([oracle_lib.oracle_fp16_to_fp32(int(h)) for h in halves[keep]], dtype=np.float32)
    assert np.array_equal(back.view(np.uint32), hv[keep].astype(np.float32).view(np.uint32))
