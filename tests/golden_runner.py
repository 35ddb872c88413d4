"""Runs the reference's golden parity cases (tests/golden/reference_parity.json)
against a backend: the CPU oracle or the CUDA library through its C ABI."""

import json
from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden" / "reference_parity.json"

STATUS_NAMES = {0: "ok", 1: "invalid_view", 2: "shape_mismatch", 3: "invalid_parameters", 4: "unexpected_event",
                18: "invalid_argument"}


def load_cases():
    return json.loads(GOLDEN.read_text())["cases"]


def host_array(spec):
    if spec["bits"]:
        return np.array(spec["values"], dtype=np.uint32).view(np.float32).copy()
    return np.array(spec["values"], dtype=np.float32)


def effective_strides(ne, nb, elem=4):
    if nb[0] != 0:
        return list(nb)
    s = [elem]
    for d in range(1, 4):
        s.append(s[-1] * ne[d - 1])
    return s


def logical_bits(storage, ne, nb):
    """tools/emel-kernel-binary-parity/src/main.rs:25-52: read every logical
    ordinal of a view through its strides."""
    s = effective_strides(ne, nb)
    raw = storage.view(np.uint32)
    count = int(np.prod(ne))
    outv = []
    for ordinal in range(count):
        rem, off = ordinal, 0
        for d in range(4):
            off += (rem % ne[d]) * s[d]
            rem //= ne[d]
        outv.append(int(raw[off // 4]))
    return outv


def ulp_distance(a_bits, b_bits):
    def ordered(u):
        u = np.int64(u)
        return np.where(u & 0x80000000, 0x80000000 - (u & 0x7FFFFFFF), u + 0x80000000)
    return np.abs(ordered(np.array(a_bits, dtype=np.int64)) - ordered(np.array(b_bits, dtype=np.int64)))


def check_case(case, status, out_storage):
    """Returns a list of mismatch descriptions (empty when the case passes)."""
    problems = []
    expect = case["expect_status"]
    got = STATUS_NAMES.get(status, f"status{status}")
    if expect == "ok":
        if got != "ok":
            problems.append(f"status {got}, expected ok")
            return problems
    elif expect == "rejected":
        if got == "ok":
            problems.append("accepted a request the reference rejects")
    elif got != expect:
        problems.append(f"status {got}, expected {expect}")
    if case["readout"] == "none" or case["expect_bits"] is None:
        return problems
    o = case["output"]
    if case["readout"] == "logical":
        bits = logical_bits(out_storage, o["ne"], o["nb"])
    else:
        bits = [int(b) for b in out_storage.view(np.uint32)]
    want = case["expect_bits"]
    if len(bits) != len(want):
        problems.append(f"readout length {len(bits)} != {len(want)}")
        return problems
    if case["compare"] == "exact":
        if bits != want:
            problems.append("bits " + ",".join(f"{b:08x}" for b in bits) + " != " + ",".join(f"{b:08x}" for b in want))
    else:
        d = ulp_distance(bits, want)
        if int(d.max()) > 4:
            problems.append(f"ulp distance {d.tolist()} exceeds 4")
    return problems
