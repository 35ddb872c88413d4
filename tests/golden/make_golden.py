"""Generate tests/golden/reference_parity.json from the reference's own evidence.

Run once in a container that has the reference checkout (read-only):

    python tests/golden/make_golden.py <emel.rs checkout>

Expected output bits and statuses are parsed from the reference's committed
parity manifests (snapshots/parity/<suite>/manifest.txt).  The inputs and
layouts that produced them are restated from the observer programs that
printed those manifests (tools/emel-kernel-*-parity/src/main.rs, cited per
case) and from the known-answer unit tests (crates/emel-kernels/tests/any/).
Nothing under the reference is read at test time: the JSON is the fixture.
"""

import json
import struct
import sys
from pathlib import Path

SENTINEL = 0x7FC00001


def f32_bits(x):
    return struct.unpack("<I", struct.pack("<f", x))[0]


def view(values, ne, nb, dtype="f32", bits=False):
    """A host buffer: `values` are f32 numbers (or raw bit patterns)."""
    return {"values": [int(v) for v in values] if bits else [float(v) for v in values],
            "bits": bits, "ne": list(ne), "nb": list(nb), "dtype": dtype}


def contiguous_nb(ne, elem=4):
    nb = [elem]
    for d in range(1, 4):
        nb.append(nb[-1] * ne[d - 1])
    return nb


def parse_manifest(root, suite):
    cases = {}
    for line in (root / "snapshots/parity" / suite / "manifest.txt").read_text().splitlines():
        if not line.startswith("case="):
            continue
        fields = dict(part.split("=", 1) for part in line.split(" ") if "=" in part)
        bits = fields.get("output_bits")
        cases[fields["case"]] = {
            "status": fields.get("status"),
            "error": fields.get("error"),
            "bits": [int(b, 16) for b in bits.split(",")] if bits else None if bits is None else [],
        }
    return cases


def status_code(manifest_case):
    st = manifest_case["status"]
    if st in ("ok", "Ok(())"):
        return "ok"
    err = manifest_case.get("error")
    if err:
        return {"InvalidView": "invalid_view", "ShapeMismatch": "shape_mismatch",
                "InvalidParameters": "invalid_parameters", "UnexpectedEvent": "unexpected_event"}[err]
    if st == "invalid_shape":
        return "shape_mismatch"
    return "rejected"  # any error status


def main(root):
    root = Path(root)
    out = []

    def add(suite, case, op, inputs, output, params=None, readout="logical", compare="exact", source=""):
        m = parse_manifest(root, suite)[case]
        out.append({
            "suite": suite, "case": case, "op": op, "params": params or {},
            "inputs": inputs, "output": output, "readout": readout, "compare": compare,
            "expect_status": status_code(m), "expect_bits": m["bits"], "source": source,
        })

    # --- kernel-binary: tools/emel-kernel-binary-parity/src/main.rs:145-254
    src = "tools/emel-kernel-binary-parity/src/main.rs:145-254"
    lhs, rhs = [1.0, 2.0, 3.0, 4.0], [10.0, 20.0, 30.0, 40.0]
    dense, dense_nb = [4, 1, 1, 1], [4, 16, 64, 64]
    for case, op in (("dense_add", 0), ("dense_sub", 1), ("dense_mul", 2), ("dense_div", 3)):
        add("kernel-binary", case, "binary", {"lhs": view(lhs, dense, dense_nb), "rhs": view(rhs, dense, dense_nb)},
            view([0.0] * 4, dense, dense_nb), {"op": op}, source=src)
    sp, sp_nb = [3, 1, 1, 1], [8, 24, 72, 72]
    add("kernel-binary", "strided_add", "binary",
        {"lhs": view([1, 99, 2, 99, 3], sp, sp_nb), "rhs": view([10, 99, 20, 99, 30], sp, sp_nb)},
        view([0.0] * 5, sp, sp_nb), {"op": 0}, source=src)
    add("kernel-binary", "count_equal_different_dimensions", "binary",
        {"lhs": view(lhs, [2, 2, 1, 1], [4, 8, 16, 16]), "rhs": view(rhs, dense, dense_nb)},
        view([0.0] * 4, dense, dense_nb), {"op": 0}, source=src)
    add("kernel-binary", "implicit_contiguous_mul", "binary",
        {"lhs": view(lhs, dense, [0] * 4), "rhs": view(rhs, dense, [0] * 4)},
        view([0.0] * 4, dense, [0] * 4), {"op": 2}, source=src)
    add("kernel-binary", "count_mismatch_rejection", "binary",
        {"lhs": view(lhs, dense, dense_nb), "rhs": view(rhs, dense, dense_nb)},
        view([9.0] * 3, [3, 1, 1, 1], [4, 12, 36, 36]), {"op": 3}, source=src)

    # --- kernel-broadcast: tools/emel-kernel-broadcast-parity/src/main.rs:50-92
    src = "tools/emel-kernel-broadcast-parity/src/main.rs:50-92"
    source, row = [1.0, 2.0, 3.0, 4.0, 5.0, 6.0], [10.0, 20.0, 30.0]
    for case, op, nb, row_nb in (("row_add", 0, [4, 12, 24, 24], [4, 12, 12, 12]),
                                 ("row_mul", 2, [4, 12, 24, 24], [4, 12, 12, 12]),
                                 ("row_add_implicit", 0, [0] * 4, [0] * 4)):
        add("kernel-broadcast", case, "broadcast_row",
            {"src0": view(source, [3, 2, 1, 1], nb), "src1": view(row, [3, 1, 1, 1], row_nb)},
            view([0.0] * 6, [3, 2, 1, 1], nb), {"op": op}, source=src)

    # --- kernel-elementwise: tools/emel-kernel-elementwise-parity/src/main.rs:68-124
    src = "tools/emel-kernel-elementwise-parity/src/main.rs:68-124"
    a, b = [1.5, -2.0, 0.25], [-0.5, 4.0, 2.0]
    d3 = [3, 1, 1, 1]
    n3 = contiguous_nb(d3)
    add("kernel-elementwise", "op_dup", "copy", {"src": view(a, d3, n3)}, view([0.0] * 3, d3, n3), source=src)
    for case, op in (("op_add", 0), ("op_sub", 1), ("op_mul", 2), ("op_div", 3)):
        add("kernel-elementwise", case, "binary", {"lhs": view(a, d3, n3), "rhs": view(b, d3, n3)},
            view([0.0] * 3, d3, n3), {"op": op}, source=src)
    add("kernel-elementwise", "op_sqr", "unary", {"src": view(a, d3, n3)}, view([0.0] * 3, d3, n3), {"op": 64}, source=src)
    add("kernel-elementwise", "op_sqrt", "unary", {"src": view([0.0, 4.0, 9.0], d3, n3)}, view([0.0] * 3, d3, n3),
        {"op": 65}, source=src)
    add("kernel-elementwise", "invalid_shape", "copy", {"src": view(a, d3, n3)},
        view([0.0] * 2, [2, 1, 1, 1], contiguous_nb([2, 1, 1, 1])), readout="none", source=src)

    # --- kernel-power: tools/emel-kernel-power-parity/src/main.rs:116-154
    src = "tools/emel-kernel-power-parity/src/main.rs:116-154"
    d4, n4 = [4, 1, 1, 1], contiguous_nb([4, 1, 1, 1])
    add("kernel-power", "dense_square", "unary", {"src": view([-2.0, -0.5, 0.5, 2.0], d4, n4)}, view([0.0] * 4, d4, n4),
        {"op": 64}, source=src)
    add("kernel-power", "strided_square", "unary", {"src": view([3, 99, -4, 99, 0.5], sp, sp_nb)},
        view([0.0] * 5, sp, sp_nb), {"op": 64}, source=src)
    add("kernel-power", "count_equal_different_dimensions", "unary", {"src": view([1, 2, 3, 4], d4, n4)},
        view([0.0] * 4, d4, n4), {"op": 64}, source=src)
    add("kernel-power", "implicit_contiguous_square", "unary", {"src": view([1, 2, 3, 4], d4, [0] * 4)},
        view([0.0] * 4, d4, [0] * 4), {"op": 64}, source=src)
    add("kernel-power", "dense_square_root", "unary", {"src": view([0, 1, 4, 9], d4, n4)}, view([0.0] * 4, d4, n4),
        {"op": 65}, source=src)
    add("kernel-power", "shape_rejection", "unary", {"src": view([1, 2, 3, 4], d4, n4)},
        view([9.0] * 3, d3, n3), {"op": 64}, source=src)

    # --- kernel-unary: tools/emel-kernel-unary-parity/src/main.rs:24-67 (generic OpUnary)
    src = "tools/emel-kernel-unary-parity/src/main.rs:24-67"
    x8 = [-10.1, -10.0, -1.2345, -0.125, 0.0, 0.12345, 10.0, 10.1]
    d8, n8 = [8, 1, 1, 1], contiguous_nb([8, 1, 1, 1])
    libm = {"exp", "tanh", "elu", "silu"}
    for name, sub in (("abs", 0), ("neg", 2), ("relu", 6), ("exp", 13), ("tanh", 4), ("elu", 5), ("gelu", 8), ("silu", 10)):
        add("kernel-unary", name, "op_unary", {"src": view(x8, d8, n8)}, view([0.0] * 8, d8, n8), {"op": sub},
            compare="ulp4" if name in libm else "exact", source=src)

    # --- kernel-target-scalar-unary: tools/emel-kernel-target-scalar-unary-parity/src/main.rs:38-113
    src = "tools/emel-kernel-target-scalar-unary-parity/src/main.rs:38-113"
    x5 = [-3.5, -0.5, 0.0, 0.5, 2.25]
    d5, n5 = [5, 1, 1, 1], contiguous_nb([5, 1, 1, 1])
    for name, op in (("exp", 13), ("tanh", 4), ("elu", 5), ("gelu", 8), ("silu_scalar_residual", 10)):
        add("kernel-target-scalar-unary", name, "unary", {"src": view(x5, d5, n5)}, view([0.0] * 5, d5, n5), {"op": op},
            compare="exact" if name == "gelu" else "ulp4", source=src)
    add("kernel-target-scalar-unary", "invalid_shape", "unary", {"src": view([1.0, -2.0, 3.0], d3, n3)},
        view([SENTINEL] * 2, [2, 1, 1, 1], contiguous_nb([2, 1, 1, 1]), bits=True), {"op": 13}, source=src)

    # --- kernel-softmax: tools/emel-kernel-softmax-parity/src/main.rs:22-81
    src = "tools/emel-kernel-softmax-parity/src/main.rs:22-81"
    sm_in, d32 = [1.0, 2.0, 4.0, 2.0, 5.0, 8.0], [3, 2, 1, 1]
    n32 = contiguous_nb(d32)
    add("kernel-softmax", "dense_rows", "soft_max", {"src": view(sm_in, d32, n32)}, view([0.0] * 6, d32, n32),
        compare="ulp4", source=src)
    add("kernel-softmax", "implicit_contiguous", "soft_max", {"src": view(sm_in, d32, [0] * 4)},
        view([0.0] * 6, d32, [0] * 4), compare="ulp4", source=src)
    add("kernel-softmax", "shape_mismatch", "soft_max", {"src": view(sm_in, d32, n32)},
        view([SENTINEL] * 4, [2, 2, 1, 1], contiguous_nb([2, 2, 1, 1]), bits=True), source=src)

    # --- kernel-target-softmax: tools/emel-kernel-target-softmax-parity/src/main.rs:30-88
    src = "tools/emel-kernel-target-softmax-parity/src/main.rs:30-88"
    add("kernel-target-softmax", "soft_max", "soft_max", {"src": view(sm_in, d32, n32)}, view([0.0] * 6, d32, n32),
        compare="ulp4", source=src)
    add("kernel-target-softmax", "zero_columns", "soft_max", {"src": view([SENTINEL], [0, 2, 1, 1], [4, 0, 0, 0], bits=True)},
        view([SENTINEL], [0, 2, 1, 1], [4, 0, 0, 0], bits=True), readout="storage", source=src)
    add("kernel-target-softmax", "shape_mismatch", "soft_max", {"src": view(sm_in, d32, n32)},
        view([SENTINEL] * 4, [2, 2, 1, 1], contiguous_nb([2, 2, 1, 1]), bits=True), source=src)

    # --- kernel-normalization: tools/emel-kernel-normalization-parity/src/main.rs:37-97
    src = "tools/emel-kernel-normalization-parity/src/main.rs:37-97"
    add("kernel-normalization", "implicit_rms_norm", "rms_norm", {"src": view(sm_in, d32, [0] * 4)},
        view([0.0] * 6, d32, [0] * 4), {"eps": 1.0}, readout="storage", source=src)
    add("kernel-normalization", "strided_norm", "norm", {"src": view([1, 2, 99, 99, 2, 5, 8], d32, [4, 16, 32, 32])},
        view([9.0] * 7, d32, [4, 16, 32, 32]), {"eps": 1.0}, readout="storage", source=src)
    add("kernel-normalization", "empty_outer_norm", "norm", {"src": view([1.0], [3, 0, 1, 1], [4, 12, 0, 0])},
        view([9.0], [3, 0, 1, 1], [4, 12, 0, 0]), {"eps": 1.0}, readout="storage", source=src)
    add("kernel-normalization", "invalid_epsilon", "norm", {"src": view(sm_in, d32, [0] * 4)},
        view([9.0] * 6, d32, [0] * 4), {"eps": float("nan")}, readout="storage", source=src)

    # --- kernel-target-normalization: tools/emel-kernel-target-normalization-parity/src/main.rs:32-109
    src = "tools/emel-kernel-target-normalization-parity/src/main.rs:32-109"
    add("kernel-target-normalization", "norm", "norm", {"src": view(sm_in, d32, n32)}, view([0.0] * 6, d32, n32),
        {"eps": 1.0}, readout="storage", source=src)
    add("kernel-target-normalization", "rms_norm", "rms_norm", {"src": view(sm_in, d32, n32)}, view([0.0] * 6, d32, n32),
        {"eps": 1.0}, readout="storage", source=src)
    add("kernel-target-normalization", "invalid_epsilon", "norm", {"src": view(sm_in, d32, n32)},
        view([SENTINEL] * 6, d32, n32, bits=True), {"eps": float("nan")}, readout="storage", source=src)
    add("kernel-target-normalization", "zero_columns", "rms_norm",
        {"src": view([SENTINEL], [0, 2, 1, 1], [4, 0, 0, 0], bits=True)},
        view([SENTINEL], [0, 2, 1, 1], [4, 0, 0, 0], bits=True), {"eps": 1.0}, readout="storage", source=src)
    add("kernel-target-normalization", "shape_mismatch", "norm", {"src": view(sm_in, d32, n32)},
        view([SENTINEL] * 4, [2, 2, 1, 1], contiguous_nb([2, 2, 1, 1]), bits=True), {"eps": 1.0},
        readout="storage", source=src)

    # --- kernel-activation: tools/emel-kernel-activation-parity/src/main.rs:31-89
    src = "tools/emel-kernel-activation-parity/src/main.rs:31-89"
    act = [f32_bits(-2.0), f32_bits(-0.5), f32_bits(0.0), f32_bits(2.0), 0x7FC01234]
    d5v = view(act, d5, n5, bits=True)
    add("kernel-activation", "op_scale", "scale", {"src": d5v}, view([0.0] * 5, d5, n5), {"scale": 1.5},
        readout="storage", source=src)
    add("kernel-activation", "op_clamp", "clamp", {"src": d5v}, view([0.0] * 5, d5, n5), {"min": -1.0, "max": 1.0},
        readout="storage", source=src)
    add("kernel-activation", "op_silu_back", "silu_back",
        {"src": view([-2.0, -0.5, 0.0, 2.0, 0.25], d5, n5), "grad": view([0.5, -2.0, 1.0, 3.0, -0.25], d5, n5)},
        view([0.0] * 5, d5, n5), readout="storage", compare="ulp4", source=src)
    add("kernel-activation", "op_leaky_relu", "leaky_relu", {"src": d5v}, view([0.0] * 5, d5, n5), {"slope": 0.125},
        readout="storage", source=src)

    # --- Known-answer unit tests (f32 literals from crates/emel-kernels/tests/any/).
    def known(name, op, inputs, output, expect, params=None, source="", readout="storage"):
        out.append({"suite": "unit-tests", "case": name, "op": op, "params": params or {}, "inputs": inputs,
                    "output": output, "readout": readout, "compare": "exact", "expect_status": "ok",
                    "expect_bits": [f32_bits(v) for v in expect], "source": source})

    known("norm_matches_reference_row_formula", "norm", {"src": view(sm_in, d32, n32)}, view([0.0] * 6, d32, n32),
          [-0.83405757, -0.20851436, 1.0425721, -1.1338935, 0.0, 1.1338935], {"eps": 1.0},
          "crates/emel-kernels/tests/any/normalization_ops.rs:29-54")
    known("rms_norm_matches_reference_row_formula", "rms_norm", {"src": view([3, 4, 0, 2], [2, 2, 1, 1], contiguous_nb([2, 2, 1, 1]))},
          view([0.0] * 4, [2, 2, 1, 1], contiguous_nb([2, 2, 1, 1])), [0.8164966, 1.0886621, 0.0, 1.1547005], {"eps": 1.0},
          "crates/emel-kernels/tests/any/normalization_ops.rs:56-73")
    r6 = [1.0, 2.0, 3.0, 4.0, 5.0, 6.0]
    one = [1, 1, 1, 1]
    known("sum", "sum", {"src": view(r6, d32, n32)}, view([0.0], one, contiguous_nb(one)), [21.0],
          source="crates/emel-kernels/tests/any/reductions.rs:58-102")
    known("mean", "mean", {"src": view(r6, d32, n32)}, view([0.0], one, contiguous_nb(one)), [3.5],
          source="crates/emel-kernels/tests/any/reductions.rs:58-102")
    known("argmax", "argmax", {"src": view(r6, d32, n32)}, view([0.0], one, contiguous_nb(one)), [5.0],
          source="crates/emel-kernels/tests/any/reductions.rs:58-102")
    known("sum_rows", "sum_rows", {"src": view(r6, d32, n32)}, view([0.0] * 2, [1, 2, 1, 1], contiguous_nb([1, 2, 1, 1])),
          [6.0, 15.0], source="crates/emel-kernels/tests/any/reductions.rs:58-102")
    known("row_add", "broadcast_row", {"src0": view(r6, d32, n32), "src1": view([10, 20, 30], d3, n3)},
          view([0.0] * 6, d32, n32), [11, 22, 33, 14, 25, 36], {"op": 0},
          "crates/emel-kernels/tests/any/broadcast_ops.rs:19-40")
    known("row_mul", "broadcast_row", {"src0": view(r6, d32, n32), "src1": view([10, 20, 30], d3, n3)},
          view([0.0] * 6, d32, n32), [10, 40, 90, 40, 100, 180], {"op": 2},
          "crates/emel-kernels/tests/any/broadcast_ops.rs:42-62")
    known("strided_row_add", "broadcast_row",
          {"src0": view([1, 99, 2, 99, 3, 99, 99, 99, 4, 99, 5, 99, 6], d32, [8, 32, 64, 128]),
           "src1": view([10, 99, 20, 99, 30], d3, [8, 24, 24, 24])},
          view([-7.0] * 13, d32, [8, 32, 64, 128]), [11, -7, 22, -7, 33, -7, -7, -7, 14, -7, 25, -7, 36], {"op": 0},
          "crates/emel-kernels/tests/any/broadcast_ops.rs:64-89")
    known("singleton_zero_stride_row_mul", "broadcast_row",
          {"src0": view(r6, d32, [4, 12, 0, 0]), "src1": view([10, 20, 30], d3, [4, 12, 0, 0])},
          view([0.0] * 6, d32, [4, 12, 0, 0]), [10, 40, 90, 40, 100, 180], {"op": 2},
          "crates/emel-kernels/tests/any/broadcast_ops.rs:91-108")

    write_flash_attn(root)

    dst = Path(__file__).resolve().parent / "reference_parity.json"
    dst.write_text(json.dumps({"generated_from": "stateforward/emel.rs snapshots/parity + tools/*-parity + tests/any",
                               "cases": out}, indent=1, allow_nan=True) + "\n")
    print(f"wrote {len(out)} cases to {dst}")


def write_flash_attn(root):
    """tests/golden/flash_attn_parity.json: the kernel-flash-attn manifest's
    cases with the inputs of tools/emel-kernel-flash-attn-parity/src/main.rs:61-104
    (query [2, 1, 2, 1] F32, key / value [2, 2, 1, 1] F16 as raw bits, the key
    buffer eight halves long as in the observer), plus the known answers of
    crates/emel-kernels/tests/any/flash_attn_ops.rs (approximate values, with
    the tolerance each test states)."""
    m = parse_manifest(root, "kernel-flash-attn")
    src = "tools/emel-kernel-flash-attn-parity/src/main.rs:61-104"
    q = [1.0, 0.0, 1.0, 0.0]
    key = [0x3C00, 0, 0, 0, 0, 0x3C00, 0, 0]
    value = [0x4000, 0x4400, 0x4600, 0x4800]
    kv = {"ne": [2, 2, 1, 1], "nb": [2, 4, 8, 8]}
    qd = {"ne": [2, 1, 2, 1], "nb": contiguous_nb([2, 1, 2, 1])}
    cases = []
    for case, scale in (("canonical", 1.0), ("invalid_scale", 0.0)):
        cases.append({"case": case, "source": src, "query": q, "query_layout": qd, "key": key, "key_layout": kv,
                      "value": value, "value_layout": kv, "dst_layout": qd, "dst_fill": 9.0 if scale == 0.0 else 0.0,
                      "scale": scale, "masked_total_tokens": 2, "expect_status": status_code(m[case]),
                      "expect_bits": m[case]["bits"], "compare": "exact"})
    t = "crates/emel-kernels/tests/any/flash_attn_ops.rs"
    one = {"ne": [1, 1, 1, 1], "nb": [2, 2, 2, 2]}
    one32 = {"ne": [1, 1, 1, 1], "nb": [4, 4, 4, 4]}

    def known(case, source, query, ql, key_, kl, value_, vl, dl, expect, tol, scale=None, masked=None, fill=0.0,
              status="ok"):
        cases.append({"case": case, "source": source, "query": query, "query_layout": ql, "key": key_,
                      "key_layout": kl, "value": value_, "value_layout": vl, "dst_layout": dl, "dst_fill": fill,
                      "scale": scale, "masked_total_tokens": masked, "expect_status": status,
                      "expect_values": expect, "tolerance": tol, "compare": "approx"})

    known("online_attention_formula", t + ":28-85", q, qd, key[:4], kv, value, kv, qd,
          [3.0758, 5.0758, 3.0758, 5.0758], 0.01, scale=1.0)
    hl = {"ne": [1, 1, 2, 1], "nb": [4, 4, 4, 8]}
    known("head_replication", t + ":87-118", [1.0, 1.0], hl, [0x3C00, 0x3C00], {"ne": [1, 2, 1, 1], "nb": [2, 2, 4, 4]},
          [0x4000, 0x4400], {"ne": [1, 2, 1, 1], "nb": [2, 2, 4, 4]}, hl, [3.0, 3.0], 0.02, scale=1.0, masked=2)
    known("implicit_contiguous", t + ":120-145", [1.0], {"ne": [1, 1, 1, 1], "nb": [0, 99, 0, 0]}, [0x3C00],
          {"ne": [1, 1, 1, 1], "nb": [0, 99, 0, 0]}, [0x4000], {"ne": [1, 1, 1, 1], "nb": [0, 99, 0, 0]},
          {"ne": [1, 1, 1, 1], "nb": [0, 99, 0, 0]}, [2.0], 0.01, scale=1.0, masked=1)
    known("singleton_unaligned_strides", t + ":147-174", [1.0], one32, [0x3C00], {"ne": [1, 1, 1, 1], "nb": [2, 0, 1, 3]},
          [0x4000], {"ne": [1, 1, 1, 1], "nb": [2, 1, 3, 5]}, one32, [2.0], 0.01, scale=1.0, masked=1)
    known("multi_element_unaligned_stride", t + ":176-198", [1.0, 0.0], {"ne": [2, 1, 1, 1], "nb": [4, 8, 8, 8]},
          [0x3C00, 0], {"ne": [2, 1, 1, 1], "nb": [3, 6, 12, 24]}, [0x4000, 0x4000],
          {"ne": [2, 1, 1, 1], "nb": [2, 4, 4, 4]}, {"ne": [2, 1, 1, 1], "nb": [4, 8, 8, 8]}, [9.0, 9.0], 0.0,
          fill=9.0, status="rejected")
    known("unexpected_then_default_options", t + ":252-275", [1.0], one32, [0x3C00], one, [0x4000], one, one32,
          [2.0], 0.01)
    known("zero_scale_rejected", t + ":220-250", [1.0, 0.0], {"ne": [2, 1, 1, 1], "nb": [4, 8, 8, 8]}, [0, 0, 0, 0],
          {"ne": [2, 2, 1, 1], "nb": [2, 4, 8, 8]}, [0, 0, 0, 0], {"ne": [2, 2, 1, 1], "nb": [2, 4, 8, 8]},
          {"ne": [2, 1, 1, 1], "nb": [4, 8, 8, 8]}, [9.0, 9.0], 0.0, scale=0.0, masked=1, fill=9.0, status="rejected")
    dst = Path(__file__).resolve().parent / "flash_attn_parity.json"
    dst.write_text(json.dumps({"generated_from": "stateforward/emel.rs snapshots/parity/kernel-flash-attn + "
                               "tools/emel-kernel-flash-attn-parity + tests/any/flash_attn_ops.rs",
                               "cases": cases}, indent=1) + "\n")
    print(f"wrote {len(cases)} cases to {dst}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_golden.py <emel.rs checkout>")
    main(sys.argv[1])
