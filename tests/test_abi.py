"""C-ABI checks that need no GPU: the device library loads, exports every
symbol include/emel_cuda.h declares, and its host-side validation classifies
requests exactly like the reference guards (restated by the oracle).

Validation runs before any CUDA call, so rejected requests return their
status with a null context; an accepted request reaches the context check
and reports INVALID_ARGUMENT instead of launching."""

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest

import oracle

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "emel_cuda.h"

ACCEPTED = 18  # EMEL_CUDA_INVALID_ARGUMENT from the null context after validation passed


def declared_symbols():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"\b(emel_(?:cuda|gguf)_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol(emel):
    lib = emel.lib()
    syms = declared_symbols()
    assert len(syms) >= 30
    missing = [s for s in syms if not hasattr(lib, s)]
    assert not missing, missing
    assert set(syms) == set(emel.SIGNATURES), set(syms) ^ set(emel.SIGNATURES)


def test_library_exports_nothing_undeclared(emel):
    import subprocess
    out = subprocess.run(["nm", "-D", "--defined-only", str(emel.LIB_PATH)], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    ours = {s for s in exported if s.startswith("emel_")}
    assert ours == set(declared_symbols())


def cview(emel, data_ptr, storage, ne, nb, dtype=0):
    v = emel.CView()
    v.data = data_ptr
    v.storage_bytes = storage
    for d in range(4):
        v.ne[d] = ne[d]
        v.nb[d] = nb[d]
    v.dtype = dtype
    return v


def oview(ptr, storage, ne, nb, dtype=0):
    return oracle.make_view(ptr, storage, ne, nb, dtype)


def random_layout(rng, elem=4):
    """Layouts around the validity boundary: zero extents, zero / unaligned /
    short strides, implicit nb[0]==0, storage one byte short."""
    ne = [int(x) for x in rng.choice([0, 1, 1, 2, 3, 4], size=4)]
    ne[0] = int(rng.choice([0, 1, 2, 3, 4, 8]))
    kind = rng.integers(0, 6)
    if kind == 0:
        nb = [0, 0, 0, 0]
    else:
        nb = [elem]
        for d in range(1, 4):
            nb.append(nb[-1] * max(ne[d - 1], 1))
        if kind == 2:
            nb[int(rng.integers(0, 4))] = 0
        elif kind == 3:
            nb[int(rng.integers(0, 4))] += int(rng.choice([1, 2, elem]))
        elif kind == 4:
            nb = [x * 2 for x in nb]
    eff = nb if nb[0] != 0 else [elem] + [elem * int(np.prod([max(n, 1) for n in ne[:d]])) for d in range(1, 4)]
    span = sum(max(n - 1, 0) * s for n, s in zip(ne, eff)) + elem
    storage = span - int(rng.choice([0, 0, 0, 1, elem]))
    return ne, nb, max(storage, 0)


FAMILIES = [
    ("binary", 3), ("broadcast_row", 3), ("binary_repeat", 3), ("unary", 2), ("op_unary", 2), ("scale", 2),
    ("norm", 2), ("rms_norm", 2), ("soft_max", 2), ("sum", 2), ("sum_rows", 2), ("argmax", 2), ("copy", 2),
]


@pytest.mark.parametrize("family,nviews", FAMILIES)
def test_validation_matches_reference_guards(emel, oracle_lib, family, nviews):
    lib = emel.lib()
    rng = np.random.default_rng(hash(family) & 0xFFFF)
    buf = np.zeros(4096, dtype=np.float32)  # backs the oracle on accepted requests
    agree = 0
    for trial in range(400):
        layouts = [random_layout(rng) for _ in range(nviews)]
        if family in ("broadcast_row", "binary_repeat") and trial % 2 == 0:
            # bias towards well-formed broadcasts
            ne0 = layouts[0][0][0] or 3
            layouts[0] = ([ne0, 2, 1, 1], [4, 4 * ne0, 8 * ne0, 8 * ne0], 8 * ne0)
            layouts[1] = ([ne0, 1, 1, 1], [0, 0, 0, 0], 4 * ne0)
            layouts[2] = ([ne0, 2, 1, 1], [0, 0, 0, 0], 8 * ne0)
        if family in ("sum", "argmax") and trial % 2 == 0:
            layouts[1] = ([1, 1, 1, 1], [0, 0, 0, 0], 4)
        if family == "sum_rows" and trial % 2 == 0:
            ne = layouts[0][0]
            layouts[1] = ([1] + ne[1:], [0, 0, 0, 0], 4 * max(1, int(np.prod(ne[1:]))))
        cv = [cview(emel, buf.ctypes.data, s, ne, nb) for ne, nb, s in layouts]
        ov = [oview(buf.ctypes.data, s, ne, nb) for ne, nb, s in layouts]
        B = ctypes.byref
        if family == "binary":
            got = lib.emel_cuda_binary(None, None, 1, B(cv[0]), B(cv[1]), B(cv[2]))
            want = oracle_lib.oracle_binary(1, B(ov[0]), B(ov[1]), B(ov[2]))
        elif family == "broadcast_row":
            got = lib.emel_cuda_broadcast_row(None, None, 0, B(cv[0]), B(cv[1]), B(cv[2]))
            want = oracle_lib.oracle_broadcast_row(0, B(ov[0]), B(ov[1]), B(ov[2]))
        elif family == "binary_repeat":
            got = lib.emel_cuda_binary_repeat(None, None, 2, B(cv[0]), B(cv[1]), B(cv[2]))
            want = oracle_lib.oracle_binary_repeat(2, B(ov[0]), B(ov[1]), B(ov[2]))
        elif family == "unary":
            got = lib.emel_cuda_unary(None, None, 13, B(cv[0]), B(cv[1]))
            want = oracle_lib.oracle_unary(13, B(ov[0]), B(ov[1]))
        elif family == "op_unary":
            sub = int(rng.choice([0, 1, 7, 10, 13, 17]))
            got = lib.emel_cuda_op_unary(None, None, sub, B(cv[0]), B(cv[1]))
            want = oracle_lib.oracle_op_unary(sub, B(ov[0]), B(ov[1]))
        elif family == "scale":
            got = lib.emel_cuda_scale(None, None, B(cv[0]), B(cv[1]), 2.0)
            want = oracle_lib.oracle_scale(B(ov[0]), B(ov[1]), 2.0)
        elif family in ("norm", "rms_norm"):
            eps = float(rng.choice([1e-5, 0.0, -1.0, float("nan"), float("inf")]))
            got = getattr(lib, f"emel_cuda_{family}")(None, None, B(cv[0]), B(cv[1]), eps)
            want = getattr(oracle_lib, f"oracle_{family}")(B(ov[0]), B(ov[1]), eps)
        elif family == "soft_max":
            got = lib.emel_cuda_soft_max(None, None, B(cv[0]), B(cv[1]))
            want = oracle_lib.oracle_soft_max(B(ov[0]), B(ov[1]))
        elif family == "copy":
            got = lib.emel_cuda_copy(None, None, B(cv[0]), B(cv[1]))
            want = oracle_lib.oracle_copy(B(ov[0]), B(ov[1]))
        else:
            got = getattr(lib, f"emel_cuda_{family}")(None, None, B(cv[0]), B(cv[1]))
            want = getattr(oracle_lib, f"oracle_{family}")(B(ov[0]), B(ov[1]))
        if want == 0:
            assert got == ACCEPTED, (family, layouts, got)
        else:
            assert got == want, (family, layouts, got, want)
        agree += 1
    assert agree == 400


def test_flash_attn_validation_matches_reference_guards(emel, oracle_lib):
    """valid_request (flash_attn.rs:262-303) on layouts around its boundary:
    the C ABI's outcome equals the oracle's restatement for every request."""
    lib = emel.lib()
    rng = np.random.default_rng(77)
    buf = np.zeros(1 << 14, dtype=np.float32)
    B = ctypes.byref
    accepted = 0
    for trial in range(600):
        d = int(rng.choice([0, 1, 2, 4, 8]))
        heads = int(rng.choice([0, 1, 2, 4]))
        kvh = int(rng.choice([0, 1, 2, 3]))
        t = int(rng.choice([0, 1, 3]))
        qne = [d, int(rng.choice([1, 1, 1, 2])), heads, 1]
        kne = [d if rng.random() < 0.9 else d + 1, t, kvh, int(rng.choice([1, 1, 1, 2]))]
        vne = list(kne) if rng.random() < 0.9 else [d, t + 1, kvh, 1]
        dne = list(qne) if rng.random() < 0.9 else [d, 1, heads + 1, 1]

        def lay(ne, elem):
            kind = rng.integers(0, 5)
            if kind == 0:
                nb = [0, 0, 0, 0]
            else:
                nb = [elem]
                for k in range(1, 4):
                    nb.append(nb[-1] * max(ne[k - 1], 1))
                if kind == 2:
                    nb = [x * 2 for x in nb]
                elif kind == 3:
                    nb[int(rng.integers(0, 4))] += int(rng.choice([1, 2, 3]))
            eff = nb if nb[0] != 0 else [elem] + [elem * int(np.prod([max(n, 1) for n in ne[:k]])) for k in range(1, 4)]
            span = sum(max(n - 1, 0) * st for n, st in zip(ne, eff)) + elem
            return ne, nb, max(span - int(rng.choice([0, 0, 0, 1, 2])), 0)

        views = [lay(qne, 4), lay(kne, 2), lay(vne, 2), lay(dne, 4)]
        dtypes = [0, 1 if rng.random() < 0.95 else 0, 1, 0]
        scale = [None, 0.5, 0.0, -1.0, float("inf"), float("nan")][int(rng.integers(0, 6))]
        masked = [None, 0, 1, 3, 4][int(rng.integers(0, 5))]
        if trial % 2 == 0:
            # a well-formed request with one perturbation at most
            d, kvh = int(rng.choice([1, 2, 4, 8])), int(rng.choice([1, 2]))
            heads, t = kvh * int(rng.choice([1, 2])), int(rng.choice([1, 3]))
            shapes = [([d, 1, heads, 1], 4), ([d, t, kvh, 1], 2), ([d, t, kvh, 1], 2), ([d, 1, heads, 1], 4)]
            views = [lay(ne, elem) if rng.random() < 0.7 else (ne, [0, 0, 0, 0], int(np.prod(ne)) * elem)
                     for ne, elem in shapes]
            dtypes = [0, 1, 1, 0]
            scale = [None, 0.5, 0.0][int(rng.integers(0, 3))]
            masked = [None, t, t + 2, max(t - 1, 0)][int(rng.integers(0, 4))]
        cv = [cview(emel, buf.ctypes.data, st, ne, nb, dt) for (ne, nb, st), dt in zip(views, dtypes)]
        ov = [oview(buf.ctypes.data, st, ne, nb, dt) for (ne, nb, st), dt in zip(views, dtypes)]
        copt = emel.CFlashAttnOptions.of(scale, masked)
        oopt = oracle.FlashAttnOptions()
        if scale is not None:
            oopt.scale, oopt.has_scale = scale, 1
        if masked is not None:
            oopt.masked_total_tokens, oopt.has_masked_total_tokens = masked, 1
        got = lib.emel_cuda_flash_attn_ext(None, None, B(cv[0]), B(cv[1]), B(cv[2]), B(cv[3]), B(copt))
        want = oracle_lib.oracle_flash_attn_ext(B(ov[0]), B(ov[1]), B(ov[2]), B(ov[3]), B(oopt))
        if want == 0:
            assert got == ACCEPTED, (views, dtypes, scale, masked, got)
            accepted += 1
        else:
            assert want == 12 and got == 12, (views, dtypes, scale, masked, got, want)
    assert accepted >= 20


def test_misaligned_or_null_device_pointer_is_an_invalid_view(emel):
    lib = emel.lib()
    ne, nb = [4, 1, 1, 1], [4, 16, 16, 16]
    good = cview(emel, 4096, 16, ne, nb)
    for bad_ptr in (0, 4098):
        bad = cview(emel, bad_ptr, 16, ne, nb)
        assert lib.emel_cuda_binary(None, None, 0, ctypes.byref(bad), ctypes.byref(good), ctypes.byref(good)) == 1
    assert lib.emel_cuda_binary(None, None, 0, ctypes.byref(good), ctypes.byref(good), ctypes.byref(good)) == ACCEPTED


def test_unknown_ops_are_unexpected_events(emel):
    lib = emel.lib()
    v = cview(emel, 4096, 16, [4, 1, 1, 1], [4, 16, 16, 16])
    B = ctypes.byref
    assert lib.emel_cuda_binary(None, None, 7, B(v), B(v), B(v)) == 4
    assert lib.emel_cuda_unary(None, None, 17, B(v), B(v)) == 4  # XIELU has no typed event
    assert lib.emel_cuda_unary(None, None, 99, B(v), B(v)) == 4
    assert lib.emel_cuda_op_unary(None, None, 7, B(v), B(v)) == 4  # sigmoid is not an OpUnary subop


def test_argmax_combine_follows_first_index_and_nan_rules(emel):
    combine = emel.argmax_combine
    # later shard wins only with a strictly greater value
    assert combine([(2.0, 1, 10, 0), (2.0, 1, 70, 0)]) == (10, 2.0)
    assert combine([(2.0, 1, 10, 0), (3.0, 1, 70, 0)]) == (70, 3.0)
    # a shard with no comparable value is skipped
    assert combine([(0.0, 0, 0, 0), (1.5, 1, 99, 0)]) == (99, 1.5)
    # NaN at element 0 of the whole tensor pins the answer to 0
    assert combine([(5.0, 1, 3, 1), (9.0, 1, 99, 0)])[0] == 0
    # a NaN first element in a later shard does not
    assert combine([(5.0, 1, 3, 0), (9.0, 1, 99, 1)])[0] == 99


def test_q8_0_argmax_guards_match_oracle(emel, oracle_lib):
    """quantized_views_valid / quantized_shape_valid (matmul.rs:1522-1564)
    for OpMulMatArgmaxQ8_0: the C ABI's status equals the oracle's."""
    lib = emel.lib()
    B = ctypes.byref
    buf = np.zeros(1 << 16, np.uint8)
    cases = []
    for k in (32, 64, 48):
        rb = k // 32 * 34
        for rows in (1, 3):
            good_l = ([k, rows, 1, 1], [1, rb, rb * rows, rb * rows], rb * rows, 8)
            cases.append((good_l, ([1, k, 1, 1], [4, 4, 4 * k, 4 * k], 4 * k), ([1, 1, 1, 1], [4, 4, 4, 4], 4)))
            cases.append((good_l, ([1, k, 1, 1], [4, 4, 4 * k, 4 * k], 4 * k - 1), ([1, 1, 1, 1], [4, 4, 4, 4], 4)))
            cases.append((good_l, ([1, k + 1, 1, 1], [4, 4, 4 * k + 4, 4 * k + 4], 4 * k + 4),
                          ([1, 1, 1, 1], [4, 4, 4, 4], 4)))
            cases.append((good_l, ([k, 1, 1, 1], [4, 4 * k, 4 * k, 4 * k], 4 * k), ([1, 1, 1, 1], [4, 4, 4, 4], 4)))
            cases.append((([k, rows, 1, 1], [1, rb + 2, (rb + 2) * rows, (rb + 2) * rows], (rb + 2) * rows, 8),
                          ([1, k, 1, 1], [4, 4, 4 * k, 4 * k], 4 * k), ([1, 1, 1, 1], [4, 4, 4, 4], 4)))
            cases.append((([k, rows, 1, 1], [1, rb, rb * rows, rb * rows], rb * rows, 2),
                          ([1, k, 1, 1], [4, 4, 4 * k, 4 * k], 4 * k), ([1, 1, 1, 1], [4, 4, 4, 4], 4)))
            cases.append((good_l, ([1, k, 1, 1], [0, 0, 0, 0], 4 * k), ([1, 1, 1, 1], [4, 4, 4, 4], 4)))
            cases.append((good_l, ([1, k, 1, 1], [4, 4, 4 * k, 4 * k], 4 * k), ([2, 1, 1, 1], [4, 8, 8, 8], 8)))
    seen = set()
    for (lne, lnb, ls, lcode), (rne, rnb, rs), (dne, dnb, ds) in cases:
        lv, ov_l = cview(emel, buf.ctypes.data, ls, lne, lnb, lcode), oview(buf.ctypes.data, ls, lne, lnb, lcode)
        rv, ov_r = cview(emel, buf.ctypes.data, rs, rne, rnb), oview(buf.ctypes.data, rs, rne, rnb)
        dv, ov_d = cview(emel, buf.ctypes.data, ds, dne, dnb), oview(buf.ctypes.data, ds, dne, dnb)
        idx = ctypes.c_int32()
        got = lib.emel_cuda_mul_mat_argmax_q8_0(None, None, B(lv), B(rv), B(dv), ctypes.c_void_p(4096))
        want = oracle_lib.oracle_mul_mat_argmax_q8_0(B(ov_l), B(ov_r), B(ov_d), B(idx))
        assert got == (ACCEPTED if want == 0 else want), (lne, lnb, lcode, rne, rnb, rs, dne, got, want)
        seen.add(want)
    assert seen == {0, 1, 2}
