"""The generic operation envelope (GenericRequest / GenericEvent,
crates/emel-kernels/src/any/generic.rs) on the CPU: the oracle reproduces
the reference's own known answers (crates/emel-kernels/tests/any/
generic_envelope.rs), and emel_cuda_generic classifies requests exactly as
the oracle does -- before any device work, so these run without a GPU (a
valid request with no context is INVALID_ARGUMENT)."""

import ctypes
import struct

import numpy as np
import pytest

import oracle

OK, INVALID_SHAPE, UNSUPPORTED, INVALID_ARGUMENT = 0, 6, 7, 18


def f32_params(*values):
    return b"".join(struct.pack("=f", v) for v in values)


def hview(arr, ne, nb=None):
    return oracle.host_view(arr, ne, nb)


def run_oracle(lib, op, src0=None, src1=None, dst=None, params=b"", unary=0):
    r = oracle.generic_request(op, src0, src1, None, dst, params, unary)
    return lib.oracle_generic(ctypes.byref(r))


# ---- known answers of generic_envelope.rs --------------------------------------
def test_oracle_generic_known_answers(oracle_lib):
    lib = oracle_lib
    layout = ([4, 1, 1, 1], [4, 16, 64, 256])  # generic_envelope.rs:9-15
    src = np.array([1.0, -2.0, 3.0, 4.0], np.float32)
    rhs = np.array([2.0, 4.0, 6.0, 8.0], np.float32)
    out = np.zeros(4, np.float32)
    # Add (generic_envelope.rs:129-148); the views' storage covers their span
    src_s = np.zeros(64, np.float32)
    rhs_s = np.zeros(64, np.float32)
    out_s = np.zeros(64, np.float32)
    src_s[:4], rhs_s[:4] = src, rhs
    assert run_oracle(lib, 1, hview(src_s, *layout), hview(rhs_s, *layout), hview(out_s, *layout)) == OK
    assert out_s[:4].tolist() == [3.0, 2.0, 9.0, 12.0]
    # Unary Abs (150-168)
    out_s[:] = 0
    assert run_oracle(lib, 85, hview(src_s, *layout), None, hview(out_s, *layout), unary=0) == OK
    assert out_s[:4].tolist() == [1.0, 2.0, 3.0, 4.0]
    # SoftMax rows (171-192)
    x = np.array([1.0, 2.0, 3.0, 4.0], np.float32)
    y = np.zeros(4, np.float32)
    assert run_oracle(lib, 46, hview(x, [2, 2, 1, 1], [4, 8, 16, 16]), None, hview(y, [2, 2, 1, 1], [4, 8, 16, 16])) == OK
    assert np.allclose(y, [0.26894143, 0.7310586, 0.26894143, 0.7310586], atol=1e-6)
    # RmsNorm with eps 1e-5 (194-209)
    assert run_oracle(lib, 24, hview(x, [2, 2, 1, 1], [4, 8, 16, 16]), None, hview(y, [2, 2, 1, 1], [4, 8, 16, 16]),
                      f32_params(1e-5)) == OK
    scale = np.float32(1.0) / np.sqrt(np.float32(2.5) + np.float32(1e-5))
    assert abs(y[0] - scale) < 1e-6 and abs(y[1] - 2 * scale) < 1e-6
    # Add1 2.0 and Clamp [-1, 1] (251-287)
    s3 = np.array([1.0, -2.0, 3.0], np.float32)
    o3 = np.zeros(3, np.float32)
    assert run_oracle(lib, 3, hview(s3, [3, 1, 1, 1]), None, hview(o3, [3, 1, 1, 1]), f32_params(2.0)) == OK
    assert o3.tolist() == [3.0, 0.0, 5.0]
    assert run_oracle(lib, 50, hview(s3, [3, 1, 1, 1]), None, hview(o3, [3, 1, 1, 1]), f32_params(-1.0, 1.0)) == OK
    assert o3.tolist() == [1.0, -1.0, 1.0]


def test_oracle_generic_loops_differ_from_typed_where_the_reference_does(oracle_lib):
    """generic GELU has no binary16 rounding or +-10 clamp; generic soft_max
    sums in binary32 in row order; generic norm squares in binary32."""
    lib = oracle_lib
    x = np.array([0.1234567, 12.0, -11.0, 3.3333333], np.float32)
    y = np.zeros(4, np.float32)
    assert run_oracle(lib, 85, hview(x, [4, 1, 1, 1]), None, hview(y, [4, 1, 1, 1]), unary=8) == OK
    want = []
    for v in x.astype(np.float64):
        v32 = np.float32(v)
        cubic = np.float32(np.float64(np.float32(np.float32(0.044715) * v32) * v32) * np.float64(v32) + np.float64(v32))
        inner = np.float32(np.float32(0.7978846) * cubic)
        want.append(np.float32(np.float32(0.5) * v32) * np.float32(np.float32(1.0) + np.float32(np.tanh(np.float64(inner)))))
    assert np.allclose(y, want, rtol=2e-7, atol=0)
    typed = np.zeros(4, np.float32)
    assert lib.oracle_unary(8, ctypes.byref(hview(x, [4, 1, 1, 1])), ctypes.byref(hview(typed, [4, 1, 1, 1]))) == 0
    assert y[0] != typed[0]  # typed GELU rounds 0.1234567 through binary16 first
    assert np.signbit(y[2]) and not np.signbit(typed[2])  # -11: formula gives -0.0, the typed clamp +0.0


# ---- request classification: device ABI == oracle ---------------------------------
FAKE = 0x100000  # a 4-byte aligned address; validation never dereferences it


def cview(emel, ne, nb=(0, 0, 0, 0), storage=None, dtype=0, addr=FAKE):
    v = emel.CView()
    v.data = addr
    span = sum((ne[d] - 1) * (nb[d] if nb[0] else 0) for d in range(4)) + 4
    if not nb[0]:
        n = 1
        for d in range(4):
            n *= ne[d]
        span = 4 * n
    v.storage_bytes = storage if storage is not None else span
    for d in range(4):
        v.ne[d] = ne[d]
        v.nb[d] = nb[d]
    v.dtype = dtype
    return v


def device_status(emel, op, src0=None, src1=None, dst=None, params=b"", unary=0, params_len=None):
    r = emel.CGenericRequest()
    r.op = op
    r.unary_subop = unary
    keep = []
    for name, v in (("src0", src0), ("src1", src1), ("dst", dst)):
        if v is not None:
            keep.append(v)
            setattr(r, name, ctypes.pointer(v))
    ctypes.memmove(r.params, params, len(params))
    r.params_len = len(params) if params_len is None else params_len
    return emel.lib().emel_cuda_generic(None, None, ctypes.byref(r))


def oracle_status(lib, op, views, params=b"", unary=0):
    """Runs the oracle on host buffers with the same layouts (sized to fit)."""
    host = []
    ovs = []
    for v in views:
        if v is None:
            ovs.append(None)
            continue
        buf = np.zeros(max(1, (v.storage_bytes + 3) // 4), np.float32)
        host.append(buf)
        ovs.append(oracle.make_view(buf.ctypes.data, v.storage_bytes, list(v.ne), list(v.nb), v.dtype))
    r = oracle.generic_request(op, ovs[0], ovs[1], None, ovs[2], params, unary)
    return lib.oracle_generic(ctypes.byref(r))


def test_generic_classification_matches_oracle(emel, oracle_lib):
    V = lambda ne, **k: cview(emel, ne, **k)  # noqa: E731
    cases = [
        # (op, src0, src1, dst, params, unary, expected)
        (1, V([4, 2, 1, 1]), V([8, 1, 1, 1]), V([2, 4, 1, 1]), b"", 0, INVALID_ARGUMENT),  # valid: count-equal
        (1, V([4, 2, 1, 1]), V([7, 1, 1, 1]), V([8, 1, 1, 1]), b"", 0, INVALID_SHAPE),    # count mismatch
        (1, V([4, 2, 1, 1]), None, V([8, 1, 1, 1]), b"", 0, INVALID_SHAPE),               # missing src1
        (0, V([4, 2, 1, 1]), None, V([8, 1, 1, 1]), b"", 0, INVALID_ARGUMENT),
        (85, V([4, 1, 1, 1]), None, V([4, 1, 1, 1]), b"", 7, INVALID_SHAPE),              # sigmoid: not maintained
        (85, V([4, 1, 1, 1]), None, V([4, 1, 1, 1]), b"", 8, INVALID_ARGUMENT),           # gelu
        (32, V([4, 1, 1, 1]), None, V([4, 1, 1, 1]), f32_params(float("inf")), 0, INVALID_SHAPE),
        (32, V([4, 1, 1, 1]), None, V([4, 1, 1, 1]), b"", 0, INVALID_SHAPE),              # no scalar
        (32, V([4, 1, 1, 1]), None, V([4, 1, 1, 1]), f32_params(0.5), 0, INVALID_ARGUMENT),
        (50, V([4, 1, 1, 1]), None, V([4, 1, 1, 1]), f32_params(1.0, -1.0), 0, INVALID_SHAPE),  # min > max
        (50, V([4, 1, 1, 1]), None, V([4, 1, 1, 1]), f32_params(-1.0, 1.0), 0, INVALID_ARGUMENT),
        (19, V([2, 3, 1, 1]), None, V([4, 6, 2, 1]), b"", 0, INVALID_ARGUMENT),
        (19, V([2, 3, 1, 1]), None, V([5, 6, 1, 1]), b"", 0, INVALID_SHAPE),              # 5 % 2 != 0
        (13, V([4, 3, 1, 1]), None, V([1, 1, 1, 1]), b"", 0, INVALID_ARGUMENT),
        (17, V([4, 3, 1, 1]), None, V([2, 1, 1, 1]), b"", 0, INVALID_SHAPE),              # dst count 2
        (46, V([4, 3, 1, 1]), None, V([3, 4, 1, 1]), b"", 0, INVALID_ARGUMENT),           # counts equal
        (24, V([4, 3, 1, 1]), None, V([4, 3, 1, 1]), f32_params(-1.0), 0, INVALID_SHAPE), # eps < 0
        (24, V([4, 3, 1, 1]), None, V([4, 3, 1, 1]), b"", 0, INVALID_SHAPE),              # no eps
        (23, V([4, 3, 1, 1]), None, V([4, 3, 1, 1]), f32_params(1e-5), 0, INVALID_ARGUMENT),
        (22, V([4, 3, 1, 1]), V([4, 3, 1, 1]), V([12, 1, 1, 1]), b"", 0, INVALID_SHAPE),  # silu_back ne
        (15, V([4, 3, 1, 1]), None, V([4, 3, 1, 1]), b"", 0, UNSUPPORTED),                # cumsum: CPU-only route
        (28, V([4, 3, 1, 1]), V([4, 2, 1, 1]), V([3, 2, 1, 1]), b"", 0, UNSUPPORTED),     # mul_mat
        (60, V([4, 3, 1, 1]), None, V([4, 3, 1, 1]), b"", 0, UNSUPPORTED),                # pool_2d
        (1, V([4, 2, 1, 1], storage=16), V([8, 1, 1, 1]), V([8, 1, 1, 1]), b"", 0, INVALID_SHAPE),  # out of bounds
        (1, V([4, 2, 1, 1], nb=(4, 0, 32, 32)), V([8, 1, 1, 1]), V([8, 1, 1, 1]), b"", 0, INVALID_SHAPE),  # zero stride
        (60, V([4, 2, 1, 1], storage=16), None, None, b"", 0, INVALID_SHAPE),             # invalid view beats unsupported
    ]
    for k, (op, s0, s1, d, params, unary, expected) in enumerate(cases):
        got = device_status(emel, op, s0, s1, d, params, unary)
        assert got == expected, (k, op, got, expected)
        want = oracle_status(oracle_lib, op, [s0, s1, d], params, unary)
        # the oracle executes what the device would (OK), and agrees on every rejection
        assert want == (OK if expected == INVALID_ARGUMENT else expected), (k, op, want, expected)


def test_generic_request_envelope_rules(emel):
    v = cview(emel, [4, 1, 1, 1])
    assert device_status(emel, 95, v, None, v) == INVALID_ARGUMENT      # KernelOperation::from_code(95) is None
    assert device_status(emel, 1, v, v, v, params_len=65) == INVALID_ARGUMENT  # OpParams::new rejects > 64
    assert emel.lib().emel_cuda_generic(None, None, None) == INVALID_ARGUMENT


def test_generic_unaligned_views_are_a_device_argument_error(emel, oracle_lib):
    """Byte strides that are not multiples of 4 are valid for the reference
    (it reads bytes) but not for the device's binary32 loads."""
    src = cview(emel, [4, 1, 1, 1], nb=(6, 24, 24, 24), storage=22)
    dst = cview(emel, [4, 1, 1, 1])
    assert device_status(emel, 85, src, None, dst, unary=2) == INVALID_ARGUMENT
    assert oracle_status(oracle_lib, 85, [src, None, dst], unary=2) == OK
    odd = cview(emel, [4, 1, 1, 1], addr=FAKE + 2)
    assert device_status(emel, 85, odd, None, dst, unary=2) == INVALID_ARGUMENT
