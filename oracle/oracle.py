"""ctypes binding for the CPU oracle (liboracle.so).

TEST INFRASTRUCTURE ONLY: the parity checker for tests/ and __graft_entry__,
and the timed CPU baseline for bench.py.  The product library never imports
this module.
"""

import ctypes
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "liboracle.so"
CR_LIB_PATH = HERE / "liboracle_cr.so"  # libm calls evaluated in binary64, rounded once

DTYPE_CODE = {np.dtype(np.float32): 0, np.dtype(np.float16): 1, np.dtype(np.int32): 26, np.dtype(np.int64): 27}

STATUS = {0: "ok", 1: "invalid_view", 2: "shape_mismatch", 3: "invalid_parameters", 4: "unexpected_event",
          18: "invalid_argument"}


class View(ctypes.Structure):
    """Field-for-field the same layout as emel_tensor_view (include/emel_cuda.h)."""

    _fields_ = [("data", ctypes.c_void_p), ("storage_bytes", ctypes.c_uint64), ("ne", ctypes.c_uint64 * 4),
                ("nb", ctypes.c_uint64 * 4), ("dtype", ctypes.c_uint32), ("reserved", ctypes.c_uint32)]


def make_view(ptr, storage_bytes, ne, nb, dtype_code):
    v = View()
    v.data = ptr
    v.storage_bytes = storage_bytes
    for d in range(4):
        v.ne[d] = int(ne[d])
        v.nb[d] = int(nb[d])
    v.dtype = dtype_code
    return v


def host_view(array, ne=None, nb=None):
    """View of a host numpy array; by default a dense row-major view whose ne[0]
    is the last numpy axis (ggml order)."""
    code = DTYPE_CODE[array.dtype]
    if ne is None:
        shape = list(array.shape)[::-1] + [1] * (4 - array.ndim)
        ne = shape[:4]
    if nb is None:
        nb = [array.itemsize]
        for d in range(1, 4):
            nb.append(nb[-1] * ne[d - 1])
    return make_view(array.ctypes.data, array.nbytes, ne, nb, code)


_libs = {}


def build():
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


class RopeParams(ctypes.Structure):
    """oracle_rope_params / emel_rope_params (rope.rs:33-48)."""
    _fields_ = [("n_dims", ctypes.c_int32), ("mode", ctypes.c_int32), ("freq_base", ctypes.c_float),
                ("freq_scale", ctypes.c_float), ("ext_factor", ctypes.c_float), ("attn_factor", ctypes.c_float)]


class FlashAttnOptions(ctypes.Structure):
    """oracle_flash_attn_options / emel_flash_attn_options (flash_attn.rs:24-31)."""
    _fields_ = [("scale", ctypes.c_float), ("has_scale", ctypes.c_uint32),
                ("masked_total_tokens", ctypes.c_uint32), ("has_masked_total_tokens", ctypes.c_uint32)]


class GenericRequest(ctypes.Structure):
    """oracle_generic_request (same layout as emel_cuda_generic_request)."""
    _fields_ = [("op", ctypes.c_uint32), ("unary_subop", ctypes.c_uint32),
                ("src0", ctypes.POINTER(View)), ("src1", ctypes.POINTER(View)),
                ("src2", ctypes.POINTER(View)), ("dst", ctypes.POINTER(View)),
                ("params", ctypes.c_uint8 * 64), ("params_len", ctypes.c_uint32), ("reserved", ctypes.c_uint32)]


def generic_request(op, src0=None, src1=None, src2=None, dst=None, params=b"", unary=0):
    """An oracle_generic_request over host views (keeps them alive)."""
    r = GenericRequest()
    r.op = op
    r.unary_subop = unary
    r._keep = []
    for name, v in (("src0", src0), ("src1", src1), ("src2", src2), ("dst", dst)):
        if v is not None:
            r._keep.append(v)
            setattr(r, name, ctypes.pointer(v))
    ctypes.memmove(r.params, bytes(params), len(params))
    r.params_len = len(params)
    return r


def load(cr=False):
    """The oracle with the host's glibc float libm (default), or with
    correctly rounded libm calls (cr=True)."""
    if cr in _libs:
        return _libs[cr]
    path = CR_LIB_PATH if cr else LIB_PATH
    if not path.exists():
        build()
    lib = ctypes.CDLL(str(path))
    P = ctypes.POINTER(View)
    sigs = {
        "oracle_binary": [ctypes.c_int, P, P, P],
        "oracle_broadcast_row": [ctypes.c_int, P, P, P],
        "oracle_binary_repeat": [ctypes.c_int, P, P, P],
        "oracle_unary": [ctypes.c_int, P, P],
        "oracle_op_unary": [ctypes.c_int, P, P],
        "oracle_scale": [P, P, ctypes.c_float],
        "oracle_clamp": [P, P, ctypes.c_float, ctypes.c_float],
        "oracle_leaky_relu": [P, P, ctypes.c_float],
        "oracle_silu_back": [P, P, P],
        "oracle_glu": [ctypes.c_int, ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p, ctypes.c_uint64],
        "oracle_add1": [P, P, ctypes.c_float],
        "oracle_copy": [P, P],
        "oracle_cpy": [P, P],
        "oracle_get_rows": [P, P, P],
        "oracle_get_rows_f32_bytes": [P, P, P],
        "oracle_mul_mat_argmax": [P, P, P, ctypes.POINTER(ctypes.c_int32)],
        "oracle_mul_mat_argmax_q8_0": [P, P, P, ctypes.POINTER(ctypes.c_int32)],
        "oracle_mul_mat_argmax_q4_0": [P, P, P, ctypes.POINTER(ctypes.c_int32)],
        "oracle_mul_mat_argmax_q4_1": [P, P, P, ctypes.POINTER(ctypes.c_int32)],
        "oracle_mul_mat_argmax_q5_0": [P, P, P, ctypes.POINTER(ctypes.c_int32)],
        "oracle_mul_mat_argmax_q4_k": [P, P, P, ctypes.POINTER(ctypes.c_int32)],
        "oracle_mul_mat_argmax_q6_k": [P, P, P, ctypes.POINTER(ctypes.c_int32)],
        "oracle_mul_mat_argmax_q2_k": [P, P, P, ctypes.POINTER(ctypes.c_int32)],
        "oracle_mul_mat_argmax_q3_k": [P, P, P, ctypes.POINTER(ctypes.c_int32)],
        "oracle_rope": [P, P, P, ctypes.POINTER(RopeParams)],
        "oracle_flash_attn_ext": [P, P, P, P, ctypes.POINTER(FlashAttnOptions)],
        "oracle_diag": [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p, ctypes.c_uint64],
        "oracle_soft_max_diag_mask_inf": [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p, ctypes.c_uint64,
                                          ctypes.c_int32, ctypes.c_void_p],
        "oracle_diag_mask": [ctypes.c_int, ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p, ctypes.c_uint64,
                             ctypes.c_int32],
        "oracle_cont": [P, P],
        "oracle_norm": [P, P, ctypes.c_float],
        "oracle_rms_norm": [P, P, ctypes.c_float],
        "oracle_rms_norm_mul": [P, P, P, ctypes.c_float],
        "oracle_soft_max": [P, P],
        "oracle_soft_max_ext": [P, P, P, ctypes.c_float],
        "oracle_sum": [P, P],
        "oracle_sum_f64": [P, ctypes.POINTER(ctypes.c_double)],
        "oracle_mean": [P, P],
        "oracle_sum_rows": [P, P],
        "oracle_argmax": [P, P],
        "oracle_argmax_index": [P, ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_float)],
        "oracle_argmax_rows": [P, P],
        "oracle_generic": [ctypes.POINTER(GenericRequest)],
    }
    for name, args in sigs.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = ctypes.c_int
    lib.oracle_unary_range.argtypes = [ctypes.c_int, P, P, ctypes.c_uint64, ctypes.c_uint64]
    lib.oracle_unary_range.restype = None
    lib.oracle_rms_norm_rows.argtypes = [P, P, ctypes.c_float, ctypes.c_uint64, ctypes.c_uint64]
    lib.oracle_rms_norm_rows.restype = None
    lib.oracle_fp32_to_fp16.argtypes = [ctypes.c_float]
    lib.oracle_fp32_to_fp16.restype = ctypes.c_uint16
    lib.oracle_fp16_to_fp32.argtypes = [ctypes.c_uint16]
    lib.oracle_fp16_to_fp32.restype = ctypes.c_float
    lib.oracle_fa_f32_to_f16.argtypes = [ctypes.c_float]
    lib.oracle_fa_f32_to_f16.restype = ctypes.c_uint16
    _libs[cr] = lib
    return lib
