"""emel.rs_b200 -- B200 (sm_100a) device op table for the emel-kernels
elementwise, broadcast and reduction operators.

This module is the host-side mirror of the reference operator contract
(stateforward/emel.rs, crates/emel-kernels/src/any/): the same event names,
argument meaning and error behaviour, dispatched through the C ABI of
libemel_cuda.so (include/emel_cuda.h) to hand-written sm_100a kernels.

    k = Kernel(device=0)
    status = k.process_event(OpAdd(lhs, rhs, out))      # binary.rs:47-81
    assert status == Status.OK

Views bind device memory: either a DeviceBuffer allocated through the
library, or any device pointer (e.g. a torch tensor's data_ptr()).  There is
no CPU fallback: without the compiled library or a CUDA device every call
raises.
"""

import ctypes
import struct
import enum
from dataclasses import dataclass
from pathlib import Path
from typing import Optional, Sequence

PACKAGE_DIR = Path(__file__).resolve().parent
LIB_PATH = PACKAGE_DIR / "libemel_cuda.so"


class DType(enum.IntEnum):
    """DType::code() wire values (tensor_view.rs:160-209)."""
    F32 = 0
    F16 = 1
    I32 = 26
    I64 = 27


DTYPE_SIZE = {DType.F32: 4, DType.F16: 2, DType.I32: 4, DType.I64: 8}


class Status(enum.IntEnum):
    OK = 0
    INVALID_VIEW = 1
    SHAPE_MISMATCH = 2
    INVALID_PARAMETERS = 3
    UNEXPECTED_EVENT = 4
    INTERNAL = 5
    INVALID_SHAPE = 6
    UNSUPPORTED_OPERATION = 7
    INVALID_LAYOUT = 8
    INDEX_OUT_OF_BOUNDS = 9
    UNSUPPORTED_SOURCE_STRIDE = 10
    INVALID_MODE = 11
    INVALID_REQUEST = 12
    MODEL_INVALID = 13
    CAPACITY = 14
    PARSE_FAILED = 15
    DEVICE_ERROR = 16
    TIMEOUT = 17
    INVALID_ARGUMENT = 18
    OUT_OF_MEMORY = 19


class BinaryOp(enum.IntEnum):
    ADD = 0
    SUB = 1
    MUL = 2
    DIV = 3


class UnaryOp(enum.IntEnum):
    """UnarySubOp wire codes (unary.rs:101-146) plus the other one-input events."""
    ABS = 0
    SGN = 1
    NEG = 2
    STEP = 3
    TANH = 4
    ELU = 5
    RELU = 6
    SIGMOID = 7
    GELU = 8
    GELU_QUICK = 9
    SILU = 10
    HARDSWISH = 11
    HARDSIGMOID = 12
    EXP = 13
    EXPM1 = 14
    SOFTPLUS = 15
    GELU_ERF = 16
    XIELU = 17
    FLOOR = 18
    CEIL = 19
    ROUND = 20
    TRUNC = 21
    SQR = 64
    SQRT = 65
    LOG = 66
    SIN = 67
    COS = 68


class CView(ctypes.Structure):
    """emel_tensor_view."""
    _fields_ = [("data", ctypes.c_void_p), ("storage_bytes", ctypes.c_uint64), ("ne", ctypes.c_uint64 * 4),
                ("nb", ctypes.c_uint64 * 4), ("dtype", ctypes.c_uint32), ("reserved", ctypes.c_uint32)]


class CArgmaxPartial(ctypes.Structure):
    """emel_cuda_argmax_partial."""
    _fields_ = [("value", ctypes.c_float), ("has_value", ctypes.c_uint32), ("index", ctypes.c_int64),
                ("first_is_nan", ctypes.c_uint32), ("reserved", ctypes.c_uint32)]


class CGenericRequest(ctypes.Structure):
    """emel_cuda_generic_request: GenericRequest (generic.rs:634-645)."""
    _fields_ = [("op", ctypes.c_uint32), ("unary_subop", ctypes.c_uint32),
                ("src0", ctypes.POINTER(CView)), ("src1", ctypes.POINTER(CView)),
                ("src2", ctypes.POINTER(CView)), ("dst", ctypes.POINTER(CView)),
                ("params", ctypes.c_uint8 * 64), ("params_len", ctypes.c_uint32), ("reserved", ctypes.c_uint32)]


class CExecuteRequest(ctypes.Structure):
    """emel_cuda_execute_request: the data fields of emel-graph's processor
    ExecuteRequest (processor/sm.rs:170-199), handles as integers."""
    _fields_ = [("step_plan", ctypes.c_uint64), ("output_out", ctypes.c_uint64), ("lifecycle", ctypes.c_uint64),
                ("tensor_machine", ctypes.c_uint64), ("step_index", ctypes.c_int32), ("step_size", ctypes.c_int32),
                ("kv_tokens", ctypes.c_int32), ("expected_outputs", ctypes.c_int32), ("memory_sm", ctypes.c_uint64),
                ("memory_view", ctypes.c_uint64), ("compute_ctx", ctypes.c_uint64)]


class CGgufRequirements(ctypes.Structure):
    """emel_gguf_requirements: emel-gguf's Requirements (loader/mod.rs:15-27)."""
    _fields_ = [("tensor_count", ctypes.c_uint32), ("kv_count", ctypes.c_uint32), ("max_key_bytes", ctypes.c_uint32),
                ("max_value_bytes", ctypes.c_uint32), ("tensor_data_bytes", ctypes.c_uint64)]


class CGgufTensorInfo(ctypes.Structure):
    """emel_gguf_tensor_info: emel-gguf's TensorInfo (loader/mod.rs:58-84)."""
    _fields_ = [("name_offset", ctypes.c_uint32), ("name_length", ctypes.c_uint32), ("tensor_type", ctypes.c_uint32),
                ("dimension_count", ctypes.c_uint32), ("dimensions", ctypes.c_uint64 * 4),
                ("data_offset", ctypes.c_uint64), ("file_offset", ctypes.c_uint64),
                ("data_section_offset", ctypes.c_uint64), ("alignment", ctypes.c_uint32),
                ("reserved", ctypes.c_uint32), ("data_size", ctypes.c_uint64)]


class CRopeParams(ctypes.Structure):
    """emel_rope_params: rope::RopeParams (rope.rs:33-48)."""
    _fields_ = [("n_dims", ctypes.c_int32), ("mode", ctypes.c_int32), ("freq_base", ctypes.c_float),
                ("freq_scale", ctypes.c_float), ("ext_factor", ctypes.c_float), ("attn_factor", ctypes.c_float)]


class CFlashAttnOptions(ctypes.Structure):
    """emel_flash_attn_options: flash_attn::FlashAttnOptions (flash_attn.rs:24-31)."""
    _fields_ = [("scale", ctypes.c_float), ("has_scale", ctypes.c_uint32),
                ("masked_total_tokens", ctypes.c_uint32), ("has_masked_total_tokens", ctypes.c_uint32)]

    @classmethod
    def of(cls, scale=None, masked_total_tokens=None):
        o = cls()
        if scale is not None:
            o.scale, o.has_scale = scale, 1
        if masked_total_tokens is not None:
            o.masked_total_tokens, o.has_masked_total_tokens = masked_total_tokens, 1
        return o


# Every symbol include/emel_cuda.h declares, with its ctypes signature.
_P = ctypes.POINTER(CView)
_V = ctypes.c_void_p
_CTX = ctypes.c_void_p
_I = ctypes.c_int
_F = ctypes.c_float
SIGNATURES = {
    "emel_cuda_context_create": (_I, [_I, ctypes.POINTER(_CTX)]),
    "emel_cuda_context_destroy": (_I, [_CTX]),
    "emel_cuda_context_last_error": (ctypes.c_char_p, [_CTX]),
    "emel_cuda_malloc": (_I, [_CTX, ctypes.c_uint64, ctypes.POINTER(_V)]),
    "emel_cuda_free": (_I, [_CTX, _V]),
    "emel_cuda_memcpy_h2d": (_I, [_CTX, _V, _V, _V, ctypes.c_uint64]),
    "emel_cuda_memcpy_d2h": (_I, [_CTX, _V, _V, _V, ctypes.c_uint64]),
    "emel_cuda_memset": (_I, [_CTX, _V, _V, _I, ctypes.c_uint64]),
    "emel_cuda_stream_create": (_I, [_CTX, ctypes.POINTER(_V)]),
    "emel_cuda_stream_destroy": (_I, [_CTX, _V]),
    "emel_cuda_stream_synchronize": (_I, [_CTX, _V]),
    "emel_cuda_launch_count": (ctypes.c_uint64, [_CTX]),
    "emel_cuda_event_create": (_I, [_CTX, ctypes.POINTER(_V)]),
    "emel_cuda_event_record": (_I, [_CTX, _V, _V]),
    "emel_cuda_event_record_timed": (_I, [_CTX, _V, _V]),
    "emel_cuda_event_elapsed_ms": (_I, [_CTX, _V, _V, ctypes.POINTER(ctypes.c_float)]),
    "emel_cuda_event_destroy": (_I, [_CTX, _V]),
    "emel_cuda_stream_wait_event": (_I, [_CTX, _V, _V]),
    "emel_cuda_graph_begin": (_I, [_CTX, _V]),
    "emel_cuda_graph_end": (_I, [_CTX, _V, ctypes.POINTER(_V)]),
    "emel_cuda_graph_launch": (_I, [_CTX, _V, _V]),
    "emel_cuda_graph_destroy": (_I, [_CTX, _V]),
    "emel_cuda_binary": (_I, [_CTX, _V, _I, _P, _P, _P]),
    "emel_cuda_broadcast_row": (_I, [_CTX, _V, _I, _P, _P, _P]),
    "emel_cuda_binary_repeat": (_I, [_CTX, _V, _I, _P, _P, _P]),
    "emel_cuda_unary": (_I, [_CTX, _V, _I, _P, _P]),
    "emel_cuda_op_unary": (_I, [_CTX, _V, _I, _P, _P]),
    "emel_cuda_scale": (_I, [_CTX, _V, _P, _P, _F]),
    "emel_cuda_clamp": (_I, [_CTX, _V, _P, _P, _F, _F]),
    "emel_cuda_leaky_relu": (_I, [_CTX, _V, _P, _P, _F]),
    "emel_cuda_silu_back": (_I, [_CTX, _V, _P, _P, _P]),
    "emel_cuda_add1": (_I, [_CTX, _V, _P, _P, _F]),
    "emel_cuda_copy": (_I, [_CTX, _V, _P, _P]),
    "emel_cuda_norm": (_I, [_CTX, _V, _P, _P, _F]),
    "emel_cuda_rms_norm": (_I, [_CTX, _V, _P, _P, _F]),
    "emel_cuda_rms_norm_mul": (_I, [_CTX, _V, _P, _P, _P, _F]),
    "emel_cuda_soft_max": (_I, [_CTX, _V, _P, _P]),
    "emel_cuda_soft_max_ext": (_I, [_CTX, _V, _P, _P, _P, _F]),
    "emel_cuda_sum": (_I, [_CTX, _V, _P, _P]),
    "emel_cuda_sum_f64": (_I, [_CTX, _V, _P, _V]),
    "emel_cuda_sum_noalloc": (_I, [_V, _P, _P]),
    "emel_cuda_mean": (_I, [_CTX, _V, _P, _P]),
    "emel_cuda_sum_rows": (_I, [_CTX, _V, _P, _P]),
    "emel_cuda_argmax": (_I, [_CTX, _V, _P, _P]),
    "emel_cuda_argmax_partial_compute": (_I, [_CTX, _V, _P, ctypes.c_int64, _V]),
    "emel_cuda_argmax_combine": (_I, [ctypes.POINTER(CArgmaxPartial), _I, ctypes.POINTER(ctypes.c_int64),
                                      ctypes.POINTER(ctypes.c_float)]),
    "emel_cuda_argmax_rows": (_I, [_CTX, _V, _P, _P]),
    "emel_cuda_generic": (_I, [_CTX, _V, ctypes.POINTER(CGenericRequest)]),
    "emel_cuda_get_rows": (_I, [_CTX, _V, _P, _P, _P]),
    "emel_cuda_get_rows_f32_bytes": (_I, [_CTX, _V, _P, _P, _P]),
    "emel_cuda_mul_mat_argmax": (_I, [_CTX, _V, _P, _P, _P, _V]),
    "emel_cuda_mul_mat_argmax_q8_0": (_I, [_CTX, _V, _P, _P, _P, _V]),
    "emel_cuda_mul_mat_argmax_q4_0": (_I, [_CTX, _V, _P, _P, _P, _V]),
    "emel_cuda_mul_mat_argmax_q4_1": (_I, [_CTX, _V, _P, _P, _P, _V]),
    "emel_cuda_mul_mat_argmax_q5_0": (_I, [_CTX, _V, _P, _P, _P, _V]),
    "emel_cuda_mul_mat_argmax_q4_k": (_I, [_CTX, _V, _P, _P, _P, _V]),
    "emel_cuda_mul_mat_argmax_q6_k": (_I, [_CTX, _V, _P, _P, _P, _V]),
    "emel_cuda_mul_mat_argmax_q2_k": (_I, [_CTX, _V, _P, _P, _P, _V]),
    "emel_cuda_mul_mat_argmax_q3_k": (_I, [_CTX, _V, _P, _P, _P, _V]),
    "emel_cuda_rope": (_I, [_CTX, _V, _P, _P, _P, ctypes.POINTER(CRopeParams)]),
    "emel_cuda_diag": (_I, [_CTX, _V, _V, ctypes.c_uint64, _V, ctypes.c_uint64]),
    "emel_cuda_diag_mask": (_I, [_CTX, _V, _I, _V, ctypes.c_uint64, _V, ctypes.c_uint64, ctypes.c_int32]),
    "emel_cuda_soft_max_diag_mask_inf": (_I, [_CTX, _V, _V, ctypes.c_uint64, _V, ctypes.c_uint64, ctypes.c_int32]),
    "emel_cuda_flash_attn_ext": (_I, [_CTX, _V, _P, _P, _P, _P, ctypes.POINTER(CFlashAttnOptions)]),
    "emel_cuda_flash_attn_workspace": (_I, [_CTX, ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64)]),
    "emel_cuda_cpy": (_I, [_CTX, _V, _P, _P]),
    "emel_cuda_cont": (_I, [_CTX, _V, _P, _P]),
    "emel_cuda_glu": (_I, [_CTX, _V, _I, _V, ctypes.c_uint64, _V, ctypes.c_uint64]),
    "emel_cuda_exchange_create": (_I, [_CTX, _I, _I, ctypes.c_uint32, ctypes.c_uint32, ctypes.POINTER(_V)]),
    "emel_cuda_exchange_handle": (_I, [_V, _V]),
    "emel_cuda_exchange_connect": (_I, [_CTX, _V, _V]),
    "emel_cuda_exchange_publish": (_I, [_CTX, _V, _V, _V]),
    "emel_cuda_exchange_wait": (_I, [_CTX, _V, _V, _V]),
    "emel_cuda_exchange_wait_sum_argmax": (_I, [_CTX, _V, _V, _V, _P, _P]),
    "emel_cuda_exchange_destroy": (_I, [_CTX, _V]),
    "emel_cuda_step_create": (_I, [_CTX, _V, ctypes.POINTER(CGenericRequest), ctypes.c_uint32, ctypes.c_uint32,
                                   ctypes.POINTER(_V)]),
    "emel_cuda_step_destroy": (_I, [_CTX, _V]),
    "emel_cuda_step_runs": (ctypes.c_uint64, [_V]),
    "emel_cuda_run_kernel": (_I, [ctypes.POINTER(CExecuteRequest), ctypes.POINTER(ctypes.c_int32)]),
    "emel_cuda_layout_view": (_I, [ctypes.POINTER(ctypes.c_uint64), ctypes.c_uint32, ctypes.c_uint32, _V,
                                   ctypes.c_uint64, _P]),
    "emel_gguf_probe": (_I, [_V, ctypes.c_uint64, ctypes.POINTER(CGgufRequirements)]),
    "emel_gguf_parse": (_I, [_V, ctypes.c_uint64, ctypes.POINTER(CGgufRequirements), ctypes.POINTER(CGgufTensorInfo),
                             ctypes.c_uint32]),
    "emel_gguf_tensor_view": (_I, [ctypes.POINTER(CGgufTensorInfo), _V, ctypes.c_uint64, _P]),
    "emel_gguf_upload": (_I, [_CTX, _V, _V, ctypes.c_uint64, ctypes.POINTER(CGgufTensorInfo), _V, ctypes.c_uint64,
                              _P]),
}

_lib = None


def lib():
    """The loaded device library.  Raises when it has not been built: the
    operators have no CPU path."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise RuntimeError(f"{LIB_PATH} is missing: build it with `make -C emel.rs_b200/csrc` "
                           "(the device op table has no CPU fallback)")
    handle = ctypes.CDLL(str(LIB_PATH))
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(handle, name)
        fn.restype = res
        fn.argtypes = args
    _lib = handle
    return handle


# ---------------------------------------------------------------------------
# Layouts and views (tensor_view.rs:215-448, 537-898)
# ---------------------------------------------------------------------------

def contiguous_nb(ne: Sequence[int], dtype: DType = DType.F32):
    nb = [DTYPE_SIZE[DType(dtype)]]
    for d in range(1, 4):
        nb.append(nb[-1] * int(ne[d - 1]))
    return nb


@dataclass(frozen=True)
class Layout:
    """Layout { dtype, ne[4], nb[4] } (tensor_view.rs:215-219); nb in bytes,
    nb[0] == 0 means implicit row-major."""
    dtype: DType
    ne: tuple
    nb: tuple

    @staticmethod
    def contiguous(dtype, ne):
        ne = tuple(int(x) for x in ne)
        return Layout(DType(dtype), ne, tuple(contiguous_nb(ne, dtype)))

    @staticmethod
    def new(dtype, ne, nb):
        return Layout(DType(dtype), tuple(int(x) for x in ne), tuple(int(x) for x in nb))

    def permuted(self, axes):
        """Layout::permuted (tensor_view.rs:318-332)."""
        return Layout(self.dtype, tuple(self.ne[a] for a in axes), tuple(self.nb[a] for a in axes))


@dataclass
class TensorView:
    """A layout bound to device storage: `ptr` is a device address and
    `storage_bytes` how far the view may reach (the slice length)."""
    ptr: int
    storage_bytes: int
    layout: Layout

    def c(self) -> CView:
        v = CView()
        v.data = self.ptr
        v.storage_bytes = self.storage_bytes
        for d in range(4):
            v.ne[d] = self.layout.ne[d]
            v.nb[d] = self.layout.nb[d]
        v.dtype = int(self.layout.dtype)
        v.reserved = 0
        return v


TensorViewMut = TensorView


def _check(status, what="call"):
    st = Status(status)
    if st != Status.OK:
        raise RuntimeError(f"{what} failed with {st.name}")
    return st


class Context:
    """emel_cuda_context: device selection, reduction workspace, handles."""

    def __init__(self, device: int = 0):
        self._lib = lib()
        h = ctypes.c_void_p()
        st = self._lib.emel_cuda_context_create(device, ctypes.byref(h))
        if st != 0:
            raise RuntimeError(f"emel_cuda_context_create(device={device}) failed: {Status(st).name}")
        self.handle = h
        self.device = device

    def close(self):
        if self.handle:
            self._lib.emel_cuda_context_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def last_error(self):
        return self._lib.emel_cuda_context_last_error(self.handle).decode()

    @property
    def launches(self):
        return int(self._lib.emel_cuda_launch_count(self.handle))

    def synchronize(self, stream=None):
        _check(self._lib.emel_cuda_stream_synchronize(self.handle, stream), "stream synchronize")


class Stream:
    """A non-blocking stream created by the library (capturable)."""

    def __init__(self, ctx: Context):
        self.ctx = ctx
        h = ctypes.c_void_p()
        _check(ctx._lib.emel_cuda_stream_create(ctx.handle, ctypes.byref(h)), "stream create")
        self.handle = h

    def synchronize(self):
        self.ctx.synchronize(self.handle)

    def wait(self, event: "CudaEvent"):
        _check(self.ctx._lib.emel_cuda_stream_wait_event(self.ctx.handle, self.handle, event.handle), "stream wait")

    def close(self):
        if self.handle:
            self.ctx._lib.emel_cuda_stream_destroy(self.ctx.handle, self.handle)
            self.handle = None


class CudaEvent:
    """A timing event (emel_cuda_event_*)."""

    def __init__(self, ctx: Context):
        self.ctx = ctx
        h = ctypes.c_void_p()
        _check(ctx._lib.emel_cuda_event_create(ctx.handle, ctypes.byref(h)), "event create")
        self.handle = h

    def record(self, stream):
        """Plain record; inside a capture it is a dependency (fork / join)."""
        _check(self.ctx._lib.emel_cuda_event_record(self.ctx.handle, self.handle, stream), "event record")

    def record_timed(self, stream):
        """Inside a capture: an event-record node, for timing graph kernels."""
        _check(self.ctx._lib.emel_cuda_event_record_timed(self.ctx.handle, self.handle, stream), "event record")

    def elapsed_ms(self, end: "CudaEvent") -> float:
        ms = ctypes.c_float()
        _check(self.ctx._lib.emel_cuda_event_elapsed_ms(self.ctx.handle, self.handle, end.handle, ctypes.byref(ms)),
               "event elapsed")
        return ms.value


class Graph:
    """Captures every entry point called on `stream` inside the `with` block
    into one CUDA graph; launch() replays it."""

    def __init__(self, ctx: Context, stream: Stream):
        self.ctx, self.stream, self.handle = ctx, stream, None

    def __enter__(self):
        _check(self.ctx._lib.emel_cuda_graph_begin(self.ctx.handle, self.stream.handle), "graph begin")
        return self

    def __exit__(self, exc_type, exc, tb):
        h = ctypes.c_void_p()
        st = self.ctx._lib.emel_cuda_graph_end(self.ctx.handle, self.stream.handle, ctypes.byref(h))
        if exc_type is None:
            _check(st, "graph end")
        self.handle = h

    def launch(self):
        _check(self.ctx._lib.emel_cuda_graph_launch(self.ctx.handle, self.handle, self.stream.handle), "graph launch")

    def close(self):
        if self.handle:
            self.ctx._lib.emel_cuda_graph_destroy(self.ctx.handle, self.handle)
            self.handle = None


class DeviceBuffer:
    """Device memory owned through the library (emel_cuda_malloc)."""

    def __init__(self, ctx: Context, nbytes: int):
        self.ctx = ctx
        self.nbytes = int(nbytes)
        p = ctypes.c_void_p()
        _check(ctx._lib.emel_cuda_malloc(ctx.handle, max(self.nbytes, 1), ctypes.byref(p)), "malloc")
        self.ptr = p.value

    def upload(self, array, stream=None):
        """Copies a host numpy array into the start of the buffer and waits."""
        _check(self.ctx._lib.emel_cuda_memcpy_h2d(self.ctx.handle, stream, self.ptr, array.ctypes.data, array.nbytes), "h2d")
        self.ctx.synchronize(stream)

    def download(self, array, stream=None):
        _check(self.ctx._lib.emel_cuda_memcpy_d2h(self.ctx.handle, stream, array.ctypes.data, self.ptr, array.nbytes), "d2h")
        self.ctx.synchronize(stream)
        return array

    def view(self, layout: Layout, storage_bytes: Optional[int] = None) -> TensorView:
        return TensorView(self.ptr, self.nbytes if storage_bytes is None else storage_bytes, layout)

    def free(self):
        if self.ptr:
            self.ctx._lib.emel_cuda_free(self.ctx.handle, self.ptr)
            self.ptr = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


# ---------------------------------------------------------------------------
# Events (crates/emel-kernels/src/any/event.rs and the per-family modules)
# ---------------------------------------------------------------------------

class Event:
    def dispatch(self, ctx: Context, stream) -> int:
        raise NotImplementedError


def _r(view):
    """A TensorView (or an already-built CView) as an emel_tensor_view pointer."""
    if view is None:
        return None
    return ctypes.byref(view if isinstance(view, CView) else view.c())


@dataclass
class _Binary(Event):
    lhs: TensorView
    rhs: TensorView
    output: TensorView
    OP = BinaryOp.ADD

    def dispatch(self, ctx, stream):
        return ctx._lib.emel_cuda_binary(ctx.handle, stream, int(self.OP), _r(self.lhs), _r(self.rhs), _r(self.output))


class OpAdd(_Binary):
    """binary::OpAdd (binary.rs:78)."""
    OP = BinaryOp.ADD


class OpSub(_Binary):
    OP = BinaryOp.SUB


class OpMul(_Binary):
    OP = BinaryOp.MUL


class OpDiv(_Binary):
    OP = BinaryOp.DIV


@dataclass
class _BroadcastRow(Event):
    src0: TensorView
    src1: TensorView
    dst: TensorView
    OP = BinaryOp.ADD

    def dispatch(self, ctx, stream):
        return ctx._lib.emel_cuda_broadcast_row(ctx.handle, stream, int(self.OP), _r(self.src0), _r(self.src1), _r(self.dst))


class OpAddBroadcastRow(_BroadcastRow):
    """broadcast::OpAddBroadcastRow (broadcast.rs:53-67)."""
    OP = BinaryOp.ADD


class OpSubBroadcastRow(_BroadcastRow):
    OP = BinaryOp.SUB


class OpMulBroadcastRow(_BroadcastRow):
    """broadcast::OpMulBroadcastRow (broadcast.rs:69-84)."""
    OP = BinaryOp.MUL


class OpDivBroadcastRow(_BroadcastRow):
    OP = BinaryOp.DIV


@dataclass
class OpBinaryRepeat(Event):
    """Repeat src1 to dst's extents (generic.rs:1641-1665), then op."""
    op: BinaryOp
    src0: TensorView
    src1: TensorView
    dst: TensorView

    def dispatch(self, ctx, stream):
        return ctx._lib.emel_cuda_binary_repeat(ctx.handle, stream, int(self.op), _r(self.src0), _r(self.src1), _r(self.dst))


@dataclass
class OpUnaryTyped(Event):
    """The typed unary events OpAbs..OpTrunc, OpSqr, OpSqrt, OpLog, OpSin, OpCos."""
    op: UnaryOp
    input: TensorView
    output: TensorView

    def dispatch(self, ctx, stream):
        return ctx._lib.emel_cuda_unary(ctx.handle, stream, int(self.op), _r(self.input), _r(self.output))


def _typed(op):
    def make(input, output):
        return OpUnaryTyped(op, input, output)
    return make


OpAbs, OpSgn, OpNeg, OpStep = _typed(UnaryOp.ABS), _typed(UnaryOp.SGN), _typed(UnaryOp.NEG), _typed(UnaryOp.STEP)
OpTanh, OpElu, OpRelu, OpSigmoid = _typed(UnaryOp.TANH), _typed(UnaryOp.ELU), _typed(UnaryOp.RELU), _typed(UnaryOp.SIGMOID)
OpGelu, OpGeluQuick, OpSilu = _typed(UnaryOp.GELU), _typed(UnaryOp.GELU_QUICK), _typed(UnaryOp.SILU)
OpHardswish, OpHardsigmoid = _typed(UnaryOp.HARDSWISH), _typed(UnaryOp.HARDSIGMOID)
OpExp, OpExpm1, OpSoftplus, OpGeluErf = _typed(UnaryOp.EXP), _typed(UnaryOp.EXPM1), _typed(UnaryOp.SOFTPLUS), _typed(UnaryOp.GELU_ERF)
OpFloor, OpCeil, OpRound, OpTrunc = _typed(UnaryOp.FLOOR), _typed(UnaryOp.CEIL), _typed(UnaryOp.ROUND), _typed(UnaryOp.TRUNC)
OpSqr, OpSqrt = _typed(UnaryOp.SQR), _typed(UnaryOp.SQRT)
OpLog, OpSin, OpCos = _typed(UnaryOp.LOG), _typed(UnaryOp.SIN), _typed(UnaryOp.COS)


@dataclass
class OpUnary(Event):
    """Generic unary::OpUnary (unary.rs:148-172): eight accepted subops."""
    subop: UnaryOp
    input: TensorView
    output: TensorView

    def dispatch(self, ctx, stream):
        return ctx._lib.emel_cuda_op_unary(ctx.handle, stream, int(self.subop), _r(self.input), _r(self.output))


@dataclass
class OpScale(Event):
    """activation::OpScale (activation.rs:58)."""
    input: TensorView
    output: TensorView
    scale: float

    def dispatch(self, ctx, stream):
        return ctx._lib.emel_cuda_scale(ctx.handle, stream, _r(self.input), _r(self.output), self.scale)


@dataclass
class OpClamp(Event):
    input: TensorView
    output: TensorView
    min: float
    max: float

    def dispatch(self, ctx, stream):
        return ctx._lib.emel_cuda_clamp(ctx.handle, stream, _r(self.input), _r(self.output), self.min, self.max)


@dataclass
class OpLeakyRelu(Event):
    input: TensorView
    output: TensorView
    negative_slope: float

    def dispatch(self, ctx, stream):
        return ctx._lib.emel_cuda_leaky_relu(ctx.handle, stream, _r(self.input), _r(self.output), self.negative_slope)


@dataclass
class OpSiluBack(Event):
    input: TensorView
    gradient: TensorView
    output: TensorView

    def dispatch(self, ctx, stream):
        return ctx._lib.emel_cuda_silu_back(ctx.handle, stream, _r(self.input), _r(self.gradient), _r(self.output))


@dataclass
class OpAdd1(Event):
    src: TensorView
    dst: TensorView
    scalar: float

    def dispatch(self, ctx, stream):
        return ctx._lib.emel_cuda_add1(ctx.handle, stream, _r(self.src), _r(self.dst), self.scalar)


@dataclass
class CopyTensor(Event):
    """tensor_view::CopyTensor (tensor_view.rs:954-967)."""
    src: TensorView
    dst: TensorView

    def dispatch(self, ctx, stream):
        return ctx._lib.emel_cuda_copy(ctx.handle, stream, _r(self.src), _r(self.dst))


@dataclass
class OpGetRows(Event):
    """get_rows::OpGetRows and its F16 / BF16 / Q4_0 / Q8_0 / Q4_K variants
    (get_rows.rs:219-512), chosen by the source view's dtype; `indices` is
    an I32 view with ne[3] == 1."""
    src: TensorView
    indices: TensorView
    dst: TensorView

    def dispatch(self, ctx, stream):
        return ctx._lib.emel_cuda_get_rows(ctx.handle, stream, _r(self.src), _r(self.indices), _r(self.dst))


@dataclass
class OpGetRowsF32Bytes(Event):
    """get_rows::OpGetRowsF32Bytes (get_rows.rs:233-255): F32 rows of a
    byte-backed source whose strides may be any byte count."""
    src: TensorView
    indices: TensorView
    dst: TensorView

    def dispatch(self, ctx, stream):
        return ctx._lib.emel_cuda_get_rows_f32_bytes(ctx.handle, stream, _r(self.src), _r(self.indices),
                                                     _r(self.dst))


@dataclass
class OpRope(Event):
    """rope::OpRope (rope.rs:135-160); params: CRopeParams or a dict of its fields."""
    source: TensorView
    positions: TensorView
    destination: TensorView
    params: object

    def dispatch(self, ctx, stream):
        pr = self.params if isinstance(self.params, CRopeParams) else CRopeParams(**self.params)
        return ctx._lib.emel_cuda_rope(ctx.handle, stream, _r(self.source), _r(self.positions), _r(self.destination),
                                       ctypes.byref(pr))


@dataclass
class OpMulMatArgmax(Event):
    """matmul::OpMulMatArgmax (matmul.rs:167-192): lhs [k, m], rhs [1, k],
    dst [1]; the best row goes to the device int32 at `index_ptr`."""
    lhs: TensorView
    rhs: TensorView
    destination: TensorView
    index_ptr: int

    def dispatch(self, ctx, stream):
        return ctx._lib.emel_cuda_mul_mat_argmax(ctx.handle, stream, _r(self.lhs), _r(self.rhs),
                                                 _r(self.destination), ctypes.c_void_p(self.index_ptr))


@dataclass
class OpDiag(Event):
    """diag::OpDiag::new(input, output) (diag.rs:44-66): device pointers to
    input_len and input_len^2 floats."""
    input: int
    input_len: int
    output: int
    output_len: int

    def dispatch(self, ctx, stream):
        return ctx._lib.emel_cuda_diag(ctx.handle, stream, ctypes.c_void_p(self.input), self.input_len,
                                       ctypes.c_void_p(self.output), self.output_len)


@dataclass
class _DiagMask(Event):
    input: int
    input_len: int
    output: int
    output_len: int
    n_past: int
    MODE = 0

    def dispatch(self, ctx, stream):
        return ctx._lib.emel_cuda_diag_mask(ctx.handle, stream, self.MODE, ctypes.c_void_p(self.input),
                                            self.input_len, ctypes.c_void_p(self.output), self.output_len,
                                            self.n_past)


class OpDiagMaskInf(_DiagMask):
    """diag::OpDiagMaskInf::new(input, output, n_past) (diag.rs:68-86)."""
    MODE = 0


class OpDiagMaskZero(_DiagMask):
    """diag::OpDiagMaskZero::new(input, output, n_past) (diag.rs:88-108)."""
    MODE = 1


@dataclass
class SoftMaxDiagMaskInf(Event):
    """diag::OpDiagMaskInf then reductions::OpSoftMax over the dense [side,
    side] result, fused (emel_cuda_soft_max_diag_mask_inf)."""
    input: int
    input_len: int
    output: int
    output_len: int
    n_past: int

    def dispatch(self, ctx, stream):
        return ctx._lib.emel_cuda_soft_max_diag_mask_inf(ctx.handle, stream, ctypes.c_void_p(self.input),
                                                         self.input_len, ctypes.c_void_p(self.output),
                                                         self.output_len, self.n_past)


@dataclass
class OpFlashAttnExt(Event):
    """flash_attn::OpFlashAttnExt::new(query, key, value, destination, options)
    (flash_attn.rs:78-99): query / destination F32 [d, 1, heads, 1], key /
    value F16 [d, tokens, kv_heads, 1]; options: FlashAttnOptions fields
    (scale, masked_total_tokens), None for the defaults."""
    query: TensorView
    key: TensorView
    value: TensorView
    destination: TensorView
    scale: Optional[float] = None
    masked_total_tokens: Optional[int] = None

    def dispatch(self, ctx, stream):
        opts = CFlashAttnOptions.of(self.scale, self.masked_total_tokens)
        return ctx._lib.emel_cuda_flash_attn_ext(ctx.handle, stream, _r(self.query), _r(self.key), _r(self.value),
                                                 _r(self.destination), ctypes.byref(opts))


def flash_attn_workspace(ctx: "Context"):
    """FlashAttnKernel::prepared_tokens / reuse_count (flash_attn.rs:205-215)
    of the context: (tokens of the last accepted call, consecutive repeats)."""
    prepared, reuse = ctypes.c_uint64(), ctypes.c_uint64()
    _check(ctx._lib.emel_cuda_flash_attn_workspace(ctx.handle, ctypes.byref(prepared), ctypes.byref(reuse)),
           "flash_attn_workspace")
    return prepared.value, reuse.value


@dataclass
class OpMulMatArgmaxQ8_0(Event):
    """matmul::OpMulMatArgmaxQ8_0 (matmul.rs:500-520): lhs Q8_0 packed rows
    [k, m], rhs [1, k] F32, dst [1]; the best row goes to the device int32
    at `index_ptr`."""
    lhs: TensorView
    rhs: TensorView
    destination: TensorView
    index_ptr: int

    def dispatch(self, ctx, stream):
        return ctx._lib.emel_cuda_mul_mat_argmax_q8_0(ctx.handle, stream, _r(self.lhs), _r(self.rhs),
                                                      _r(self.destination), ctypes.c_void_p(self.index_ptr))


def _packed_argmax(suffix, doc):
    @dataclass
    class E(Event):
        lhs: TensorView
        rhs: TensorView
        destination: TensorView
        index_ptr: int

        def dispatch(self, ctx, stream):
            fn = getattr(ctx._lib, f"emel_cuda_mul_mat_argmax_{suffix}")
            return fn(ctx.handle, stream, _r(self.lhs), _r(self.rhs), _r(self.destination),
                      ctypes.c_void_p(self.index_ptr))
    E.__doc__ = doc
    E.__name__ = E.__qualname__ = f"OpMulMatArgmax{suffix.upper()}"
    return E


OpMulMatArgmaxQ4_0 = _packed_argmax("q4_0", "matmul::OpMulMatArgmaxQ4_0 (matmul.rs:490-500): Q4_0 rows.")
OpMulMatArgmaxQ4_1 = _packed_argmax("q4_1", "matmul::OpMulMatArgmaxQ4_1 (matmul.rs:500-510): Q4_1 rows.")
OpMulMatArgmaxQ5_0 = _packed_argmax("q5_0", "matmul::OpMulMatArgmaxQ5_0 (matmul.rs:510-516): Q5_0 rows.")
OpMulMatArgmaxQ4K = _packed_argmax("q4_k", "matmul::OpMulMatArgmaxQ4K (matmul.rs:530-535): Q4_K rows.")
OpMulMatArgmaxQ6K = _packed_argmax("q6_k", "matmul::OpMulMatArgmaxQ6K (matmul.rs:536-540): Q6_K rows.")
OpMulMatArgmaxQ2K = _packed_argmax("q2_k", "matmul::OpMulMatArgmaxQ2K (matmul.rs:520-524): Q2_K rows.")
OpMulMatArgmaxQ3K = _packed_argmax("q3_k", "matmul::OpMulMatArgmaxQ3K (matmul.rs:525-529): Q3_K rows.")


@dataclass
class OpCpy(Event):
    """shape::OpCpy (shape.rs:55-69): ordinal copy between count-equal views."""
    src: TensorView
    dst: TensorView

    def dispatch(self, ctx, stream):
        return ctx._lib.emel_cuda_cpy(ctx.handle, stream, _r(self.src), _r(self.dst))


@dataclass
class OpCont(Event):
    """shape::OpCont (shape.rs:71-84): OpCpy into a dense row-major destination."""
    src: TensorView
    dst: TensorView

    def dispatch(self, ctx, stream):
        return ctx._lib.emel_cuda_cont(ctx.handle, stream, _r(self.src), _r(self.dst))


@dataclass
class OpNorm(Event):
    """normalization::OpNorm (normalization.rs:58-76)."""
    input: TensorView
    output: TensorView
    epsilon: float

    def dispatch(self, ctx, stream):
        return ctx._lib.emel_cuda_norm(ctx.handle, stream, _r(self.input), _r(self.output), self.epsilon)


@dataclass
class OpRmsNorm(Event):
    """normalization::OpRmsNorm (normalization.rs:78-96)."""
    input: TensorView
    output: TensorView
    epsilon: float

    def dispatch(self, ctx, stream):
        return ctx._lib.emel_cuda_rms_norm(ctx.handle, stream, _r(self.input), _r(self.output), self.epsilon)


@dataclass
class OpRmsNormMul(Event):
    """OpRmsNorm then OpMulBroadcastRow by `weight`, fused."""
    input: TensorView
    weight: TensorView
    output: TensorView
    epsilon: float

    def dispatch(self, ctx, stream):
        return ctx._lib.emel_cuda_rms_norm_mul(ctx.handle, stream, _r(self.input), _r(self.weight), _r(self.output),
                                               self.epsilon)


@dataclass
class OpSoftMax(Event):
    """reductions::OpSoftMax (reductions.rs:150-163)."""
    src: TensorView
    dst: TensorView

    def dispatch(self, ctx, stream):
        return ctx._lib.emel_cuda_soft_max(ctx.handle, stream, _r(self.src), _r(self.dst))


@dataclass
class OpSoftMaxExt(Event):
    """Softmax of src * scale + mask (mask optional, F16 or F32)."""
    src: TensorView
    mask: Optional[TensorView]
    dst: TensorView
    scale: float

    def dispatch(self, ctx, stream):
        return ctx._lib.emel_cuda_soft_max_ext(ctx.handle, stream, _r(self.src), _r(self.mask), _r(self.dst), self.scale)


def _reduce(name, doc):
    @dataclass
    class R(Event):
        src: TensorView
        dst: TensorView

        def dispatch(self, ctx, stream):
            return getattr(ctx._lib, name)(ctx.handle, stream, _r(self.src), _r(self.dst))
    R.__doc__ = doc
    return R


OpSum = _reduce("emel_cuda_sum", "reductions::OpSum (reductions.rs:90-103).")
OpMean = _reduce("emel_cuda_mean", "reductions::OpMean (reductions.rs:120-133).")
OpSumRows = _reduce("emel_cuda_sum_rows", "reductions::OpSumRows (reductions.rs:105-118).")
OpArgmax = _reduce("emel_cuda_argmax", "reductions::OpArgmax (reductions.rs:135-148).")
OpArgmaxRows = _reduce("emel_cuda_argmax_rows", "Per-row argmax (reductions.rs:715-730 per row).")


class KernelOperation(enum.IntEnum):
    """KernelOperation wire codes of the routes the device table executes
    (generic.rs:220-316); every other code in 0..94 is accepted by the
    envelope and answered with UNSUPPORTED_OPERATION."""
    DUP = 0
    ADD = 1
    ADD1 = 3
    SUB = 5
    MUL = 6
    DIV = 7
    SQR = 8
    SQRT = 9
    LOG = 10
    SIN = 11
    COS = 12
    SUM = 13
    MEAN = 16
    ARGMAX = 17
    REPEAT = 19
    SILU_BACK = 22
    NORM = 23
    RMS_NORM = 24
    SCALE = 32
    SOFT_MAX = 46
    CLAMP = 50
    LEAKY_RELU = 70
    UNARY = 85


def op_params(*values):
    """OpParams from 4-byte slots: floats as f32, ints as i32 (native order)."""
    raw = b"".join(struct.pack("=f", v) if isinstance(v, float) else struct.pack("=i", v) for v in values)
    if len(raw) > 64:
        raise ValueError("op_params holds 64 bytes")
    return raw


@dataclass
class GenericEvent(Event):
    """GenericEvent(GenericRequest) (generic.rs:634-797): an op-coded request
    with up to three sources, a destination, the op_params bytes and, for
    KernelOperation.UNARY, a UnarySubOp code."""
    op: int
    src0: Optional[TensorView] = None
    src1: Optional[TensorView] = None
    src2: Optional[TensorView] = None
    dst: Optional[TensorView] = None
    params: bytes = b""
    unary: int = 0

    def request(self) -> CGenericRequest:
        r = CGenericRequest()
        r.op = int(self.op)
        r.unary_subop = int(self.unary)
        self._keep = []
        for name in ("src0", "src1", "src2", "dst"):
            v = getattr(self, name)
            if v is not None:
                c = v.c()
                self._keep.append(c)
                setattr(r, name, ctypes.pointer(c))
        ctypes.memmove(r.params, bytes(self.params), len(self.params))
        r.params_len = len(self.params)
        return r

    def dispatch(self, ctx, stream):
        r = self.request()
        return ctx._lib.emel_cuda_generic(ctx.handle if ctx is not None else None, stream, ctypes.byref(r))


class GluSubOp(enum.IntEnum):
    """glu::GluSubOp wire codes (glu.rs:22-38)."""
    REGLU = 0
    GEGLU = 1
    SWIGLU = 2
    SWIGLU_OAI = 3
    GEGLU_ERF = 4
    GEGLU_QUICK = 5


@dataclass
class OpGlu(Event):
    """glu::OpGlu::new(input, output, subop) (glu.rs:66-82) over device f32
    arrays: `input` and `output` are (device pointer, element count) pairs,
    the counterpart of the reference's slices."""
    input: tuple
    output: tuple
    subop: GluSubOp

    def dispatch(self, ctx, stream):
        (ip, il), (op, ol) = self.input, self.output
        return ctx._lib.emel_cuda_glu(ctx.handle, stream, int(self.subop), ctypes.c_void_p(ip), il,
                                      ctypes.c_void_p(op), ol)


class Kernel:
    """Mirror of emel_kernels::Kernel (actor.rs:905-949): single-writer,
    dispatches one typed event per call.  Device work is enqueued on
    `stream` (None = legacy default stream); process_event returns the
    reference-style status without waiting for the device unless
    `synchronize` is set."""

    def __init__(self, device: int = 0, ctx: Optional[Context] = None, stream=None, synchronize: bool = False):
        self.ctx = ctx or Context(device)
        self.stream = stream
        self.synchronize = synchronize

    def process_event(self, event: Event) -> Status:
        st = Status(event.dispatch(self.ctx, self.stream))
        if st == Status.OK and self.synchronize:
            self.ctx.synchronize(self.stream)
        return st


def argmax_combine(partials):
    """Combines per-shard (value, has_value, index, first_is_nan) tuples in
    shard order through emel_cuda_argmax_combine."""
    arr = (CArgmaxPartial * len(partials))()
    for k, (value, has, index, first_nan) in enumerate(partials):
        arr[k].value = value
        arr[k].has_value = has
        arr[k].index = index
        arr[k].first_is_nan = first_nan
    idx = ctypes.c_int64()
    val = ctypes.c_float()
    _check(lib().emel_cuda_argmax_combine(arr, len(partials), ctypes.byref(idx), ctypes.byref(val)), "argmax_combine")
    return idx.value, val.value


# ---------------------------------------------------------------------------
# Graph seam: a device kernel step run through the RunKernelFn callback
# (emel-graph processor/kernel_step/sm.rs:125-126)
# ---------------------------------------------------------------------------

STEP_CAPTURE = 1
STEP_ASYNC = 2


class ElementType(enum.IntEnum):
    """emel-tensor's ElementType (crates/emel-tensor/src/lib.rs:8-20)."""
    F32 = 0
    F16 = 1
    BF16 = 2
    QUANTIZED = 3


def layout_view(dimensions, element_type, data_ptr: int, storage_bytes: int) -> "CView":
    """The dense device view of a TensorLayout (row-major dimensions,
    element type) stored at `data_ptr`, through emel_cuda_layout_view."""
    dims = (ctypes.c_uint64 * max(1, len(dimensions)))(*[int(d) for d in dimensions])
    out = CView()
    _check(lib().emel_cuda_layout_view(dims, len(dimensions), int(element_type), ctypes.c_void_p(data_ptr),
                                       storage_bytes, ctypes.byref(out)), "layout_view")
    return out


class KernelStep:
    """A processor step on the device: the generic events, in order, as one
    emel_cuda_step; run() calls emel_cuda_run_kernel with an ExecuteRequest
    naming the step and the context, as the processor's RunKernelFn would."""

    def __init__(self, ctx: Context, stream, events, capture: bool = False, asynchronous: bool = False):
        self.ctx = ctx
        reqs = (CGenericRequest * len(events))()
        keep = []
        for k, ev in enumerate(events):
            r = ev.request()
            keep.append(ev)
            ctypes.memmove(ctypes.addressof(reqs[k]), ctypes.addressof(r), ctypes.sizeof(r))
        flags = (STEP_CAPTURE if capture else 0) | (STEP_ASYNC if asynchronous else 0)
        h = ctypes.c_void_p()
        self.stream = stream
        _check(ctx._lib.emel_cuda_step_create(ctx.handle, stream, reqs, len(events), flags, ctypes.byref(h)),
               "step create")  # the step copied the requests and their views
        self.handle = h

    def request(self, step_index: int = 0) -> CExecuteRequest:
        r = CExecuteRequest()
        r.step_plan = self.handle.value or 0
        r.compute_ctx = self.ctx.handle.value or 0
        r.step_index = step_index
        r.step_size = 1
        return r

    def run(self, step_index: int = 0):
        """(ok, status) of one RunKernelFn call."""
        err = ctypes.c_int32(-1)
        ok = self.ctx._lib.emel_cuda_run_kernel(ctypes.byref(self.request(step_index)), ctypes.byref(err))
        return bool(ok), Status(err.value)

    @property
    def runs(self) -> int:
        return int(self.ctx._lib.emel_cuda_step_runs(self.handle))

    def close(self):
        if self.handle:
            self.ctx._lib.emel_cuda_step_destroy(self.ctx.handle, self.handle)
            self.handle = None


# ---------------------------------------------------------------------------
# GGUF tensor tables into device buffers (emel-gguf loader/mod.rs:137-232)
# ---------------------------------------------------------------------------

class GgufError(RuntimeError):
    def __init__(self, status, what):
        super().__init__(f"{what}: {Status(status).name}")
        self.status = Status(status)


class GgufImage:
    """A GGUF image in host memory, probed then parsed (the reference's
    probe -> bind -> parse: the record storage is allocated here from the
    probed requirements).  tensors: list of (name, CGgufTensorInfo)."""

    def __init__(self, image: bytes):
        self.image = bytes(image)
        self._buf = ctypes.create_string_buffer(self.image, len(self.image)) if self.image else None
        ptr = ctypes.cast(self._buf, ctypes.c_void_p) if self._buf is not None else None
        self.requirements = CGgufRequirements()
        st = lib().emel_gguf_probe(ptr, len(self.image), ctypes.byref(self.requirements))
        if st != 0:
            raise GgufError(st, "gguf probe")
        n = self.requirements.tensor_count
        self._records = (CGgufTensorInfo * max(1, n))()
        st = lib().emel_gguf_parse(ptr, len(self.image), ctypes.byref(self.requirements), self._records, n)
        if st != 0:
            raise GgufError(st, "gguf parse")
        self.tensors = []
        for k in range(n):
            t = self._records[k]
            self.tensors.append((self.image[t.name_offset:t.name_offset + t.name_length].decode("utf-8", "replace"), t))

    def record(self, name: str) -> CGgufTensorInfo:
        for n, t in self.tensors:
            if n == name:
                return t
        raise KeyError(name)

    def upload(self, ctx: Context, name: str, stream=None):
        """(DeviceBuffer, CView) holding the tensor's serialized bytes."""
        t = self.record(name)
        buf = DeviceBuffer(ctx, max(16, t.data_size))
        view = CView()
        _check(ctx._lib.emel_gguf_upload(ctx.handle, stream, ctypes.cast(self._buf, ctypes.c_void_p), len(self.image),
                                         ctypes.byref(t), ctypes.c_void_p(buf.ptr), max(16, t.data_size),
                                         ctypes.byref(view)), f"gguf upload {name}")
        return buf, view
