"""The graph seam's host side, without a GPU: emel_cuda_layout_view maps
emel-tensor's TensorLayout (row-major dimensions, ElementType;
crates/emel-tensor/src/lib.rs:24-50) to a dense view, and the RunKernelFn
callback emel_cuda_run_kernel (emel-graph processor/kernel_step/sm.rs:126)
reports bad handles through its error code without touching a device."""

import ctypes

import pytest


def test_layout_view_reverses_dimensions_into_dense_strides(emel):
    v = emel.layout_view([3, 5, 7], emel.ElementType.F32, 0x1000, 3 * 5 * 7 * 4)
    assert list(v.ne) == [7, 5, 3, 1] and list(v.nb) == [4, 28, 140, 420] and v.dtype == 0
    v = emel.layout_view([64, 4096], emel.ElementType.F16, 0x2000, 64 * 4096 * 2)
    assert list(v.ne) == [4096, 64, 1, 1] and list(v.nb)[:2] == [2, 8192] and v.dtype == int(emel.DType.F16)
    v = emel.layout_view([9], emel.ElementType.BF16, 0x3000, 18)
    assert list(v.ne) == [9, 1, 1, 1] and v.dtype == 30
    v = emel.layout_view([], emel.ElementType.F32, 0x3000, 4)  # a scalar
    assert list(v.ne) == [1, 1, 1, 1]


@pytest.mark.parametrize("dims,etype,storage", [([4, 4], 3, 1 << 20),      # Quantized: no element size
                                                ([2, 2, 2, 2, 2], 0, 1 << 20),  # rank 5
                                                ([4, 4], 0, 63),           # storage below the dense span
                                                ([4, 4], 7, 1 << 20)])     # unknown element type
def test_layout_view_rejects(emel, dims, etype, storage):
    with pytest.raises(RuntimeError, match="INVALID_ARGUMENT"):
        emel.layout_view(dims, etype, 0x1000, storage)


def test_run_kernel_reports_bad_handles(emel):
    lib = emel.lib()
    err = ctypes.c_int32(-1)
    r = emel.CExecuteRequest()  # no step plan, no compute context
    assert lib.emel_cuda_run_kernel(ctypes.byref(r), ctypes.byref(err)) == 0
    assert err.value == int(emel.Status.INVALID_ARGUMENT)
    assert lib.emel_cuda_run_kernel(None, ctypes.byref(err)) == 0
    assert lib.emel_cuda_run_kernel(ctypes.byref(r), None) == 0


def test_step_create_rejects_without_a_context(emel):
    lib = emel.lib()
    reqs = (emel.CGenericRequest * 1)()
    h = ctypes.c_void_p()
    assert lib.emel_cuda_step_create(None, None, reqs, 1, 0, ctypes.byref(h)) == int(emel.Status.INVALID_ARGUMENT)
    assert not h.value
