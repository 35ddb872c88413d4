"""GGUF tensors into device buffers, end to end: a synthetic model image
(tests/gguf_writer.py) holding a Q4_K and a Q8_0 vocabulary matrix and an
F32 embedding table is probed and parsed (emel_gguf_probe / emel_gguf_parse,
the reference loader's scanner), each tensor is uploaded with
emel_gguf_upload, and the device kernels run on the uploaded views: the
vocabulary argmax (matmul.rs OpMulMatArgmaxQ4K / Q8_0) and the row gather
(get_rows.rs), bit-exact against the oracle on the same serialized bytes."""

import ctypes

import numpy as np
import pytest

import gguf_writer as gw
import oracle
from test_gpu_matvec import cview, nb_of, q4k_rows, q8_rows

pytestmark = pytest.mark.gpu
B = ctypes.byref


def argmax_both(emel, ctx, olib, img, name, suffix, code, bb, k, rows, rhs):
    buf, view = img.upload(ctx, name)
    t = img.record(name)
    rb = k // (256 if code in (10, 11, 12, 14) else 32) * bb
    assert list(view.ne) == [k, rows, 1, 1] and list(view.nb)[:2] == [1, rb] and view.dtype == code
    br, bd, bi = emel.DeviceBuffer(ctx, rhs.nbytes), emel.DeviceBuffer(ctx, 16), emel.DeviceBuffer(ctx, 16)
    br.upload(rhs)
    fn = getattr(emel.lib(), f"emel_cuda_mul_mat_argmax_{suffix}")
    st = fn(ctx.handle, None, B(view), B(cview(emel, br, rhs.nbytes, [1, k, 1, 1])), B(cview(emel, bd, 4, [1, 1, 1, 1])),
            ctypes.c_void_p(bi.ptr))
    assert st == 0, ctx.last_error
    assert emel.lib().emel_cuda_stream_synchronize(ctx.handle, None) == 0
    got_v = bd.download(np.empty(4, np.float32))[0]
    got_i = int(bi.download(np.empty(4, np.int32))[0])
    blob = np.frombuffer(img.image[t.file_offset:t.file_offset + t.data_size], np.uint8).copy()
    out = np.full(1, 9.0, np.float32)
    idx = ctypes.c_int32()
    ost = getattr(olib, f"oracle_mul_mat_argmax_{suffix}")(
        B(oracle.make_view(blob.ctypes.data, blob.nbytes, [k, rows, 1, 1], [1, rb, rb * rows, rb * rows], code)),
        B(oracle.make_view(rhs.ctypes.data, rhs.nbytes, [1, k, 1, 1], nb_of([1, k, 1, 1]), 0)),
        B(oracle.make_view(out.ctypes.data, out.nbytes, [1, 1, 1, 1], nb_of([1, 1, 1, 1]), 0)), B(idx))
    assert ost == 0
    for b in (buf, br, bd, bi):
        b.free()
    return got_i, np.float32(got_v), idx.value, out[0]


def test_gguf_model_tensors_drive_the_device_kernels(emel, oracle_lib):
    ctx = emel.Context(0)
    rng = np.random.default_rng(2718)
    k, vq4, vq8, emb_rows = 4096, 3000, 2000, 5000
    q4 = q4k_rows(rng, k, vq4, planted=1234)
    q8 = q8_rows(rng, k, vq8, planted=777)
    table = rng.standard_normal(256 * emb_rows).astype(np.float32)
    data = gw.image([(b"output_q4k.weight", [k, vq4], 12, q4.tobytes()),
                     (b"output_q8.weight", [k, vq8], 8, q8.tobytes()),
                     (b"token_embd.weight", [256, emb_rows], 0, table.tobytes())],
                    metadata=[(b"general.architecture", gw.GGUF_STRING, gw.string(b"synthetic"))], alignment=64)
    img = emel.GgufImage(data)
    assert img.requirements.tensor_count == 3 and img.requirements.kv_count == 2
    rhs = rng.standard_normal(k).astype(np.float32)
    gi, gv, oi, ov = argmax_both(emel, ctx, oracle_lib, img, "output_q4k.weight", "q4_k", 12, 144, k, vq4, rhs)
    assert gi == oi and gv.view(np.uint32) == ov.view(np.uint32)
    gi, gv, oi, ov = argmax_both(emel, ctx, oracle_lib, img, "output_q8.weight", "q8_0", 8, 34, k, vq8,
                                 np.abs(rhs))
    assert gi == oi and gv.view(np.uint32) == ov.view(np.uint32)

    # row gather from the uploaded embedding table
    buf, tview = img.upload(ctx, "token_embd.weight")
    tokens = rng.integers(0, emb_rows, 300).astype(np.int32)
    bi = emel.DeviceBuffer(ctx, tokens.nbytes)
    bi.upload(tokens)
    bd = emel.DeviceBuffer(ctx, 256 * 300 * 4)
    iv = emel.CView()
    iv.data, iv.storage_bytes, iv.dtype = bi.ptr, tokens.nbytes, 26
    for d, (n, s) in enumerate(zip([300, 1, 1, 1], [4, 1200, 1200, 1200])):
        iv.ne[d], iv.nb[d] = n, s
    dv = cview(emel, bd, 256 * 300 * 4, [256, 300, 1, 1])
    assert emel.lib().emel_cuda_get_rows(ctx.handle, None, B(tview), B(iv), B(dv)) == 0, ctx.last_error
    assert emel.lib().emel_cuda_stream_synchronize(ctx.handle, None) == 0
    got = bd.download(np.empty(256 * 300, np.float32))
    want = np.empty_like(got)
    ost = oracle_lib.oracle_get_rows(B(oracle.make_view(table.ctypes.data, table.nbytes, [256, emb_rows, 1, 1],
                                                        nb_of([256, emb_rows, 1, 1]), 0)),
                                     B(oracle.make_view(tokens.ctypes.data, tokens.nbytes, [300, 1, 1, 1],
                                                        [4, 1200, 1200, 1200], 26)),
                                     B(oracle.make_view(want.ctypes.data, want.nbytes, [256, 300, 1, 1],
                                                        nb_of([256, 300, 1, 1]), 0)))
    assert ost == 0
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    for b in (buf, bi, bd):
        b.free()
