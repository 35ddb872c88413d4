"""emel_cuda_cpy / emel_cuda_cont (shape.rs OpCpy / OpCont on the device)
against the oracle: bit-exact, NaN payloads included, on strided, permuted,
reshaped and implicit-stride views; rejected requests write nothing."""

import ctypes

import numpy as np
import pytest

import gpu_helpers as gh
import oracle

pytestmark = pytest.mark.gpu
B = ctypes.byref


@pytest.fixture(scope="module")
def kern(emel):
    return emel.Kernel(device=0, synchronize=True)


def run(emel, kern, olib, kind, src_host, src_ne, src_nb, dst_n, dst_ne, dst_nb, fill=7.0):
    ctx = kern.ctx
    ps = gh.Pair(emel, ctx, src_host, src_ne, src_nb)
    pd = gh.Pair(emel, ctx, np.full(dst_n, fill, np.float32), dst_ne, dst_nb)
    ev = (emel.OpCpy if kind == "cpy" else emel.OpCont)(ps.dview(), pd.dview())
    st = kern.process_event(ev)
    got = pd.download()
    want = pd.host.copy()
    fn = olib.oracle_cpy if kind == "cpy" else olib.oracle_cont
    ost = fn(B(ps.oview()), B(oracle.make_view(want.ctypes.data, want.nbytes, pd.ne, pd.nb, 0)))
    ps.free()
    pd.free()
    return int(st), ost, got, want


def test_reference_shape_test_on_the_device(emel, kern, oracle_lib):
    source = np.array([1, 99, 2, 99, 3, 99, 4], np.float32)
    st, ost, got, _ = run(emel, kern, oracle_lib, "cpy", source, [2, 2, 1, 1], [8, 16, 32, 64], 7, [2, 2, 1, 1],
                          [8, 16, 32, 64], fill=0.0)
    assert st == ost == 0 and got.tolist() == [1, 0, 2, 0, 3, 0, 4]
    st, ost, got, _ = run(emel, kern, oracle_lib, "cont", source, [2, 2, 1, 1], [8, 16, 32, 64], 4, [2, 2, 1, 1],
                          [4, 8, 16, 16], fill=0.0)
    assert st == ost == 0 and got.tolist() == [1, 2, 3, 4]


@pytest.mark.parametrize("kind,dst_ne,dst_nb,status", [
    ("cont", [2, 2, 1, 1], [8, 16, 32, 64], 8),       # strided destination: InvalidLayout
    ("cont", [4, 1, 1, 1], [0, 0, 0, 0], 8),          # implicit strides are not dense for OpCont
    ("cpy", [3, 1, 1, 1], [4, 12, 12, 12], 2),        # count mismatch
    ("cont", [3, 1, 1, 1], [4, 12, 12, 12], 2),
])
def test_rejections_write_nothing(emel, kern, oracle_lib, kind, dst_ne, dst_nb, status):
    src = np.array([1, 2, 3, 4], np.float32)
    n = sum((dst_ne[d] - 1) * dst_nb[d] for d in range(4)) // 4 + 1 if dst_nb[0] else int(np.prod(dst_ne))
    st, ost, got, want = run(emel, kern, oracle_lib, kind, src, [2, 2, 1, 1], [4, 8, 16, 16], n, dst_ne, dst_nb)
    assert st == ost == status
    assert np.all(got == 7.0)


def permuted_case(rng, ne, perm):
    """Storage dense in the permuted order; the view reads it in logical order."""
    store_ne = [ne[p] for p in perm]
    store_nb = gh.contiguous_nb(store_ne, 4)
    nb = [0] * 4
    for k, p in enumerate(perm):
        nb[p] = store_nb[k]
    host = rng.standard_normal(int(np.prod(ne))).astype(np.float32)
    host[:4] = np.array([0x7fa00001, 0xffc00002, 0x7f800000, 0x80000000], np.uint32).view(np.float32)
    return host, nb


@pytest.mark.parametrize("ne,perm", [([64, 33, 5, 3], [1, 0, 2, 3]), ([128, 32, 64, 2], [0, 2, 1, 3]),
                                     ([7, 5, 3, 2], [3, 2, 1, 0]), ([128, 32, 2048, 2], [0, 2, 1, 3])])
def test_cont_of_permuted_views(emel, kern, oracle_lib, ne, perm):
    rng = np.random.default_rng(sum(ne))
    host, nb = permuted_case(rng, ne, perm)
    n = int(np.prod(ne))
    st, ost, got, want = run(emel, kern, oracle_lib, "cont", host, ne, nb, n, ne, gh.contiguous_nb(ne, 4))
    assert st == ost == 0
    gh.assert_bits_equal(got, want, f"cont {ne} perm {perm}")


def test_cpy_reshaped_into_strided_destination(emel, kern, oracle_lib):
    """Count-equal copy: [40, 30, 2] source, [60, 40] destination that
    writes every other float."""
    rng = np.random.default_rng(5)
    host = rng.standard_normal(2400).astype(np.float32)
    host[7] = np.uint32(0x7f800001).view(np.float32)
    dst_ne, dst_nb = [60, 40, 1, 1], [8, 480, 19200, 19200]
    n = 2 * 2400
    st, ost, got, want = run(emel, kern, oracle_lib, "cpy", host, [40, 30, 2, 1], gh.contiguous_nb([40, 30, 2, 1], 4),
                             n, dst_ne, dst_nb)
    assert st == ost == 0
    gh.assert_bits_equal(got, want, "cpy reshaped strided")
