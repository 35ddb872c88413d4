"""emel_cuda_flash_attn_ext (flash_attn.rs OpFlashAttnExt on the device)
against the oracle, through the C ABI.

The reference's exp is a libm call; the device evaluates it in binary64 and
rounds once, as the oracle's correctly rounded build does, so the two agree
bit for bit except where a binary64 double rounding lands on the other side
of a binary32 midpoint (about one exp in 10^7).  Such a miss moves one
per-token factor by an ulp and can move that head's binary16 accumulator by
one step.  Bar against the correctly rounded oracle: at least 99 % of heads
bit-identical, every element within two binary16 steps of the head's
largest magnitude, NaN positions identical.  Against the glibc oracle (the
reference's own libm) the same bound.  The reference's golden vectors
(kernel-flash-attn manifest) are bit-exact."""

import ctypes
import json
from pathlib import Path

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu
B = ctypes.byref
GOLDEN = Path(__file__).resolve().parent / "golden" / "flash_attn_parity.json"


@pytest.fixture(scope="module")
def kern(emel):
    return emel.Kernel(device=0, synchronize=True)


@pytest.fixture(scope="module")
def cr_lib():
    return oracle.load(cr=True)


class Dev:
    def __init__(self, emel, ctx, host, ne, nb, code):
        self.emel, self.host, self.ne, self.nb, self.code = emel, np.ascontiguousarray(host), list(ne), list(nb), code
        self.buf = emel.DeviceBuffer(ctx, max(self.host.nbytes, 16))
        self.buf.upload(self.host)

    def c(self):
        v = self.emel.CView()
        v.data, v.storage_bytes, v.dtype = self.buf.ptr, self.host.nbytes, self.code
        for d in range(4):
            v.ne[d], v.nb[d] = self.ne[d], self.nb[d]
        return v

    def o(self, arr=None):
        a = self.host if arr is None else arr
        return oracle.make_view(a.ctypes.data, a.nbytes, self.ne, self.nb, self.code)


def opts(scale, masked):
    o = oracle.FlashAttnOptions()
    if scale is not None:
        o.scale, o.has_scale = scale, 1
    if masked is not None:
        o.masked_total_tokens, o.has_masked_total_tokens = masked, 1
    return o


def run(emel, kern, olib, q, k, v, qne, qnb, kne, knb, vne, vnb, dne, dnb, scale=None, masked=None, fill=9.0):
    ctx = kern.ctx
    dq = Dev(emel, ctx, np.asarray(q, np.float32), qne, qnb, 0)
    dk = Dev(emel, ctx, np.asarray(k, np.uint16), kne, knb, 1)
    dv = Dev(emel, ctx, np.asarray(v, np.uint16), vne, vnb, 1)
    n_out = max(1, int(np.prod(dne)))
    dd = Dev(emel, ctx, np.full(n_out, fill, np.float32), dne, dnb, 0)
    st = kern.process_event(emel.OpFlashAttnExt(dq.c(), dk.c(), dv.c(), dd.c(), scale, masked))
    got = dd.buf.download(np.empty_like(dd.host))
    want = dd.host.copy()
    ost = olib.oracle_flash_attn_ext(B(dq.o()), B(dk.o()), B(dv.o()), B(dd.o(want)), B(opts(scale, masked)))
    for x in (dq, dk, dv, dd):
        x.buf.free()
    return int(st), ost, got, want


def nb_of(ne, size):
    nb = [size]
    for d in range(1, 4):
        nb.append(nb[-1] * ne[d - 1])
    return nb


def agree(got, want, d, heads, min_identical=0.99):
    assert np.array_equal(np.isnan(got), np.isnan(want))
    g = got.reshape(heads, d)
    w = want.reshape(heads, d)
    same_heads = 0
    for h in range(heads):
        gb, wb = g[h].view(np.uint32), w[h].view(np.uint32)
        ok = np.isnan(w[h]) | (gb == wb)
        if ok.all():
            same_heads += 1
            continue
        fin = np.isfinite(w[h])
        mag = float(np.max(np.abs(w[h][fin]))) if fin.any() else 0.0
        assert np.array_equal(np.isinf(g[h]), np.isinf(w[h]))
        assert np.max(np.abs(g[h][fin] - w[h][fin])) <= 2.0 * 2.0 ** -10 * max(mag, 1e-30), h
    assert same_heads >= min_identical * heads, (same_heads, heads)


def golden_cases():
    return json.loads(GOLDEN.read_text())["cases"]


@pytest.mark.parametrize("case", golden_cases(), ids=lambda c: c["case"])
def test_reference_golden_vectors(emel, kern, case):
    ql, kl, vl, dl = case["query_layout"], case["key_layout"], case["value_layout"], case["dst_layout"]
    ctx = kern.ctx
    dq = Dev(emel, ctx, np.array(case["query"], np.float32), ql["ne"], ql["nb"], 0)
    dk = Dev(emel, ctx, np.array(case["key"], np.uint16), kl["ne"], kl["nb"], 1)
    dv = Dev(emel, ctx, np.array(case["value"], np.uint16), vl["ne"], vl["nb"], 1)
    n_out = max(1, int(np.prod(dl["ne"])))
    dd = Dev(emel, ctx, np.full(n_out, case["dst_fill"], np.float32), dl["ne"], dl["nb"], 0)
    st = kern.process_event(emel.OpFlashAttnExt(dq.c(), dk.c(), dv.c(), dd.c(), case["scale"],
                                                case["masked_total_tokens"]))
    out = dd.buf.download(np.empty_like(dd.host))
    for x in (dq, dk, dv, dd):
        x.buf.free()
    if case["expect_status"] == "ok":
        assert st == emel.Status.OK
        if case["compare"] == "exact":
            assert [int(b) for b in out.view(np.uint32)] == case["expect_bits"]
        else:
            assert np.all(np.abs(out - np.array(case["expect_values"], np.float32)) < case["tolerance"])
    else:
        assert st == emel.Status.INVALID_REQUEST
        want = case.get("expect_bits") or [int(b) for b in np.array(case["expect_values"], np.float32).view(np.uint32)]
        assert [int(b) for b in out.view(np.uint32)] == want


def gqa_inputs(rng, d, t, heads, kvh, kv_std=1.0):
    q = rng.standard_normal(heads * d).astype(np.float32)
    k = (rng.standard_normal(kvh * t * d) * kv_std).astype(np.float16).view(np.uint16)
    v = (rng.standard_normal(kvh * t * d) * kv_std).astype(np.float16).view(np.uint16)
    return q, k, v


SHAPES = [
    # d, tokens, heads, kv_heads, scale, masked
    (128, 4096, 32, 8, None, None),   # a decode step of an 8-kv-head, 32-head model at 4096 tokens
    (64, 257, 4, 4, None, None),
    (128, 1, 2, 1, None, 1),
    (4, 300, 3, 1, 0.7, 305),         # rows too short for vector loads
    (3, 33, 2, 2, None, None),
    (1, 10, 1, 1, 1.0, None),
    (256, 600, 2, 2, None, None),
    (320, 300, 2, 1, None, None),     # two columns per thread
    (768, 100, 2, 2, None, None),     # four columns per thread
    (2048, 40, 2, 1, None, None),     # eight columns per thread
    (4096, 9, 1, 1, None, None),      # the largest head_dim
    (64, 512, 2, 1, 2.5, None),       # wide score spread: binary16 subnormal value factors
]


@pytest.mark.parametrize("d,t,heads,kvh,scale,masked", SHAPES)
def test_parity_contiguous(emel, kern, cr_lib, oracle_lib, d, t, heads, kvh, scale, masked):
    rng = np.random.default_rng(d * 7919 + t)
    q, k, v = gqa_inputs(rng, d, t, heads, kvh)
    qne, kne = [d, 1, heads, 1], [d, t, kvh, 1]
    args = (q, k, v, qne, nb_of(qne, 4), kne, nb_of(kne, 2), kne, nb_of(kne, 2), qne, nb_of(qne, 4), scale, masked)
    st, ost, got, want = run(emel, kern, cr_lib, *args)
    assert st == 0 and ost == 0
    agree(got, want, d, heads)
    _, _, _, want_glibc = run(emel, kern, oracle_lib, *args)
    agree(got, want_glibc, d, heads, min_identical=0.5)


def test_parity_strided_layouts(emel, kern, cr_lib):
    rng = np.random.default_rng(5)
    d, t, heads, kvh = 64, 200, 4, 2
    q = rng.standard_normal(heads * d).astype(np.float32)
    # key stored token-major across kv heads: [t][kvh][d] (rows unit-stride, head interleaved)
    k = rng.standard_normal(t * kvh * d).astype(np.float16).view(np.uint16)
    knb = [2, 2 * d * kvh, 2 * d, 2 * d * kvh * t]
    # value stored transposed per kv head: [kvh][d][t] (column-major rows)
    v = rng.standard_normal(kvh * d * t).astype(np.float16).view(np.uint16)
    vnb = [2 * t, 2, 2 * t * d, 2 * t * d * kvh]
    qne, kne = [d, 1, heads, 1], [d, t, kvh, 1]
    st, ost, got, want = run(emel, kern, cr_lib, q, k, v, qne, nb_of(qne, 4), kne, knb, kne, vnb, qne,
                             nb_of(qne, 4))
    assert st == 0 and ost == 0
    agree(got, want, d, heads)
    # the same with a transposed key (no vector path) and implicit query / destination strides
    kt = rng.standard_normal(kvh * d * t).astype(np.float16).view(np.uint16)
    st, ost, got, want = run(emel, kern, cr_lib, q, kt, v, qne, [0, 0, 0, 0], kne, vnb, kne, vnb, qne, [0, 0, 0, 0])
    assert st == 0 and ost == 0
    agree(got, want, d, heads)


def test_special_values(emel, kern, cr_lib):
    rng = np.random.default_rng(9)
    d, t, heads, kvh = 16, 70, 6, 1
    qne, kne = [d, 1, heads, 1], [d, t, kvh, 1]
    q, k, v = gqa_inputs(rng, d, t, heads, kvh)
    q[1 * d + 3] = np.inf           # head 1: infinite scores
    q[2 * d + 0] = np.nan           # head 2: NaN scores
    q[3 * d + 5] = 1e9              # head 3: query beyond binary16 (rounds to inf)
    k16 = k.view(np.float16).copy()
    k16[7 * d + 2] = np.float16(np.nan)  # token 7: NaN score for every head
    v16 = v.view(np.float16).copy()
    v16[11 * d + 4] = np.float16(np.inf)  # token 11, column 4: infinite value
    args = (q, k16.view(np.uint16), v16.view(np.uint16), qne, nb_of(qne, 4), kne, nb_of(kne, 2), kne,
            nb_of(kne, 2), qne, nb_of(qne, 4))
    st, ost, got, want = run(emel, kern, cr_lib, *args)
    assert st == 0 and ost == 0
    assert np.isnan(want).any()
    agree(got, want, d, heads, min_identical=1.0)
    # tiny values: binary16 subnormal accumulators (the reference's own rounding there)
    v_small = (rng.standard_normal(t * d) * 3e-6).astype(np.float16).view(np.uint16)
    q_ok, k_ok, _ = gqa_inputs(rng, d, t, heads, kvh)
    st, ost, got, want = run(emel, kern, cr_lib, q_ok, k_ok, v_small, qne, nb_of(qne, 4), kne, nb_of(kne, 2), kne,
                             nb_of(kne, 2), qne, nb_of(qne, 4))
    assert st == 0 and ost == 0
    agree(got, want, d, heads, min_identical=1.0)
    # huge scale: scores overflow to inf
    st, ost, got, want = run(emel, kern, cr_lib, q_ok, k_ok, v_small, qne, nb_of(qne, 4), kne, nb_of(kne, 2), kne,
                             nb_of(kne, 2), qne, nb_of(qne, 4), scale=1e38)
    assert st == 0 and ost == 0
    agree(got, want, d, heads, min_identical=1.0)


def test_rejections_write_nothing_and_workspace_counts(emel, kern, cr_lib):
    rng = np.random.default_rng(2)
    d, t, heads, kvh = 8, 5, 2, 1
    q, k, v = gqa_inputs(rng, d, t, heads, kvh)
    qne, kne = [d, 1, heads, 1], [d, t, kvh, 1]
    base = (q, k, v, qne, nb_of(qne, 4), kne, nb_of(kne, 2), kne, nb_of(kne, 2), qne, nb_of(qne, 4))
    for scale, masked in ((0.0, None), (float("nan"), None), (None, t - 1)):
        st, ost, got, _ = run(emel, kern, cr_lib, *base, scale=scale, masked=masked)
        assert st == emel.Status.INVALID_REQUEST and ost == 12
        assert np.all(got == 9.0)
    # FlashAttnKernel::prepared_tokens / reuse_count (flash_attn_ops.rs:87-118)
    ctx = emel.Context(0)
    k2 = emel.Kernel(ctx=ctx, synchronize=True)
    assert emel.flash_attn_workspace(ctx) == (0, 0)
    for n in range(2):
        run(emel, k2, cr_lib, *base)
    assert emel.flash_attn_workspace(ctx) == (t, 1)
    run(emel, k2, cr_lib, *base, scale=0.0)  # rejected: no change
    assert emel.flash_attn_workspace(ctx) == (t, 1)
    ctx.close()
