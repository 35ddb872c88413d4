"""The single-query attention oracle (oracle_flash_attn_ext, restating
flash_attn.rs OpFlashAttnExt) on the reference's own evidence: the
kernel-flash-attn parity manifest (bit-exact output bits and the rejected
case), the known answers of tests/any/flash_attn_ops.rs, the binary16
helper's known answers (flash_attn.rs:483-525), and a float64 softmax
attention as a sanity bound on seeded inputs."""

import ctypes
import json
from pathlib import Path

import numpy as np
import pytest

import oracle

B = ctypes.byref
GOLDEN = Path(__file__).resolve().parent / "golden" / "flash_attn_parity.json"


@pytest.fixture(scope="module", params=[False, True], ids=["glibc", "cr"])
def lib(request):
    return oracle.load(cr=request.param)


def options(scale=None, masked=None):
    o = oracle.FlashAttnOptions()
    if scale is not None:
        o.scale, o.has_scale = scale, 1
    if masked is not None:
        o.masked_total_tokens, o.has_masked_total_tokens = masked, 1
    return o


def run_case(lib, c):
    q = np.array(c["query"], np.float32)
    k = np.array(c["key"], np.uint16)
    v = np.array(c["value"], np.uint16)
    dl = c["dst_layout"]
    n_out = max(1, int(np.prod(dl["ne"])))
    out = np.full(n_out, c["dst_fill"], np.float32)
    ql, kl, vl = c["query_layout"], c["key_layout"], c["value_layout"]
    st = lib.oracle_flash_attn_ext(B(oracle.make_view(q.ctypes.data, q.nbytes, ql["ne"], ql["nb"], 0)),
                                   B(oracle.make_view(k.ctypes.data, k.nbytes, kl["ne"], kl["nb"], 1)),
                                   B(oracle.make_view(v.ctypes.data, v.nbytes, vl["ne"], vl["nb"], 1)),
                                   B(oracle.make_view(out.ctypes.data, out.nbytes, dl["ne"], dl["nb"], 0)),
                                   B(options(c["scale"], c["masked_total_tokens"])))
    return st, out


def golden_cases():
    return json.loads(GOLDEN.read_text())["cases"]


@pytest.mark.parametrize("case", golden_cases(), ids=lambda c: c["case"])
def test_reference_evidence(lib, case):
    st, out = run_case(lib, case)
    if case["expect_status"] == "ok":
        assert st == oracle_ok()
        if case["compare"] == "exact":
            assert [int(b) for b in out.view(np.uint32)] == case["expect_bits"]
        else:
            assert np.all(np.abs(out - np.array(case["expect_values"], np.float32)) < case["tolerance"])
    else:
        assert st == 12  # FlashAttnError::InvalidRequest
        if case.get("expect_bits"):
            assert [int(b) for b in out.view(np.uint32)] == case["expect_bits"]
        else:
            assert out.tolist() == case["expect_values"]


def oracle_ok():
    return 0


def r16(lib, x):
    return np.float32(lib.oracle_fp16_to_fp32(lib.oracle_fa_f32_to_f16(x)))


def test_binary16_helper_known_answers(lib):
    # flash_attn.rs:488-492
    assert r16(lib, 1.0003) == np.float32(1.0)
    assert r16(lib, 1.0006) == np.float32(1.0009766)


def test_binary16_helper_rounding_rules(lib):
    f = lib.oracle_fa_f32_to_f16
    # normal range: IEEE round to nearest even
    rng = np.random.default_rng(3)
    xs = (rng.standard_normal(20000) * 300).astype(np.float32)
    for x in xs[:2000]:
        assert f(float(x)) == int(np.float16(x).view(np.uint16)), x
    # below 2^-24 flushes to a signed zero (IEEE would round (2^-25, 2^-24) up)
    assert f(float(np.float32(1.5 * 2.0 ** -25))) == 0
    assert f(float(np.float32(-1.5 * 2.0 ** -25))) == 0x8000
    # subnormal ties round half up (IEEE: to even): 2.5 * 2^-24 -> 3 units
    assert f(float(np.float32(2.5 * 2.0 ** -24))) == 3
    # overflow and NaN
    assert f(65520.0) == 0x7C00 and f(float("inf")) == 0x7C00
    assert f(float("nan")) == 0x7E00 and f(float(-np.float32("nan"))) == 0xFE00


def attention_f64(q, k, v, heads, kv_heads, d, t, scale):
    rep = heads // kv_heads
    out = np.zeros((heads, d))
    for h in range(heads):
        kh = k[h // rep].astype(np.float64)
        vh = v[h // rep].astype(np.float64)
        s = kh @ q[h].astype(np.float16).astype(np.float64) * scale
        w = np.exp(s - s.max())
        out[h] = (w / w.sum()) @ vh
    return out


def test_seeded_gqa_case_is_close_to_exact_attention(lib):
    rng = np.random.default_rng(11)
    heads, kv_heads, d, t = 4, 2, 64, 300
    q = rng.standard_normal((heads, d)).astype(np.float32)
    k = rng.standard_normal((kv_heads, t, d)).astype(np.float16)
    v = rng.standard_normal((kv_heads, t, d)).astype(np.float16)
    out = np.zeros((heads, d), np.float32)
    kl = [d, t, kv_heads, 1]
    st = lib.oracle_flash_attn_ext(
        B(oracle.make_view(q.ctypes.data, q.nbytes, [d, 1, heads, 1], [4, 4 * d, 4 * d, 4 * d * heads], 0)),
        B(oracle.make_view(k.ctypes.data, k.nbytes, kl, [2, 2 * d, 2 * d * t, 2 * d * t * kv_heads], 1)),
        B(oracle.make_view(v.ctypes.data, v.nbytes, kl, [2, 2 * d, 2 * d * t, 2 * d * t * kv_heads], 1)),
        B(oracle.make_view(out.ctypes.data, out.nbytes, [d, 1, heads, 1], [4, 4 * d, 4 * d, 4 * d * heads], 0)),
        B(options()))
    assert st == 0
    want = attention_f64(q, k, v, heads, kv_heads, d, t, 1.0 / np.sqrt(d))
    # the binary16 running accumulator drifts by a few binary16 steps over 300 tokens
    assert np.max(np.abs(out - want)) < 2e-2


def test_guards(lib):
    q = np.zeros(4, np.float32)
    k = np.zeros(8, np.uint16)
    out = np.full(4, 9.0, np.float32)
    qv = oracle.make_view(q.ctypes.data, q.nbytes, [2, 1, 2, 1], [4, 8, 8, 16], 0)
    ov = oracle.make_view(out.ctypes.data, out.nbytes, [2, 1, 2, 1], [4, 8, 8, 16], 0)

    def call(kne, knb, vne=None, vnb=None, opts=None, qview=qv, kdtype=1):
        kv = oracle.make_view(k.ctypes.data, k.nbytes, kne, knb, kdtype)
        vv = oracle.make_view(k.ctypes.data, k.nbytes, vne or kne, vnb or knb, 1)
        return lib.oracle_flash_attn_ext(B(qview), B(kv), B(vv), B(ov), B(opts or options()))

    assert call([2, 2, 1, 1], [2, 4, 8, 8]) == 0
    out[:] = 9.0
    assert call([2, 2, 1, 1], [4, 8, 16, 16], kdtype=0) == 12          # F32 key
    assert call([2, 2, 3, 1], [2, 4, 8, 24]) == 12                     # 2 heads not a multiple of 3 kv heads
    assert call([2, 2, 1, 1], [2, 4, 8, 8], opts=options(masked=1)) == 12   # masked total below the token count
    assert call([2, 2, 1, 1], [2, 4, 8, 8], opts=options(scale=float("inf"))) == 12
    assert call([2, 2, 1, 1], [2, 4, 8, 8], opts=options(scale=-1.0)) == 12
    assert call([3, 2, 1, 1], [2, 6, 12, 12]) == 12                     # key head_dim differs
    assert call([2, 2, 1, 1], [2, 4, 8, 8], vne=[2, 1, 1, 1], vnb=[2, 4, 4, 4]) == 12
    assert call([2, 5, 1, 1], [2, 4, 20, 20]) == 12                     # key span beyond its storage
    strided_q = oracle.make_view(q.ctypes.data, q.nbytes, [2, 1, 1, 1], [8, 16, 16, 16], 0)
    assert call([2, 2, 1, 1], [2, 4, 8, 8], qview=strided_q) == 12      # query not dense
    assert out.tolist() == [9.0] * 4
