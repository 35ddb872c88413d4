"""Seeded synthetic inputs for the five benchmark configurations.

No public dataset exists for this path; each configuration is generated
from a fixed seed with the shapes, value distributions and special values
its description names.  "N(0, v)" is read as a normal distribution with
variance v.  Arrays are numpy, in ggml order: numpy shape = ne reversed.

Algorithmic bytes per op count every input element read once and every
output element written once (the HBM roofline's numerator).
"""

import math
from dataclasses import dataclass, field
from typing import Dict, List

import numpy as np

F32, F16 = 4, 2


def normal(rng, shape, variance=1.0):
    x = rng.standard_normal(size=shape, dtype=np.float32)
    if variance != 1.0:
        x *= np.float32(math.sqrt(variance))
    return x


@dataclass
class OpSpec:
    name: str
    bytes: int        # algorithmic bytes per launch
    elements: int     # logical elements processed per launch


@dataclass
class Config:
    name: str
    ops: List[OpSpec] = field(default_factory=list)


# ---- config 1: row-broadcast binary ops ------------------------------------
CFG1_NE = (4096, 2048)


def cfg1(seed=1):
    rng = np.random.default_rng(seed)
    src0 = normal(rng, (CFG1_NE[1], CFG1_NE[0]))
    src1 = rng.uniform(0.5, 1.5, size=CFG1_NE[0]).astype(np.float32)
    return src0, src1


def cfg1_spec():
    n = CFG1_NE[0] * CFG1_NE[1]
    b = 2 * n * F32 + CFG1_NE[0] * F32
    return Config("cfg1", [OpSpec(f"broadcast_row_{op}", b, n) for op in ("add", "sub", "mul", "div")])


# ---- config 2: unary / activation sweep -------------------------------------
CFG2_NE = (14336, 512)
CFG2_OPS = ("silu", "gelu", "relu", "exp", "neg", "sqr", "sqrt", "pow2")


def cfg2(seed=2):
    """x ~ N(0, 2) clamped to [-10, 10]; sqrt and pow take |x| + 1e-3."""
    rng = np.random.default_rng(seed)
    x = np.clip(normal(rng, (CFG2_NE[1], CFG2_NE[0]), 2.0), -10.0, 10.0).astype(np.float32)
    xa = (np.abs(x) + np.float32(1e-3)).astype(np.float32)
    return x, xa


def cfg2_spec():
    n = CFG2_NE[0] * CFG2_NE[1]
    ops = [OpSpec(f"{op}_f32", 2 * n * F32, n) for op in CFG2_OPS]
    ops += [OpSpec(f"{op}_f16", 2 * n * F16, n) for op in CFG2_OPS]
    return Config("cfg2", ops)


# ---- config 3: row normalisation -------------------------------------------
CFG3_NE = (4096, 8192)


def cfg3(seed=3):
    """x ~ N(0, 1) with 1% of entries (a seeded index set) scaled by 20;
    weight ~ U(0.5, 1.5) over ne0."""
    rng = np.random.default_rng(seed)
    n = CFG3_NE[0] * CFG3_NE[1]
    x = normal(rng, n)
    idx = rng.choice(n, size=n // 100, replace=False)
    x[idx] *= np.float32(20.0)
    w = rng.uniform(0.5, 1.5, size=CFG3_NE[0]).astype(np.float32)
    return x.reshape(CFG3_NE[1], CFG3_NE[0]), w


def cfg3_spec():
    n = CFG3_NE[0] * CFG3_NE[1]
    rows = CFG3_NE[1]
    return Config("cfg3", [
        OpSpec("rms_norm", 2 * n * F32, n),
        OpSpec("rms_norm_mul", 2 * n * F32 + CFG3_NE[0] * F32, n),
        OpSpec("norm", 2 * n * F32, n),
        OpSpec("sum_rows", n * F32 + rows * F32, n),
    ])


# ---- config 4: softmax and argmax -------------------------------------------
CFG4A_NE = (4096, 512, 32)   # kv, q, heads
CFG4A_SCALE = np.float32(1.0 / math.sqrt(128.0))
CFG4A_QOFF = 3584
CFG4B_NE = (151936, 64)


def cfg4a(seed=4):
    """scores ~ N(0, 4); f16 causal mask: 0 where kv <= q + 3584, else -inf."""
    rng = np.random.default_rng(seed)
    kv, q, h = CFG4A_NE
    scores = normal(rng, (h, q, kv), 4.0)
    kvi = np.arange(kv)[None, :]
    qi = np.arange(q)[:, None]
    mask = np.where(kvi <= qi + CFG4A_QOFF, 0.0, -np.inf).astype(np.float16)
    return scores, mask


def cfg4b(seed=5):
    """logits ~ N(0, 3) with one planted maximum per row (seeded column)."""
    rng = np.random.default_rng(seed)
    v, rows = CFG4B_NE
    logits = normal(rng, (rows, v), 3.0)
    cols = rng.integers(0, v, size=rows)
    logits[np.arange(rows), cols] = logits.max(axis=1) + np.float32(1.0)
    return logits, cols


def cfg4_spec():
    kv, q, h = CFG4A_NE
    na = kv * q * h
    v, rows = CFG4B_NE
    nb = v * rows
    return Config("cfg4", [
        OpSpec("soft_max_ext", 2 * na * F32 + kv * q * F16, na),
        OpSpec("soft_max_vocab", 2 * nb * F32, nb),
        OpSpec("argmax_rows", nb * F32 + rows * 8, nb),
    ])


# ---- config 5: permuted 4-D broadcast, sharded along dim 3 -----------------
CFG5_NE = (128, 32, 8192, 8)  # logical view of src0


def cfg5_src0_view(ne3=CFG5_NE[3]):
    """ne/nb (bytes) of src0: contiguous storage [128, 8192, 32, ne3] viewed
    with dimensions 1 and 2 swapped."""
    ne0, ne1, ne2, _ = CFG5_NE
    storage_nb = [F32, F32 * ne0, F32 * ne0 * ne2, F32 * ne0 * ne2 * ne1]
    return [ne0, ne1, ne2, ne3], [storage_nb[0], storage_nb[2], storage_nb[1], storage_nb[3]]


def cfg5(seed=6, ne3=CFG5_NE[3], shard=0):
    """src0 storage (numpy shape (ne3, 32, 8192, 128)) ~ N(0, 1) and src1
    (shape (1, 8192, 1, 128)) ~ N(0, 1).  A shard holds the dim-3 slices
    [shard * ne3, (shard + 1) * ne3) of the full tensor; every shard draws
    its own slices from a per-slice seed so any sharding yields the same
    global tensor."""
    ne0, ne1, ne2, _ = CFG5_NE
    src0 = np.empty((ne3, ne1, ne2, ne0), dtype=np.float32)
    for k in range(ne3):
        rng = np.random.default_rng([seed, shard * ne3 + k])
        src0[k] = normal(rng, (ne1, ne2, ne0))
    src1 = normal(np.random.default_rng([seed, 1 << 20]), (1, ne2, 1, ne0))
    return src0, src1


def cfg5_spec(ne3=CFG5_NE[3]):
    ne0, ne1, ne2, _ = CFG5_NE
    n = ne0 * ne1 * ne2 * ne3
    b1 = ne0 * ne2 * F32
    return Config("cfg5", [
        OpSpec("repeat_mul", 2 * n * F32 + b1, n),
        OpSpec("repeat_add", 2 * n * F32 + b1, n),
        OpSpec("sum", n * F32, n),
        OpSpec("argmax", n * F32, n),
    ])


SPECS: Dict[str, callable] = {"cfg1": cfg1_spec, "cfg2": cfg2_spec, "cfg3": cfg3_spec, "cfg4": cfg4_spec,
                              "cfg5": cfg5_spec}


# Gated linear units (glu.rs) -- no configuration in the benchmark set names
# them; the bench suite uses the feed-forward gate of configuration 2's shape:
# value and gate halves of [14336, 512] each, value ~ N(0, 1), gate ~ N(0, 2).
GLU_N = CFG2_NE[0] * CFG2_NE[1]
GLU_OPS = ("reglu", "geglu", "swiglu", "swiglu_oai", "geglu_erf", "geglu_quick")


def glu_ffn(seed=7):
    rng = np.random.default_rng(seed)
    values = normal(rng, (GLU_N,), 1.0).astype(np.float32)
    gates = normal(rng, (GLU_N,), 2.0).astype(np.float32)
    return np.concatenate([values, gates])


def glu_spec():
    # read 2n floats, write n
    return Config("glu", [OpSpec(op, 3 * GLU_N * F32, GLU_N) for op in GLU_OPS])


# Row gather (get_rows.rs) -- no configuration in the benchmark set names it;
# the bench suite gathers 8192 token rows from a [4096, 32000] embedding
# table stored as F32, F16, BF16, Q8_0, Q4_0 and Q4_K (random block bytes
# with binary16 scales in [2^-7, 1)), plus the byte-backed F32 table of
# OpGetRowsF32Bytes with a row stride of 4 * 4096 + 1 bytes, so successive
# rows start at every byte offset modulo 4.
EMB_COLS, EMB_ROWS, EMB_TOKENS = 4096, 32000, 8192
EMB_BYTES_STRIDE = 4 * EMB_COLS + 1
EMB_FORMATS = {"f32": (0, 4, 1, 4), "f32_bytes": (0, 4, 1, 4), "f16": (1, 2, 1, 2), "bf16": (30, 2, 1, 2),
               "q8_0": (8, 34, 32, 0), "q4_0": (2, 18, 32, 0), "q4_k": (12, 144, 256, 0)}


def emb_row_bytes(fmt):
    code, unit, per, _ = EMB_FORMATS[fmt]
    return EMB_COLS // per * unit


def emb_table(fmt, seed=11):
    """Host bytes of the table in `fmt` (uint8 array) and its (ne, nb)."""
    code, unit, per, elem = EMB_FORMATS[fmt]
    rng = np.random.default_rng(seed)
    row_bytes = emb_row_bytes(fmt)
    if fmt == "f32":
        data = rng.standard_normal(EMB_COLS * EMB_ROWS).astype(np.float32).view(np.uint8)
    elif fmt == "f32_bytes":
        rows = rng.standard_normal(EMB_COLS * EMB_ROWS).astype(np.float32).view(np.uint8).reshape(EMB_ROWS, -1)
        data = np.zeros((EMB_ROWS, EMB_BYTES_STRIDE), np.uint8)
        data[:, :row_bytes] = rows
        data = data.reshape(-1)
        ne = [EMB_COLS, EMB_ROWS, 1, 1]
        return data, ne, [4, EMB_BYTES_STRIDE, EMB_BYTES_STRIDE * EMB_ROWS, EMB_BYTES_STRIDE * EMB_ROWS], code
    elif fmt in ("f16", "bf16"):
        x = rng.standard_normal(EMB_COLS * EMB_ROWS).astype(np.float32)
        h = x.astype(np.float16).view(np.uint16) if fmt == "f16" else (x.view(np.uint32) >> 16).astype(np.uint16)
        data = h.view(np.uint8)
    else:
        data = rng.integers(0, 256, size=row_bytes * EMB_ROWS, dtype=np.uint32).astype(np.uint8)
        blocks = data.reshape(-1, unit)
        scales = rng.integers(0x2000, 0x3c00, size=blocks.shape[0])
        blocks[:, 0] = scales & 0xff
        blocks[:, 1] = scales >> 8
        if fmt == "q4_k":
            mins = rng.integers(0x2000, 0x3c00, size=blocks.shape[0])
            blocks[:, 2] = mins & 0xff
            blocks[:, 3] = mins >> 8
    ne = [EMB_COLS, EMB_ROWS, 1, 1]
    nb = [elem if elem else 1, row_bytes, row_bytes * EMB_ROWS, row_bytes * EMB_ROWS]
    return data, ne, nb, code


def emb_tokens(seed=12):
    return np.random.default_rng(seed).integers(0, EMB_ROWS, size=EMB_TOKENS).astype(np.int32)


def emb_spec():
    # rows read + rows written + the indices
    return Config("get_rows", [OpSpec(f"get_rows_{fmt}", EMB_TOKENS * (emb_row_bytes(fmt) + EMB_COLS * F32 + 4),
                                      EMB_TOKENS * EMB_COLS) for fmt in EMB_FORMATS])


# Rotary position embedding (rope.rs) -- no configuration in the benchmark
# set names it; the suite rotates query rows [128 dims, 32 heads, 4096
# positions] (N(0, 1) values, positions 0 .. 4095) in neox and norm modes.
ROPE_NE = (128, 32, 4096, 1)


def rope_inputs(seed=13):
    rng = np.random.default_rng(seed)
    x = normal(rng, (int(np.prod(ROPE_NE)),), 1.0).astype(np.float32)
    return x, np.arange(ROPE_NE[2], dtype=np.int32)


def rope_spec():
    n = int(np.prod(ROPE_NE))
    return Config("rope", [OpSpec(f"rope_{m}", 2 * n * F32 + ROPE_NE[2] * 4, n) for m in ("neox", "norm")])


# Vocabulary matvec + argmax (matmul.rs OpMulMatArgmax, F32): the next-token
# step after the last hidden state -- lhs [4096, 151936] N(0, 1) / 64 (the
# vocabulary of configuration 4b), rhs [1, 4096] N(0, 1).
MV_K, MV_ROWS = 4096, 151936


def mv_inputs(seed=14):
    rng = np.random.default_rng(seed)
    lhs = (normal(rng, (MV_ROWS * MV_K,), 1.0) / 64.0).astype(np.float32)
    rhs = normal(rng, (MV_K,), 1.0).astype(np.float32)
    return lhs, rhs


def mv_spec():
    return Config("matvec", [OpSpec("mul_mat_argmax_vocab", (MV_K * MV_ROWS + MV_K) * F32 + 8, MV_K * MV_ROWS)])



# Single-query attention (flash_attn.rs OpFlashAttnExt): one decode step of a
# model with 32 query heads, 8 key/value heads and head_dim 128 (the head
# shape of configuration 4a) over 4096 and 32768 cached tokens; query
# N(0, 1) in binary32, key / value N(0, 1) in binary16.  Algorithmic bytes:
# query and output once, every key / value element once.
FA_D, FA_HEADS, FA_KV_HEADS = 128, 32, 8
FA_TOKENS = (4096, 32768)


def fa_inputs(tokens, seed=15):
    rng = np.random.default_rng(seed + tokens)
    q = normal(rng, (FA_HEADS * FA_D,))
    k = normal(rng, (FA_KV_HEADS * tokens * FA_D,)).astype(np.float16)
    v = normal(rng, (FA_KV_HEADS * tokens * FA_D,)).astype(np.float16)
    return q, k, v


def fa_spec():
    return Config("attention", [OpSpec(f"flash_attn_decode_{t // 1024}k",
                                       2 * FA_HEADS * FA_D * F32 + 2 * FA_KV_HEADS * t * FA_D * 2,
                                       FA_HEADS * t * FA_D) for t in FA_TOKENS])


# Diagonal family (diag.rs): a causal mask over a [4096, 4096] score matrix
# (n_past 0, the query / key extent of configuration 4a), N(0, 1) scores.
# Algorithmic bytes: the kept lower triangle read once, every element written.
DIAG_SIDE = 4096


def diag_inputs(seed=16):
    rng = np.random.default_rng(seed)
    return normal(rng, (DIAG_SIDE * DIAG_SIDE,))


def diag_spec():
    n = DIAG_SIDE * DIAG_SIDE
    kept = DIAG_SIDE * (DIAG_SIDE + 1) // 2
    return Config("diag", [OpSpec("diag_mask_inf_causal", (kept + n) * F32, n),
                           OpSpec("diag_mask_zero_causal", (kept + n) * F32, n),
                           OpSpec("soft_max_diag_mask_inf_causal", (kept + n) * F32, n)])


# The same vocabulary step with Q8_0 rows (matmul.rs OpMulMatArgmaxQ8_0):
# [4096, 151936] as 128 blocks of 34 bytes per row (binary16 scales
# 2^-10 * U(0.5, 1), quants uniform in [-127, 127]), rhs N(0, 1).
def mvq8_inputs(seed=17):
    rng = np.random.default_rng(seed)
    blocks = MV_K // 32
    blob = rng.integers(-127, 128, size=(MV_ROWS, blocks, 34), dtype=np.int8).view(np.uint8)
    d = (rng.uniform(0.5, 1.0, size=(MV_ROWS, blocks)) / 1024.0).astype(np.float16)
    blob[:, :, :2] = d.view(np.uint8).reshape(MV_ROWS, blocks, 2)
    rhs = normal(rng, (MV_K,), 1.0).astype(np.float32)
    return blob.reshape(-1), rhs


def mvq8_spec():
    row_bytes = MV_K // 32 * 34
    return Config("matvec", [OpSpec("mul_mat_argmax_q8_0_vocab", MV_ROWS * row_bytes + MV_K * F32 + 8,
                                    MV_K * MV_ROWS)])


# The vocabulary step with K-quant rows (matmul.rs OpMulMatArgmaxQ2K / Q3K /
# Q4K / Q6K):
# [4096, 151936] as 16 blocks of 256 values per row, random block bytes with
# binary16 scales 2^-10 * U(0.5, 1) (Q6_K: signed group scales in [-64, 64)).
K_BLOCK_BYTES = {"q2_k": 84, "q3_k": 110, "q4_k": 144, "q6_k": 210}


def mvk_inputs(fmt, seed=18):
    rng = np.random.default_rng(seed)
    blocks, bb = MV_K // 256, K_BLOCK_BYTES[fmt]
    blob = rng.integers(0, 256, size=(MV_ROWS, blocks, bb), dtype=np.uint8)
    if fmt in ("q2_k", "q3_k"):
        pos, nd = (80, 2) if fmt == "q2_k" else (108, 1)
        d = (rng.uniform(0.5, 1.0, size=(MV_ROWS, blocks, nd)) / 1024.0).astype(np.float16)
        blob[:, :, pos:pos + 2 * nd] = d.view(np.uint8).reshape(MV_ROWS, blocks, 2 * nd)
    elif fmt == "q4_k":
        d = (rng.uniform(0.5, 1.0, size=(MV_ROWS, blocks, 2)) / 1024.0).astype(np.float16)
        blob[:, :, :4] = d.view(np.uint8).reshape(MV_ROWS, blocks, 4)
    else:
        blob[:, :, 192:208] = rng.integers(-64, 64, size=(MV_ROWS, blocks, 16), dtype=np.int8).view(np.uint8)
        d = (rng.uniform(0.5, 1.0, size=(MV_ROWS, blocks)) / 1024.0).astype(np.float16)
        blob[:, :, 208:210] = d.view(np.uint8).reshape(MV_ROWS, blocks, 2)
    rhs = normal(rng, (MV_K,), 1.0).astype(np.float32)
    return blob.reshape(-1), rhs


def mvk_spec(fmt):
    row_bytes = MV_K // 256 * K_BLOCK_BYTES[fmt]
    return OpSpec(f"mul_mat_argmax_{fmt}_vocab", MV_ROWS * row_bytes + MV_K * F32 + 8, MV_K * MV_ROWS)
