"""Multi-GPU sharding for the hot path: one process per GPU.

Tensors are partitioned along their outermost independent dimension
(dim 3 for the 4-D broadcast workload, rows or heads for the row
operators); the small broadcast operand is replicated on every rank.
Elementwise and row operators need no communication.  Only whole-tensor
sum and argmax combine per-shard partials, with one tiny all-gather: on
B200 through PeerExchange (peer stores over NVLink by two small kernels of
the library, emel_cuda_exchange_*), or over a process group (NCCL, or gloo
on CPU for tests):

  * sum: each rank's f64 accumulator (emel_cuda_sum_f64); the partials are
    added in rank order and rounded once to f32, so the result does not
    depend on timing;
  * argmax: each rank's (value, has_value, global index, first_is_nan)
    partial (emel_cuda_argmax_partial_compute), combined in rank order
    with the reference's first-index and NaN rules
    (emel_cuda_argmax_combine).
"""

import ctypes
import struct

import numpy as np

PARTIAL_BYTES = 24  # sizeof(emel_cuda_argmax_partial)


def shard_bounds(extent, world, rank):
    """[begin, end) of `rank`'s slice of a dimension of `extent`, split as
    evenly as possible (earlier ranks take the remainder)."""
    base, extra = divmod(extent, world)
    begin = rank * base + min(rank, extra)
    return begin, begin + base + (1 if rank < extra else 0)


def pack_partial(value, has_value, index, first_is_nan):
    return struct.pack("<fIqII", value, has_value, index, first_is_nan, 0)


def unpack_partial(raw):
    value, has_value, index, first_is_nan, _ = struct.unpack("<fIqII", bytes(raw))
    return value, has_value, index, first_is_nan


def all_gather_bytes(torch, dist, payload, device=None, group=None):
    """All-gathers one fixed-size byte string per rank (rank order)."""
    t = torch.frombuffer(bytearray(payload), dtype=torch.uint8)
    if device is not None:
        t = t.to(device)
    world = dist.get_world_size(group)
    out = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(out, t, group=group)
    return [bytes(o.cpu().numpy().tobytes()) for o in out]


def combine_sum(partials_f64):
    """Rank-ordered f64 addition, rounded once to f32 (reductions.rs:671-681
    accumulates in f64 and casts the total)."""
    total = 0.0
    for p in partials_f64:
        total += float(p)
    return np.float32(total), total


def combine_argmax(pkg, partials):
    """partials: list of (value, has_value, index, first_is_nan) in rank order."""
    return pkg.argmax_combine(partials)


def global_sum(torch, dist, local_f64, device=None, group=None):
    raw = all_gather_bytes(torch, dist, struct.pack("<d", float(local_f64)), device, group)
    return combine_sum([struct.unpack("<d", r)[0] for r in raw])


def global_argmax(pkg, torch, dist, local_partial, device=None, group=None):
    raw = all_gather_bytes(torch, dist, pack_partial(*local_partial), device, group)
    return combine_argmax(pkg, [unpack_partial(r) for r in raw])


def read_partial(pkg, ctx, device_ptr):
    """Copies an emel_cuda_argmax_partial from device memory."""
    hp = pkg.CArgmaxPartial()
    st = pkg.lib().emel_cuda_memcpy_d2h(ctx.handle, None, ctypes.addressof(hp), device_ptr, ctypes.sizeof(hp))
    if st != 0:
        raise RuntimeError(ctx.last_error)
    ctx.synchronize()
    return hp.value, hp.has_value, hp.index, hp.first_is_nan


EXCHANGE_BYTES = 32  # one rank's payload: f64 shard sum, then its argmax partial


class PeerExchange:
    """The library's NVLink peer exchange (emel_cuda_exchange_*): every rank
    publishes a fixed-size device payload into every rank's buffer and waits
    for all of them, on a stream, inside captured graphs too.  Buffer handles
    travel once over the process group (`dist`) at construction."""

    def __init__(self, pkg, ctx, dist, world, rank, nbytes=EXCHANGE_BYTES, timeout_ms=10000):
        self.pkg, self.ctx, self.lib = pkg, ctx, pkg.lib()
        self.world, self.rank, self.nbytes = world, rank, nbytes
        h = ctypes.c_void_p()
        self._check(self.lib.emel_cuda_exchange_create(ctx.handle, world, rank, nbytes, timeout_ms, ctypes.byref(h)),
                    "exchange create")
        self.handle = h
        mine = (ctypes.c_uint8 * 64)()
        self._check(self.lib.emel_cuda_exchange_handle(self.handle, mine), "exchange handle")
        handles = [None] * world
        dist.all_gather_object(handles, bytes(mine))
        flat = (ctypes.c_uint8 * (64 * world)).from_buffer_copy(b"".join(handles))
        self._check(self.lib.emel_cuda_exchange_connect(ctx.handle, self.handle, flat), "exchange connect")

    def _check(self, st, what):
        if st != 0:
            raise RuntimeError(f"{what} failed: status {st}: {self.ctx.last_error}")

    def publish(self, stream, payload_ptr):
        self._check(self.lib.emel_cuda_exchange_publish(self.ctx.handle, stream, self.handle,
                                                         ctypes.c_void_p(payload_ptr)), "exchange publish")

    def wait(self, stream, gathered_ptr):
        self._check(self.lib.emel_cuda_exchange_wait(self.ctx.handle, stream, self.handle,
                                                      ctypes.c_void_p(gathered_ptr)), "exchange wait")

    def close(self):
        if self.handle:
            self.lib.emel_cuda_exchange_destroy(self.ctx.handle, self.handle)
            self.handle = None


def combine_gathered(pkg, raw, world):
    """Sum and argmax of the whole tensor from `world` 32-byte exchange
    payloads (rank order): (f32 sum, index)."""
    sums = [struct.unpack("<d", raw[32 * k:32 * k + 8])[0] for k in range(world)]
    partials = [unpack_partial(raw[32 * k + 8:32 * (k + 1)]) for k in range(world)]
    total32, _ = combine_sum(sums)
    index, _ = combine_argmax(pkg, partials)
    return total32, index
