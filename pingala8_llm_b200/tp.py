"""Tensor-parallel split of Pingala-8 projections over the GPUs of one node (one process per GPU, torch.distributed).

The reference runs one GPU; this layer is new. It follows the usual decoder-layer split, so no activation moves
between the two projections of a pair:

  column-parallel (q, k, v, gate, up)  rank i holds the ORIGINAL output rows [r0_i, r1_i) as a standalone slot
                                       (p8_tp_shard_rows: rows re-tiled, lane rotation remapped); its output is the
                                       rank's slice of y, consumed locally (attention heads, SwiGLU).
  row-parallel    (o, down)            rank i holds the 256-column blocks of its input slice (p8_tp_shard_cols); its
                                       output is a partial y over all rows, summed over ranks either inside the GEMV
                                       (TpComm: p8_tp_gemv_allreduce, the epilogue stores the partial rows into the
                                       peers' exchange buffers over NVLink and sums the ranks' rows in rank order) or
                                       by an NCCL all-reduce after it.

Split units keep the pairs consistent. q/k/v are split by whole GQA groups: rank i holds KV heads [k0, k1) and exactly
the query heads that read them, so attention needs no exchange. o's input columns are then the rank's q rows; where
that range is not a whole number of 256-column Hadamard blocks (Qwen3-14B at TP8: 5 query heads = 640 columns per rank)
the rank's o shard holds every block its range touches, and a boundary block is held by both neighbours: the Hadamard
transform is linear, so each rank multiplies the full block's weights by its own columns with the other rank's
columns zero, and the two partial outputs add up to the block's product. gate/up and down's input are split in
256-row units (whole blocks). Uneven counts are spread by a balanced contiguous split.
"""
import ctypes as C
from dataclasses import dataclass
from typing import NamedTuple

import numpy as np

from . import fmt


def balanced(n, world, rank):
    """contiguous share [lo, hi) of n units for rank of world (sizes differ by at most one unit)"""
    return n * rank // world, n * (rank + 1) // world


@dataclass
class Shard:
    kind: str      # "col" (rows [lo, hi)) or "row" (columns [lo, hi))
    lo: int
    hi: int
    rows: int      # rows of the shard slot
    K: int         # K of the shard slot
    slot: np.ndarray


def column_shard(slot, K, rows, world, rank, unit=32):
    """Column-parallel shard: ORIGINAL rows [lo, hi) of this rank, split in units of `unit` rows (a multiple of 32)."""
    if unit % 32 or rows % unit:
        raise ValueError("column split unit must divide rows and be a multiple of 32")
    u0, u1 = balanced(rows // unit, world, rank)
    lo, hi = u0 * unit, u1 * unit
    if hi == lo:
        return Shard("col", lo, hi, 0, K, np.zeros(0, np.uint8))
    s, _ = fmt.shard_rows(slot, K, rows, lo, hi)
    return Shard("col", lo, hi, hi - lo, K, s)


def row_shard(slot, K, rows, world, rank, unit=256, cols=None):
    """Row-parallel shard: input columns [lo, hi) of this rank, split in units of `unit` columns (a multiple of 256),
    or the explicit range cols = (lo, hi). The shard holds the 256-column blocks that [lo, hi) touches; with an
    unaligned range its boundary blocks are also held by the neighbouring rank, and the caller zeroes the input
    columns outside [lo, hi) (RowParallel does)."""
    if cols is None:
        if unit % 256 or K % unit:
            raise ValueError("row split unit must divide K and be a multiple of 256")
        u0, u1 = balanced(K // unit, world, rank)
        lo, hi = u0 * unit, u1 * unit
    else:
        lo, hi = cols
        if not 0 <= lo <= hi <= K:
            raise ValueError("row shard columns outside [0, K)")
    if hi == lo:
        return Shard("row", lo, hi, rows, 0, np.zeros(0, np.uint8))
    b0, b1 = lo // 256, (hi + 255) // 256
    s = fmt.shard_cols(slot, K, rows, b0, b1)
    return Shard("row", lo, hi, rows, 256 * (b1 - b0), s)


@dataclass
class LayerDims:
    hidden: int
    ffn: int
    heads: int
    kv_heads: int
    head_dim: int


LLAMA3_8B = LayerDims(hidden=4096, ffn=14336, heads=32, kv_heads=8, head_dim=128)


QWEN3_14B = LayerDims(hidden=5120, ffn=17408, heads=40, kv_heads=8, head_dim=128)
QWEN3_4B = LayerDims(hidden=2560, ffn=9728, heads=32, kv_heads=8, head_dim=128)


class PlanEntry(NamedTuple):
    """One projection's split on one rank. col: original output rows [lo, hi). row: input columns [lo, hi), held as
    the 256-column blocks [b0, b1) (b0 = lo // 256, b1 = ceil(hi / 256); the rank's input is zero outside [lo, hi))."""
    kind: str
    unit: int
    lo: int
    hi: int
    rows: int
    K: int
    b0: int = 0
    b1: int = 0

    @property
    def shard_rows(self):
        return self.hi - self.lo if self.kind == "col" else self.rows

    @property
    def shard_K(self):
        return self.K if self.kind == "col" else 256 * (self.b1 - self.b0)


def layer_plan(d: LayerDims, world, rank):
    """PlanEntry per projection of a decoder layer on this rank. o's input range equals q's row range and down's input
    range equals gate/up's row range, so each rank feeds its row-parallel projections from its own outputs; q/k/v
    follow whole GQA groups (the rank's query heads read exactly the rank's KV heads)."""
    g = d.heads // d.kv_heads
    hd = d.head_dim
    k0, k1 = balanced(d.kv_heads, world, rank)
    f0, f1 = balanced(d.ffn // 256, world, rank)
    plan = {
        "q": PlanEntry("col", g * hd, k0 * g * hd, k1 * g * hd, d.heads * hd, d.hidden),
        "k": PlanEntry("col", hd, k0 * hd, k1 * hd, d.kv_heads * hd, d.hidden),
        "v": PlanEntry("col", hd, k0 * hd, k1 * hd, d.kv_heads * hd, d.hidden),
        "o": PlanEntry("row", g * hd, k0 * g * hd, k1 * g * hd, d.hidden, d.heads * hd,
                       (k0 * g * hd) // 256, (k1 * g * hd + 255) // 256),
        "gate": PlanEntry("col", 256, 256 * f0, 256 * f1, d.ffn, d.hidden),
        "up": PlanEntry("col", 256, 256 * f0, 256 * f1, d.ffn, d.hidden),
        "down": PlanEntry("row", 256, 256 * f0, 256 * f1, d.hidden, d.ffn, f0, f1),
    }
    assert plan["o"][2:4] == plan["q"][2:4] and plan["down"][2:4] == plan["gate"][2:4]
    return plan


def shard_for(e, slot, world, rank):
    """this rank's shard of one projection's slot, as the plan entry e says"""
    if e.kind == "col":
        if e.hi == e.lo:
            return Shard("col", e.lo, e.hi, 0, e.K, np.zeros(0, np.uint8))
        s, _ = fmt.shard_rows(slot, e.K, e.rows, e.lo, e.hi)
        return Shard("col", e.lo, e.hi, e.hi - e.lo, e.K, s)
    return row_shard(slot, e.K, e.rows, world, rank, cols=(e.lo, e.hi))


def reduce_partials(y, group=None):
    """sum of the row-parallel partial outputs over the ranks of group, in place (NCCL on CUDA tensors)"""
    import torch.distributed as dist

    if dist.is_initialized() and dist.get_world_size(group) > 1:
        dist.all_reduce(y, op=dist.ReduceOp.SUM, group=group)
    return y


class TpComm:
    """This rank's exchange buffer for fused row-parallel calls (p8_tp_comm_*): rank of world (<= 8) on the current
    device, up to max_rows output rows per call, device waits bounded by timeout_ms. connect() makes one per rank of a
    process group and maps every peer's buffer (CUDA IPC handles exchanged through the group)."""

    def __init__(self, rank, world, max_rows, timeout_ms=1000):
        from ._lib import check, lib

        h = C.c_void_p()
        check(lib().p8_tp_comm_create(rank, world, max_rows, timeout_ms, C.byref(h)), "p8_tp_comm_create")
        self._h = h
        self.rank, self.world, self.max_rows, self.timeout_ms = rank, world, max_rows, timeout_ms

    @classmethod
    def connect(cls, max_rows, group=None, timeout_ms=1000):
        import torch.distributed as dist

        rank, world = dist.get_rank(group), dist.get_world_size(group)
        c = cls(rank, world, max_rows, timeout_ms)
        info = [None] * world
        dist.all_gather_object(info, (world, max_rows, c.ipc_handle()), group=group)
        if any(w != world or m != max_rows for w, m, _ in info):
            c.close()
            raise ValueError("TpComm.connect: ranks asked for different world sizes or max_rows")
        for q, (_, _, hnd) in enumerate(info):
            if q != rank:
                c.open_peer(q, hnd)
        return c

    @property
    def handle(self):
        from ._lib import P8Error

        if self._h is None:
            raise P8Error(-1, "TpComm closed")
        return self._h

    def ipc_handle(self):
        from ._lib import check, lib

        buf = C.create_string_buffer(64)
        check(lib().p8_tp_comm_ipc_handle(self.handle, buf, 64), "p8_tp_comm_ipc_handle")
        return buf.raw

    def open_peer(self, q, ipc_handle):
        from ._lib import check, lib

        check(lib().p8_tp_comm_open_peer(self.handle, q, C.c_char_p(bytes(ipc_handle)), len(ipc_handle)),
              "p8_tp_comm_open_peer")

    def set_peer(self, q, dev_ptr):
        """attach peer q's buffer by device address (one process, or a local stand-in buffer)"""
        from ._lib import check, lib

        check(lib().p8_tp_comm_set_peer(self.handle, q, C.c_void_p(int(dev_ptr))), "p8_tp_comm_set_peer")

    def buffer(self):
        """this rank's exchange buffer as an int64 CUDA tensor [2, world, max_rows] (entry layout: p8_tp_gemv_allreduce)"""
        import torch

        from ._lib import check, lib

        p, n = C.c_void_p(), C.c_size_t()
        check(lib().p8_tp_comm_buffer(self.handle, C.byref(p), C.byref(n)), "p8_tp_comm_buffer")
        shape = (2, self.world, self.max_rows)
        owner = self

        class _View:
            __cuda_array_interface__ = {"shape": shape, "typestr": "<i8", "data": (p.value, False), "version": 3}
            keep = owner

        return torch.as_tensor(_View(), device="cuda")

    def epoch(self):
        """fused calls made so far on this communicator"""
        from ._lib import check, lib

        e = C.c_uint32()
        check(lib().p8_tp_comm_epoch(self.handle, C.byref(e)), "p8_tp_comm_epoch")
        return e.value

    def reset(self, stream=None):
        """zero the buffer and the call count (after a failed exchange: every rank, between steps)"""
        from ._lib import check, lib
        from .ops import _stream

        check(lib().p8_tp_comm_reset(self.handle, _stream(stream)), "p8_tp_comm_reset")

    def close(self):
        if getattr(self, "_h", None) is not None:
            from ._lib import lib

            lib().p8_tp_comm_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def exchange_entries(y, rows):
    """A rank's exchange entries (int64 bit patterns, output-row order) for its partial output y (float32 CUDA) of a
    tensor with `rows` rows: entry ro holds y[ro] with the tag 0x80000000 | ro << 16 | rows / 32 in its high word
    (layout: p8_tp_gemv_allreduce)."""
    import torch

    p = torch.arange(y.numel(), dtype=torch.int64, device=y.device)
    bits = y.view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    tag = (0x80000000 | (p << 16) | (int(rows) >> 5)) - (1 << 32)  # the tag as a negative int32 (bit 31 set)
    return bits | (tag << 32)  # the same 64 bits as a signed int64


class ColumnParallel:
    """this rank's rows of a column-parallel projection: y_local = W[lo:hi] x"""

    def __init__(self, slot, K, rows, world, rank, unit=32, device="cuda"):
        import torch

        from .ops import P8Tensor

        self.shard = column_shard(slot, K, rows, world, rank, unit)
        self.lo, self.hi = self.shard.lo, self.shard.hi
        self.t = P8Tensor(torch.from_numpy(self.shard.slot).to(device), K, self.shard.rows) if self.shard.rows else None

    def __call__(self, x, out=None, workspace=None, stream=None):
        if self.t is None:  # more ranks than split units: this rank holds no rows
            import torch

            return torch.empty(0, dtype=torch.float32, device=x.device)
        return self.t.mul_mat_vec(x, out=out, workspace=workspace, stream=stream)

    def mul_mat(self, X, out=None, workspace=None, stream=None):
        """batched product [tokens, K] -> this rank's output columns [tokens, hi - lo] (prefill)"""
        if self.t is None:
            import torch

            return torch.empty(X.shape[0], 0, dtype=torch.float32, device=X.device)
        return self.t.mul_mat(X, out=out, workspace=workspace, stream=stream)


class RowParallel:
    """this rank's input columns of a row-parallel projection: y = all_reduce_sum(W[:, lo:hi] x[lo:hi]).

    With comm (a TpComm of the group) the sum happens inside the GEMV (p8_tp_gemv_allreduce); every rank must then
    hold input columns (world <= K / unit), else the NCCL all-reduce after the GEMV is used on every rank."""

    def __init__(self, slot, K, rows, world, rank, unit=256, device="cuda", group=None, comm=None, cols=None):
        import torch

        from .ops import P8Tensor

        self.shard = row_shard(slot, K, rows, world, rank, unit, cols=cols)
        self.lo, self.hi = self.shard.lo, self.shard.hi
        self.off = self.lo - 256 * (self.lo // 256)  # the rank's columns inside its first block
        self.group = group
        self.t = P8Tensor(torch.from_numpy(self.shard.slot).to(device), self.shard.K, rows) if self.shard.K else None
        # the same decision on every rank: it depends only on the split, which every rank computes alike
        every_rank_has_columns = (cols is None and world <= K // unit) or (cols is not None and self.hi > self.lo)
        self.comm = comm if comm is not None and every_rank_has_columns and world > 1 else None
        self._xpad = None

    def padded(self, x_local):
        """x_local (the rank's hi - lo input columns) placed into the shard's blocks, zero outside [lo, hi)"""
        if self.t is None or (self.off == 0 and x_local.shape[-1] == self.shard.K):
            return x_local
        import torch

        shape = x_local.shape[:-1] + (self.shard.K,)
        if self._xpad is None or self._xpad.shape != shape or self._xpad.device != x_local.device:
            self._xpad = torch.zeros(shape, dtype=torch.float32, device=x_local.device)
        self._xpad[..., self.off:self.off + x_local.shape[-1]] = x_local
        return self._xpad

    def __call__(self, x_local, out=None, workspace=None, stream=None):
        x_local = self.padded(x_local)
        if self.comm is not None:
            return self.t.mul_mat_vec_allreduce(x_local, self.comm, out=out, workspace=workspace, stream=stream)
        if self.t is None:  # no input columns on this rank: contribute zeros to the sum
            import torch

            y = out.zero_() if out is not None else torch.zeros(self.shard.rows, dtype=torch.float32, device=x_local.device)
        else:
            y = self.t.mul_mat_vec(x_local, out=out, workspace=workspace, stream=stream)
        return reduce_partials(y, self.group)

    def mul_mat(self, X_local, out=None, workspace=None, stream=None):
        """batched product (prefill): X_local [tokens, hi - lo] (this rank's input columns) -> the summed output
        [tokens, rows] on every rank: the rank's partial from the batched product, then an NCCL all-reduce (the
        partials are [tokens, rows] f32, large enough for the collective's bandwidth-optimised algorithms)"""
        import torch

        if self.t is None:
            Y = out.zero_() if out is not None else torch.zeros(X_local.shape[0], self.shard.rows, dtype=torch.float32,
                                                                 device=X_local.device)
        else:
            Y = self.t.mul_mat(self.padded(X_local).contiguous(), out=out, workspace=workspace, stream=stream)
        return reduce_partials(Y, self.group)
