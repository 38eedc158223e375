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

Split units keep the pairs consistent: q and o's input in units of two heads (256 columns, o's K-shards must be
whole 256-column blocks), k/v in single KV heads (query heads of rank i use KV heads of rank i under GQA), gate/up
and down's input in 256-row units. Uneven counts are spread by a balanced contiguous split.
"""
import ctypes as C
from dataclasses import dataclass

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


def row_shard(slot, K, rows, world, rank, unit=256):
    """Row-parallel shard: input columns [lo, hi) of this rank, split in units of `unit` columns (a multiple of 256)."""
    if unit % 256 or K % unit:
        raise ValueError("row split unit must divide K and be a multiple of 256")
    u0, u1 = balanced(K // unit, world, rank)
    lo, hi = u0 * unit, u1 * unit
    if hi == lo:
        return Shard("row", lo, hi, rows, 0, np.zeros(0, np.uint8))
    s = fmt.shard_cols(slot, K, rows, lo // 256, hi // 256)
    return Shard("row", lo, hi, rows, hi - lo, s)


@dataclass
class LayerDims:
    hidden: int
    ffn: int
    heads: int
    kv_heads: int
    head_dim: int


LLAMA3_8B = LayerDims(hidden=4096, ffn=14336, heads=32, kv_heads=8, head_dim=128)


def layer_units(d: LayerDims):
    """split unit (rows for column-parallel, input columns for row-parallel) of each projection of a layer"""
    qunit = 2 * d.head_dim if (2 * d.head_dim) % 256 == 0 else 256
    return {"q": qunit, "k": d.head_dim, "v": d.head_dim, "o": qunit, "gate": 256, "up": 256, "down": 256}


def layer_plan(d: LayerDims, world, rank):
    """(kind, unit) per projection and the rank's ranges; o's input range equals q's row range and down's input range
    equals gate/up's row range, so each rank feeds its row-parallel projections from its own outputs."""
    u = layer_units(d)
    kinds = {"q": "col", "k": "col", "v": "col", "o": "row", "gate": "col", "up": "col", "down": "row"}
    rows = {"q": d.heads * d.head_dim, "k": d.kv_heads * d.head_dim, "v": d.kv_heads * d.head_dim,
            "o": d.hidden, "gate": d.ffn, "up": d.ffn, "down": d.hidden}
    K = {"q": d.hidden, "k": d.hidden, "v": d.hidden, "o": d.heads * d.head_dim, "gate": d.hidden, "up": d.hidden,
         "down": d.ffn}
    plan = {}
    for n in kinds:
        n_units = (rows[n] if kinds[n] == "col" else K[n]) // u[n]
        lo, hi = balanced(n_units, world, rank)
        plan[n] = (kinds[n], u[n], lo * u[n], hi * u[n], rows[n], K[n])
    assert plan["o"][2:4] == plan["q"][2:4] and plan["down"][2:4] == plan["gate"][2:4]
    return plan


def shard_for(plan_entry, slot, world, rank):
    kind, unit, _, _, rows, K = plan_entry
    if kind == "col":
        return column_shard(slot, K, rows, world, rank, unit)
    return row_shard(slot, K, rows, world, rank, unit)


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


def exchange_entries(y, prm, rows):
    """A rank's exchange entries (int64 bit patterns, sorted-row order) for its partial output y (original row order,
    float32 CUDA) of a tensor with row permutation prm (sorted -> original row): entry i holds y[prm[i]] with the tag
    0x80000000 | prm[i] << 16 | rows / 32 in its high word (layout: p8_tp_gemv_allreduce)."""
    import torch

    p = torch.as_tensor(np.asarray(prm, np.int64), device=y.device)
    bits = y[p].view(torch.int32).to(torch.int64) & 0xFFFFFFFF
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

    def __init__(self, slot, K, rows, world, rank, unit=256, device="cuda", group=None, comm=None):
        import torch

        from .ops import P8Tensor

        self.shard = row_shard(slot, K, rows, world, rank, unit)
        self.lo, self.hi = self.shard.lo, self.shard.hi
        self.group = group
        self.t = P8Tensor(torch.from_numpy(self.shard.slot).to(device), self.shard.K, rows) if self.shard.K else None
        # the same decision on every rank: it depends only on K, unit and world
        self.comm = comm if comm is not None and world <= K // unit and world > 1 else None

    def __call__(self, x_local, out=None, workspace=None, stream=None):
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
            Y = self.t.mul_mat(X_local, out=out, workspace=workspace, stream=stream)
        return reduce_partials(Y, self.group)
