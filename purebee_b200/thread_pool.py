"""Row split of the Q4 matvec across GPUs: the multi-device form of
thread-pool.js's AtomicsThreadPool (thread-pool.js:57-345).

The reference splits the rows of every matvec over worker threads
(thread-pool.js:165-246: rowsPerThread = floor(N / T), the remainder to the
first workers, the main thread takes the tail) and copies the per-thread row
slices back into one output.  Here the workers are GPUs, one process per GPU:
each rank keeps a contiguous slice of the rows resident on its device,
computes it with the CUDA matvec, and the library's NCCL all-gather
(pb_comm_allgather) assembles y on every rank.  torch.distributed only
carries the communicator's unique id between the processes.  A row's result does not depend on which rows
share its launch, so the gathered y has the same bits as a one-device matvec.

Slices are whole 8-row tiles (the device layout's unit) and all but the last
rank get the same number of rows, so the gathered buffer's first N values are
y in order with no reassembly.
"""
from __future__ import annotations

import ctypes
from typing import List, Optional, Tuple

import numpy as np

from . import _native as N_

TILE = 8
_GGUF_BLOCK = {N_.TYPE_Q4_0: 18, N_.TYPE_Q4_1: 20}


def row_split(n_rows: int, world: int) -> List[Tuple[int, int]]:
    """[lo, hi) row range of each rank: ceil(tiles / world) tiles per rank,
    the last rank takes what is left (possibly nothing)."""
    if n_rows <= 0 or world <= 0:
        raise ValueError("row_split needs n_rows > 0 and world > 0")
    tiles = (n_rows + TILE - 1) // TILE
    per = (tiles + world - 1) // world * TILE
    return [(min(n_rows, r * per), min(n_rows, (r + 1) * per)) for r in range(world)]


def rows_per_rank(n_rows: int, world: int) -> int:
    """Padded slice length every rank contributes to the all-gather."""
    lo, hi = row_split(n_rows, world)[0]
    return hi - lo


def assemble_rows(slices, n_rows: int) -> np.ndarray:
    """The full y from the ranks' padded slices in rank order (what the
    all-gather leaves in its receive buffer): their concatenation cut to
    n_rows.  Host-side statement of the layout the device gather produces."""
    world = len(slices)
    per = rows_per_rank(n_rows, world)
    flat = np.concatenate([np.asarray(s, np.float32).reshape(-1)[:per] for s in slices])
    return flat[:n_rows]


class RowSplitMatvec:
    """One Q4_0/Q4_1 matrix split by rows over the ranks of a communicator
    (NcclComm: the library's pb_comm, one rank per process and GPU).

    `raw` is the whole matrix as GGUF bytes (row-major blocks, as the
    reference's rawBuf); each rank uploads only its own rows.  `matvec(x_ptr)`
    takes x (K floats) at a device address on this rank's device, runs the
    rank's rows into its slice and all-gathers the slices with
    pb_comm_allgather on the library stream; the first N floats of `y` are
    the full result on every rank."""

    def __init__(self, ctx: N_.Context, raw: np.ndarray, quant_type: int, n_rows: int, k: int, comm):
        if quant_type not in _GGUF_BLOCK:
            raise ValueError("row-split matvec supports Q4_0 and Q4_1")
        if k % 32:
            raise ValueError("K must be a multiple of 32")
        self.ctx, self.N, self.K, self.comm = ctx, n_rows, k, comm
        self.rank, self.world = comm.rank, comm.world
        self.lo, self.hi = row_split(n_rows, self.world)[self.rank]
        self.per = rows_per_rank(n_rows, self.world)
        row_bytes = (k // 32) * _GGUF_BLOCK[quant_type]
        raw = np.ascontiguousarray(raw, np.uint8)
        if raw.size != n_rows * row_bytes:
            raise ValueError(f"raw holds {raw.size} bytes, expected {n_rows * row_bytes}")
        self.m = None
        if self.hi > self.lo:
            self.m = N_.QMat(ctx, quant_type, raw[self.lo * row_bytes:self.hi * row_bytes], self.hi - self.lo, k)
        self.y_local = ctx.alloc(self.per * 4)
        self.y = ctx.alloc(self.world * self.per * 4)
        ctx._check(N_.lib().pb_memset(ctx.h, self.y_local.ptr, 0, self.per * 4))

    def local(self, x_ptr: int) -> None:
        """This rank's rows into y_local (enqueued on the library's stream)."""
        if self.m is not None:
            self.ctx._check(N_.lib().pb_qmat_matvec(self.ctx.h, self.m.h, ctypes.c_void_p(x_ptr),
                                                    ctypes.c_void_p(self.y_local.ptr), 0, 0))

    def gather(self) -> None:
        """Every rank's slice into y (pb_comm_allgather, library stream)."""
        self.comm.allgather(self.y_local.ptr, self.y.ptr, self.per * 4)

    def matvec(self, x_ptr: int) -> N_.DeviceBuffer:
        """Full y on every rank (device buffer; the first N floats), enqueued
        on the library's stream: local rows, then the all-gather."""
        self.local(x_ptr)
        self.gather()
        return self.y

    def free(self) -> None:
        if self.m is not None:
            self.m.free()
            self.m = None
        for b in (getattr(self, "y_local", None), getattr(self, "y", None)):
            if b is not None:
                b.free()


class AtomicsThreadPool:
    """thread-pool.js:57-345 over GPUs: `matvec(x, rawBuf, quantType, N, K)`
    with host arrays in and out, every rank computing its rows.  Like the
    reference, each call copies the weight slice in (here to the device); a
    runtime that keeps weights resident uses RowSplitMatvec instead."""

    def __init__(self, ctx: N_.Context, comm):
        self.ctx, self.comm = ctx, comm

    def matvec(self, x: np.ndarray, rawBuf: np.ndarray, quantType: int, N: int, K: int) -> np.ndarray:
        rs = RowSplitMatvec(self.ctx, rawBuf, quantType, N, K, self.comm)
        try:
            xd = self.ctx.to_device(np.ascontiguousarray(x, np.float32))
            y = rs.matvec(xd.ptr)
            out = y.download(np.float32, self.world_rows(rs))[:N]
            xd.free()
            return out
        finally:
            rs.free()

    @staticmethod
    def world_rows(rs: RowSplitMatvec) -> int:
        return rs.world * rs.per

    def shutdown(self) -> None:
        pass


def split_plan(config, world: int, rank: int) -> "N_.SplitPlan":
    """pb_batch_split_plan: the rows `rank` of `world` holds in a row-split
    batch (heads, wo / w2 / gate|up row chunks, vocab rows).  `config` is a
    ModelConfig or a LlamaConfig."""
    if isinstance(config, N_.ModelConfig):
        c = config
    else:
        c = N_.ModelConfig(N_.MODEL_STREAMING_Q4, N_.TYPE_Q4_0, config.dim, config.hiddenDim, config.nLayers,
                           config.nHeads, config.nKvHeads, config.headDim, config.vocabSize, config.seqLen,
                           config.ropeTheta, config.rmsNormEps)
    p = N_.SplitPlan()
    rc = N_.lib().pb_batch_split_plan(ctypes.byref(c), int(world), int(rank), ctypes.byref(p))
    if rc != N_.PB_OK:
        raise ValueError(f"no row split of this model over {world} ranks (n_kv_heads, dim / 64 and hidden_dim / 64 "
                         f"must divide by it)")
    return p


class NcclComm:
    """An NCCL communicator of the library (pb_comm), one rank per process and
    device: the row-split batch's all-gathers run on it, inside the recorded
    decode graph.  `from_torch` sends rank 0's unique id to the other ranks
    over an initialised torch.distributed group (any backend)."""

    def __init__(self, ctx, world: int, rank: int, uid: bytes):
        if len(uid) != N_.COMM_ID_BYTES:
            raise ValueError("an NCCL unique id is 128 bytes")
        self.ctx = ctx
        self.world, self.rank = int(world), int(rank)
        buf = ctypes.create_string_buffer(bytes(uid), N_.COMM_ID_BYTES)
        h = ctypes.c_void_p()
        ctx._check(N_.lib().pb_comm_init(ctx.h, self.world, self.rank, buf, ctypes.byref(h)))
        self.h = h.value

    @staticmethod
    def new_id() -> bytes:
        buf = ctypes.create_string_buffer(N_.COMM_ID_BYTES)
        if N_.lib().pb_comm_id(buf) != N_.PB_OK:
            raise RuntimeError("ncclGetUniqueId failed (is libnccl.so.2 present?)")
        return buf.raw

    @staticmethod
    def exchange_id(group=None) -> bytes:
        """Rank 0 makes the id; every rank returns it."""
        import torch.distributed as dist
        obj = [NcclComm.new_id() if dist.get_rank(group) == 0 else None]
        dist.broadcast_object_list(obj, src=0, group=group)
        return obj[0]

    @classmethod
    def from_torch(cls, ctx, group=None) -> "NcclComm":
        import torch.distributed as dist
        uid = cls.exchange_id(group)
        return cls(ctx, dist.get_world_size(group), dist.get_rank(group), uid)

    @property
    def peer_access(self) -> bool:
        """True when exchanges run over peer memory (else NCCL all-gathers)."""
        return bool(N_.lib().pb_comm_peer_access(self.h))

    def allgather(self, send_ptr: int, recv_ptr: int, nbytes: int) -> None:
        """recv [world][nbytes] <- every rank's send [nbytes] (device pointers,
        on the context's stream)."""
        self.ctx._check(N_.lib().pb_comm_allgather(self.h, send_ptr, recv_ptr, int(nbytes)))

    def free(self):
        if getattr(self, "h", None) and self.ctx.h:
            N_.lib().pb_comm_free(self.h)
        self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass
