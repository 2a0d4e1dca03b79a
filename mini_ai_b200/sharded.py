"""Row-sharded quantized linear across GPUs (one process per GPU).

The hot path's multi-GPU form: a projection of N = G*R output rows is split
into G equal row shards, rank r holding rows [r*R, (r+1)*R). Each rank runs
the ordinary kernels on its shard and one NCCL all-gather over NVLink
assembles the full output on every rank (mq_linear_sharded_allgather). Rows
are independent, so the result equals the unsharded product up to fp32
summation order (the kernels split each tile's K range by the launch's total
work, so a shard may sum in another order; bit-identical where both launches
split alike, as for products with no more (tile, K step) chunks than SMs).

The reference runs every linear on one device (``--device N``,
src/main.cc:249-250); this module is new surface for the multi-GPU row.
Only the communicator id travels through torch.distributed (any backend);
the data path is the C ABI.
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from . import _lib
from ._lib import check, lib
from .quantized_tensor import CudaWeight, QuantizedStorage, _stream_handle, _torch

COMM_ID_BYTES = 128


def shard_rows(rows: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [begin, end) of rank `rank`: equal slices (the all-gather moves equal counts)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    if rows % world:
        raise ValueError(f"{rows} rows do not split into {world} equal shards")
    r = rows // world
    return rank * r, (rank + 1) * r


def assemble(slices: list[np.ndarray]) -> np.ndarray:
    """Host statement of what the all-gather builds: per-rank [m, R] slices,
    rank order, side by side -> [m, G*R]."""
    return np.concatenate([np.asarray(s) for s in slices], axis=-1)


class CudaComm:
    """An NCCL communicator over the ranks that hold one weight's shards."""

    def __init__(self, device: int, world: int, rank: int, comm_id: bytes):
        if len(comm_id) != COMM_ID_BYTES:
            raise ValueError("communicator id must be 128 bytes")
        self.device, self.world, self.rank = device, world, rank
        handle = C.c_void_p()
        buf = C.create_string_buffer(bytes(comm_id), COMM_ID_BYTES)
        check(lib().mq_comm_create(device, world, rank, buf, COMM_ID_BYTES, C.byref(handle)), "mq_comm_create")
        self.handle = handle

    @staticmethod
    def new_id() -> bytes:
        buf = C.create_string_buffer(COMM_ID_BYTES)
        check(lib().mq_comm_unique_id(buf, COMM_ID_BYTES), "mq_comm_unique_id")
        return buf.raw

    @classmethod
    def from_process_group(cls, device: int, group=None) -> "CudaComm":
        """Rank 0 creates the id; torch.distributed carries it to the other ranks."""
        import torch.distributed as dist

        world, rank = dist.get_world_size(group), dist.get_rank(group)
        obj = [cls.new_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0, group=group)
        return cls(device, world, rank, obj[0])

    @property
    def uses_peer_gather(self) -> bool:
        """True when the gather runs over NVLink peer memory, False when over NCCL."""
        rc = lib().mq_comm_uses_peer_gather(self.handle)
        if rc < 0:
            check(rc, "mq_comm_uses_peer_gather")
        return rc == 1

    def close(self) -> None:
        if getattr(self, "handle", None):
            lib().mq_comm_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class ShardedLinear:
    """This rank's row shard of a weight plus the communicator that gathers outputs."""

    def __init__(self, storage: QuantizedStorage, comm: CudaComm, stream=None):
        self.comm = comm
        self.rows, self.cols = storage.rows, storage.cols
        self.row_range = shard_rows(storage.rows, comm.world, comm.rank)
        self.shard = CudaWeight(storage, device=comm.device, row_range=self.row_range, stream=stream)

    @classmethod
    def from_shard(cls, shard: CudaWeight, comm: CudaComm) -> "ShardedLinear":
        """Wrap a shard uploaded by the caller (e.g. from device blocks)."""
        if (shard.row_begin, shard.row_end) != shard_rows(shard.full_rows, comm.world, comm.rank):
            raise ValueError("the shard is not this rank's equal slice")
        self = cls.__new__(cls)
        self.comm, self.shard = comm, shard
        self.rows, self.cols = shard.full_rows, shard.cols
        self.row_range = (shard.row_begin, shard.row_end)
        return self

    def linear(self, x, bias=None, out=None, stream=None):
        """Full y = x · Wᵀ (+ bias) on every rank; x float32 CUDA [M, K] (or [K])."""
        torch = _torch()
        squeeze = x.dim() == 1
        x2 = x.unsqueeze(0) if squeeze else x
        if x2.dim() != 2 or x2.shape[1] != self.cols or x2.dtype != torch.float32 or not x2.is_cuda:
            raise RuntimeError("LinearDispatch: dimension mismatch")
        if x2.stride(1) != 1:
            x2 = x2.contiguous()
        m = x2.shape[0]
        if out is None:
            out = torch.empty((m, self.rows), dtype=torch.float32, device=x.device)
        if out.shape[-1] != self.rows or out.dtype != torch.float32:
            raise RuntimeError("output shape mismatch")
        out2 = out.view(m, self.rows) if out.dim() == 1 else out
        if bias is not None and (bias.numel() != self.rows or bias.dtype != torch.float32):
            raise RuntimeError("bias shape mismatch")
        check(lib().mq_linear_sharded_allgather(self.shard.handle, x2.data_ptr(), m, x2.stride(0),
                                                bias.data_ptr() if bias is not None else None, out2.data_ptr(),
                                                out2.stride(0), self.comm.handle, _stream_handle(stream)),
              "mq_linear_sharded_allgather")
        return out2.view(self.rows) if squeeze and out.dim() != 1 else out

    def close(self) -> None:
        self.shard.close()


__all__ = ["shard_rows", "assemble", "CudaComm", "ShardedLinear", "COMM_ID_BYTES"]
