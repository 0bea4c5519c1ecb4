"""Process-group plumbing for the sharded optimizer: one process per GPU,
torch.distributed for rendezvous, and the library's own NCCL communicator
for the in-step 16-byte exchange (so the C ABI stays free of torch types).
"""
from __future__ import annotations

import ctypes
import os

from . import _lib


def env_rank_world():
    """(rank, world, local_rank) from the torchrun environment, (0, 1, 0) without it."""
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1)),
            int(os.environ.get("LOCAL_RANK", 0)))


def share_unique_id(id_bytes: bytes | None, rank: int) -> bytes:
    """Broadcast rank 0's 128-byte NCCL unique id over the torch process group
    (any backend, gloo included)."""
    import torch.distributed as dist
    obj = [id_bytes if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    return obj[0]


def nccl_unique_id() -> bytes:
    buf = ctypes.create_string_buffer(128)
    _lib.check("ark_cuda_nccl_unique_id", _lib.lib().ark_cuda_nccl_unique_id(buf))
    return buf.raw


def nccl_comm(rank: int, world: int, device: int):
    """Create the library's NCCL communicator for this rank (collective:
    every rank calls it).  Returns an opaque handle for Optimizer(comm=...)."""
    uid = nccl_unique_id() if rank == 0 else None
    uid = share_unique_id(uid, rank)
    buf = ctypes.create_string_buffer(uid, 128)
    comm = ctypes.c_void_p()
    _lib.check("ark_cuda_nccl_comm_init",
               _lib.lib().ark_cuda_nccl_comm_init(world, rank, buf, device, ctypes.byref(comm)))
    return comm.value


def nccl_comm_destroy(comm):
    if comm:
        _lib.check("ark_cuda_nccl_comm_destroy", _lib.lib().ark_cuda_nccl_comm_destroy(comm))
