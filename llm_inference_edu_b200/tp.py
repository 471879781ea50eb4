"""Tensor-parallel plumbing: one process per GPU, the model sharded by
attention heads and FFN columns (``Decoder(..., tp=(rank, size))``), the
ranks' exchange buffers opened through CUDA IPC (``TpComm``).  The
handles travel over any host channel; here torch.distributed (gloo or
NCCL) gathers them.  The data path itself uses no library collective."""
from __future__ import annotations


def connect(comm, rank: int, size: int, group=None) -> None:
    """Gathers every rank's communicator handle (torch.distributed, rank
    order) and opens the peers' buffers.  A single rank needs no channel."""
    if size == 1:
        comm.connect(rank, [comm.handle()])
        return
    import torch.distributed as dist
    handles = [None] * size
    dist.all_gather_object(handles, comm.handle(), group=group)
    comm.connect(rank, handles)


def batch(model, comm_rows: int, sequences: int, capacity: int, kv_dtype: str, rank: int, size: int,
          group=None):
    """A BatchSession over this rank's shard with a connected communicator
    of `comm_rows` rows (at least max(sequences, 256))."""
    from . import api
    comm = api.TpComm(model.device, comm_rows, model.config.hidden_dim)
    connect(comm, rank, size, group)
    return api.BatchSession(model, sequences, capacity, kv_dtype=kv_dtype, comm=comm)
