"""Data-parallel plumbing for independent sequences (one process per GPU).

Batch-1 decode of independent sequences shards by sequence: every rank holds
the whole model and decodes its own prompts; ranks exchange nothing on the
data path.  Only measurement crosses ranks: a barrier before each timed
region and the maximum of the per-rank device times after it.

Launch: ``python -m torch.distributed.run --nproc-per-node N ...`` (RANK,
LOCAL_RANK, WORLD_SIZE and MASTER_* from the environment).
"""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass


@dataclass(frozen=True)
class Topology:
    rank: int
    world: int
    local_rank: int

    @property
    def distributed(self) -> bool:
        return self.world > 1


def topology_from_env() -> Topology:
    """Rank, world size and local rank from the torchrun environment
    (a single process when the variables are absent)."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", str(rank)))
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"inconsistent distributed environment: rank {rank} of {world}")
    return Topology(rank, world, local_rank)


def init(topo: Topology, backend: str = "nccl", timeout_s: float = 120.0) -> None:
    """Joins the process group (no-op for one process).  The short timeout
    turns a missing or failed rank into an error instead of a hang."""
    if not topo.distributed:
        return
    import torch.distributed as dist
    if backend == "nccl":
        import torch
        torch.cuda.set_device(topo.local_rank)
    dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s),
                            rank=topo.rank, world_size=topo.world)


def shutdown(topo: Topology) -> None:
    if topo.distributed:
        import torch.distributed as dist
        if dist.is_initialized():
            dist.destroy_process_group()


def sequence_ids(topo: Topology, sequences: int) -> list:
    """The global sequence indices this rank decodes: a contiguous block of
    ceil(sequences / world) (the last ranks may get fewer or none)."""
    if sequences < 0:
        raise ValueError("sequences must be non-negative")
    per = -(-sequences // topo.world)
    lo = min(sequences, topo.rank * per)
    return list(range(lo, min(sequences, lo + per)))


def barrier(topo: Topology) -> None:
    if topo.distributed:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(topo: Topology, value: float, device=None) -> float:
    """The maximum of `value` over all ranks (every rank gets it)."""
    if not topo.distributed:
        return float(value)
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
