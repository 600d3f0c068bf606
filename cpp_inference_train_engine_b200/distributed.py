"""Data-parallel plumbing of the GRPO step: one process (rank) per GPU.

The rollout groups of a step are split evenly over the ranks, whole groups per rank
(``rollout_shard``), so group advantages stay local and a rank's rollout i is global rollout
``rank * R + i``. Every rank runs its own rollouts, teacher-forced passes and backward; the
engine divides each token's coefficient by the global rollout count, sums gradients and the
loss/KL scalars with an NCCL all-reduce over NVLink and ORs the "any non-zero advantage" flag
before the replicated AdamW (the reference's single-process update, trainer.cpp:784-891, with
its gradient sum split over ranks). torch.distributed carries only the bootstrap: the NCCL
unique id is broadcast from rank 0 (``init_comm``).
"""
from __future__ import annotations


def rollout_shard(n_rollouts: int, group: int, rank: int, world: int) -> slice:
    """Rollouts [rank * R, (rank + 1) * R) with R = n_rollouts / world, whole groups only."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    if group < 1 or n_rollouts % group:
        raise ValueError("rollouts must form whole groups")
    if n_rollouts % world or (n_rollouts // world) % group:
        raise ValueError("rollouts must split into whole groups per rank")
    R = n_rollouts // world
    return slice(rank * R, (rank + 1) * R)


def broadcast_unique_id(rank: int, make_id, process_group=None) -> bytes:
    """Rank 0 creates the id with ``make_id()``; every rank returns the same bytes."""
    import torch.distributed as dist
    box = [make_id() if rank == 0 else None]
    dist.broadcast_object_list(box, src=0, group=process_group)
    uid = box[0]
    if not isinstance(uid, (bytes, bytearray)) or len(uid) != 128:
        raise RuntimeError("NCCL unique id broadcast failed")
    return bytes(uid)


def init_comm(execution, rank: int, world: int, process_group=None) -> None:
    """Bootstrap the execution's NCCL communicator (mm_cuda_init_comm) over torch.distributed."""
    from .engine import CudaExecution
    uid = broadcast_unique_id(rank, CudaExecution.nccl_unique_id, process_group)
    execution.init_comm(rank, world, uid)
