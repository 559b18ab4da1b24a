"""Batch-row sharding across GPUs: one replica per GPU, no collective on the verify/accept path.

Every request's acceptance, attention, Markov rows and ctx_store are independent of every other request's, so a
batch splits by rows: rank r of N serves rows shard_rows(total, N, r).  torch.distributed (NCCL on GPUs, gloo on
CPU) carries only the plumbing around it: a barrier before and after timed regions and the max / sum of
per-rank numbers.
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def shard_rows(total: int, world: int, rank: int) -> range:
    """Rows of `total` served by `rank` of `world`: contiguous, sizes differing by at most one."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def _device() -> torch.device:
    if dist.is_initialized() and dist.get_backend() == "nccl":
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device("cpu")


def reduce_scalar(value: float, op: str) -> float:
    """value reduced over all ranks ("max" or "sum"); the value itself without a process group."""
    if not dist.is_initialized():
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=_device())
    dist.all_reduce(t, op={"max": dist.ReduceOp.MAX, "sum": dist.ReduceOp.SUM}[op])
    return float(t.item())


def barrier() -> None:
    if torch.cuda.is_available() and torch.cuda.is_initialized():
        torch.cuda.synchronize()
    if dist.is_initialized():
        dist.barrier()
    if torch.cuda.is_available() and torch.cuda.is_initialized():
        torch.cuda.synchronize()
