"""Request sharding across the GPUs of one box (one process per GPU).

Banks of different requests never interact, so requests are partitioned
across ranks and each rank owns its pools, its free stacks and a replica of
the shared initial memory: decode has no collective.  The only collective is
off the data path: reducing a timing (or a counter) to its max / sum over ranks.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def shard_requests(total: int, world: int, rank: int) -> range:
    """Contiguous block of request ids owned by ``rank`` (sizes differ by at most one)."""
    if world <= 0 or not 0 <= rank < world or total < 0:
        raise ValueError("invalid shard request")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def least_loaded(loads: list[int]) -> int:
    """Rank that should admit the next request (fewest live requests, lowest rank on ties)."""
    return min(range(len(loads)), key=lambda r: (loads[r], r))


def reduce_over_ranks(values: list[float], op: str = "max", device: torch.device | None = None) -> list[float]:
    """Element-wise max or sum of host floats over all ranks (identity without a process group)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return list(values)
    backend = dist.get_backend()
    dev = device if device is not None else (
        torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu"))
    t = torch.tensor(values, dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX if op == "max" else dist.ReduceOp.SUM)
    return t.cpu().tolist()
