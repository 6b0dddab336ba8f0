"""Multi-GPU host logic: positions shard across ranks with no data-path
collective (each rank evaluates its own positions end to end), and timing is
reduced as the maximum over ranks.

The reference evaluates on one device under a lock (klent/train.py:85, 106);
positions are independent, so N processes, one per GPU, each take a
contiguous slice of a batch (or their own positions, as the benchmark does)
and the only cross-rank traffic is the timing barrier and reduce.
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def shard_bounds(n_total: int, rank: int, world: int) -> tuple[int, int]:
    """[start, stop) of rank's contiguous share of ``n_total`` positions: the
    first ``n_total % world`` ranks take one more."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    if n_total < 0:
        raise ValueError("n_total must be >= 0")
    base, extra = divmod(n_total, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def max_over_ranks(x: float, device=None) -> float:
    """The largest ``x`` over the process group (``x`` itself when no group
    is initialised or it has one rank). ``device``: where the reduce runs
    (a CUDA device under NCCL; CPU under gloo)."""
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size() == 1:
        return float(x)
    t = torch.tensor([float(x)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
