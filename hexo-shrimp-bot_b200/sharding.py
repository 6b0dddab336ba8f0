"""Multi-GPU host logic. Positions are independent (attention is
block-diagonal, message passing never crosses positions), so a batch shards
by positions with no data-path collective:

- across processes, one per GPU: each rank takes a contiguous share of the
  positions (``shard_bounds``) and timing is reduced as the maximum over
  ranks (``max_over_ranks``);
- across the GPUs of one process (one evaluator call spanning several
  devices): the batch is cut into contiguous slices balanced by a cost
  model, per position cells + windows + radius edges (``position_costs``,
  ``balanced_cuts``); every slice runs on its own device and writes its
  rows of one host output; a slice whose worker fails is re-run on a worker
  still alive, and the failed worker is left out of later calls
  (``run_slices``).

The reference evaluates on one device under a lock (klent/train.py:85, 106).
"""

from __future__ import annotations

import threading
from concurrent.futures import ThreadPoolExecutor

import numpy as np
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


def position_costs(n_cells: np.ndarray, n_windows: np.ndarray, n_radius_edges: np.ndarray | None = None) -> np.ndarray:
    """Per-position cost of an evaluation: cells + windows + radius edges
    (the rows and edges the dominant kernels stream)."""
    c = np.asarray(n_cells, dtype=np.int64) + np.asarray(n_windows, dtype=np.int64)
    if n_radius_edges is not None:
        c = c + np.asarray(n_radius_edges, dtype=np.int64)
    if c.ndim != 1 or (c.size and c.min() < 0):
        raise ValueError("position costs must be a 1-D array of counts >= 0")
    return c


def balanced_cuts(costs: np.ndarray, n: int) -> list[int]:
    """``n + 1`` position boundaries of ``n`` contiguous slices whose summed
    costs are as even as contiguous cuts allow: boundary k is the prefix
    point nearest to k / n of the total (ties to the earlier point). Slices
    may be empty (fewer positions than slices, or one position outweighing
    the rest)."""
    if n < 1:
        raise ValueError(f"need at least one slice (got {n})")
    costs = np.asarray(costs, dtype=np.int64)
    prefix = np.concatenate([[0], np.cumsum(costs)])
    total, p = int(prefix[-1]), len(costs)
    cuts = [0]
    for k in range(1, n):
        target = total * k / n
        j = int(np.searchsorted(prefix, target, side="left"))
        j = min(max(j, 1), p) if p else 0
        if j > 0 and target - prefix[j - 1] <= prefix[j] - target:
            j -= 1
        cuts.append(max(j, cuts[-1]))
    cuts.append(p)
    return cuts


class WorkerLost(RuntimeError):
    """Every worker of a multi-device evaluator has failed."""


def run_slices(cuts: list[int], workers: list, run, lost: set, pool: ThreadPoolExecutor | None = None) -> None:
    """Run slice k = positions [cuts[k], cuts[k + 1]) as ``run(worker, p0,
    p1)`` on the k-th worker not in ``lost``, all slices concurrently. A slice
    whose run raises is re-queued on the next live worker (in index order,
    after the others finish) and its first worker's index joins ``lost``.
    Raises ``WorkerLost`` (from the last failure) when no live worker is
    left. ``len(cuts) - 1`` must not exceed the live worker count."""
    alive = [i for i in range(len(workers)) if i not in lost]
    slices = [(cuts[k], cuts[k + 1]) for k in range(len(cuts) - 1)]
    if len(slices) > len(alive):
        raise ValueError(f"{len(slices)} slices for {len(alive)} live workers")
    own = pool is None
    pool = pool or ThreadPoolExecutor(max(1, len(alive)))
    try:
        pending = [(s, alive[k]) for k, s in enumerate(slices) if s[1] > s[0]]
        last_exc = None
        while pending:
            futures = [(s, w, pool.submit(run, workers[w], *s)) for s, w in pending]
            failed = []
            for s, w, f in futures:
                try:
                    f.result()
                except Exception as exc:  # the worker is lost; its slice is re-queued
                    lost.add(w)
                    failed.append(s)
                    last_exc = exc
            live = [i for i in range(len(workers)) if i not in lost]
            if failed and not live:
                raise WorkerLost(f"all {len(workers)} workers failed; last error: {last_exc}") from last_exc
            pending = [(s, live[k % len(live)]) for k, s in enumerate(failed)]
    finally:
        if own:
            pool.shutdown(wait=True)
