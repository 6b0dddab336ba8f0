"""The multi-GPU host path on CPU: two gloo ranks shard a batch of positions
with no data-path collective, each encodes its own share, and the timing
reduce is the maximum over ranks. Together the shards are the whole batch."""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as tmp

from golden_io import mb


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank: int, world: int, port: int, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=60))
    try:
        specs = mb.engine.random_positions(7, 5, 40, seed=11)
        a, b = mb.sharding.shard_bounds(len(specs), rank, world)
        batch = mb.encoder.encode(specs[a:b], threads=1)
        cells = torch.tensor([batch.n_cells], dtype=torch.int64)
        gathered = [torch.zeros(1, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(gathered, cells)  # test bookkeeping only; the data path has no collective
        slowest = mb.sharding.max_over_ranks(1.5 + rank)
        out.put((rank, a, b, [int(g) for g in gathered], slowest))
    finally:
        dist.destroy_process_group()


def test_shard_bounds_cover_in_order():
    for n in (0, 1, 7, 4096):
        for world in (1, 2, 3, 8):
            spans = [mb.sharding.shard_bounds(n, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(spans[i][1] == spans[i + 1][0] for i in range(world - 1))
            assert max(b - a for a, b in spans) - min(b - a for a, b in spans) <= 1
    with pytest.raises(ValueError):
        mb.sharding.shard_bounds(4, 2, 2)


def test_two_gloo_ranks_shard_and_reduce():
    if not mb._lib.LIB_PATH.exists():
        pytest.skip("library not built")
    ctx = tmp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    specs = mb.engine.random_positions(7, 5, 40, seed=11)
    whole = mb.encoder.encode(specs, threads=1)
    (r0, a0, b0, cells0, m0), (r1, a1, b1, cells1, m1) = res
    assert (a0, b0, a1, b1) == (0, 4, 4, 7)
    assert cells0 == cells1 and sum(cells0) == whole.n_cells
    assert m0 == m1 == 2.5
