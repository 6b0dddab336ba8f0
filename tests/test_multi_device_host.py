"""Host logic of the multi-device evaluator (CPU): cost-balanced contiguous
slices, concurrent slice runs assembled in position order, and the fault
model of a lost worker (its slice is re-queued on a live worker, the worker
is left out of later calls). Failures are raised on the host by fake
workers; no device is involved."""

from __future__ import annotations

import threading

import numpy as np
import pytest

from golden_io import mb

S = mb.sharding


def test_position_costs():
    c = S.position_costs([3, 0, 5], [2, 1, 0], [10, 0, 4])
    assert c.tolist() == [15, 1, 9]
    assert S.position_costs([1, 2], [0, 0]).tolist() == [1, 2]
    with pytest.raises(ValueError):
        S.position_costs([1, -4], [0, 0])


@pytest.mark.parametrize("n", [1, 2, 3, 8])
@pytest.mark.parametrize("seed", [0, 1, 2])
def test_balanced_cuts_cover_in_order_and_balance(n, seed):
    rng = np.random.default_rng(seed)
    costs = rng.integers(1, 500, size=int(rng.integers(0, 60)))
    cuts = S.balanced_cuts(costs, n)
    assert len(cuts) == n + 1 and cuts[0] == 0 and cuts[-1] == len(costs)
    assert all(a <= b for a, b in zip(cuts, cuts[1:]))
    if len(costs):
        loads = [int(costs[a:b].sum()) for a, b in zip(cuts, cuts[1:])]
        # each boundary lies within half a position of its ideal point
        assert max(loads) <= costs.sum() / n + costs.max()


def test_balanced_cuts_edge_cases():
    assert S.balanced_cuts([], 3) == [0, 0, 0, 0]
    assert S.balanced_cuts([7], 1) == [0, 1]
    assert S.balanced_cuts([5, 5, 5, 5], 2) == [0, 2, 4]
    assert S.balanced_cuts([1, 1, 1, 10], 2) == [0, 3, 4]
    with pytest.raises(ValueError):
        S.balanced_cuts([1], 0)


class _Worker:
    def __init__(self, name, fail_times=0):
        self.name, self.fail_times, self.ran = name, fail_times, []

    def run(self, out, p0, p1):
        if self.fail_times:
            self.fail_times -= 1
            raise RuntimeError(f"{self.name} lost")
        self.ran.append((p0, p1))
        out[p0:p1] = np.arange(p0, p1) * 10


def _go(workers, cuts, lost):
    out = np.full(cuts[-1], -1)
    S.run_slices(cuts, workers, lambda w, a, b: w.run(out, a, b), lost)
    return out


def test_slices_assemble_in_position_order():
    ws = [_Worker(f"w{i}") for i in range(3)]
    lost = set()
    out = _go(ws, [0, 4, 4, 9], lost)
    assert out.tolist() == [10 * i for i in range(9)] and not lost
    assert ws[0].ran == [(0, 4)] and ws[1].ran == [] and ws[2].ran == [(4, 9)]  # empty slices are skipped


def test_slices_run_concurrently():
    barrier = threading.Barrier(3, timeout=10)
    seen = []

    def run(w, a, b):
        barrier.wait()  # passes only when all three slices are in flight at once
        seen.append(w)

    S.run_slices([0, 1, 2, 3], ["a", "b", "c"], run, set())
    assert sorted(seen) == ["a", "b", "c"]


def test_lost_worker_requeues_its_slice():
    ws = [_Worker("w0"), _Worker("w1", fail_times=1), _Worker("w2")]
    lost = set()
    out = _go(ws, [0, 3, 6, 9], lost)
    assert out.tolist() == [10 * i for i in range(9)]
    assert lost == {1}
    assert (3, 6) in ws[0].ran and ws[1].ran == []
    # the lost worker stays out: the next call has two slices for two workers
    with pytest.raises(ValueError):
        _go(ws, [0, 3, 6, 9], lost)
    out = _go(ws, [0, 5, 9], lost)
    assert out.tolist() == [10 * i for i in range(9)] and ws[1].ran == []


def test_requeue_moves_on_until_a_worker_survives():
    ws = [_Worker("w0", fail_times=5), _Worker("w1", fail_times=5), _Worker("w2")]
    lost = set()
    out = _go(ws, [0, 2, 5, 9], lost)
    assert out.tolist() == [10 * i for i in range(9)]
    assert lost == {0, 1} and sorted(ws[2].ran) == [(0, 2), (2, 5), (5, 9)]


def test_every_worker_lost_raises():
    ws = [_Worker("w0", fail_times=9), _Worker("w1", fail_times=9)]
    lost = set()
    with pytest.raises(S.WorkerLost, match="all 2 workers failed"):
        _go(ws, [0, 2, 4], lost)
    assert lost == {0, 1}
