"""The Gumbel search's host logic on the CPU: the halving schedule
(reference klent/search.py:47-76 cases) and the engine methods the search
relies on."""

from __future__ import annotations

import pytest

from golden_io import mb

search = mb.search
eng = mb.engine


def test_halving_schedule():
    assert search.halving_schedule(32, 16) == [(16, 1), (8, 2)]
    assert search.halving_schedule(0, 4) == []
    assert search.halving_schedule(7, 1) == [(1, 7)]
    plan = search.halving_schedule(200, 16)
    assert sum(n * d for n, d in plan) <= 200 and plan[0] == (16, 1) and plan[1][1] == 2
    assert search.halving_schedule(3, 4) == []
    with pytest.raises(ValueError):
        search.halving_schedule(-1, 4)
    with pytest.raises(ValueError):
        search.halving_schedule(8, 0)


def test_position_copy_replay_and_ranks():
    root = eng.Position.replay([(0, 0)])
    assert len(root.legal_moves()) == 216 and root.nth_legal(0) == (-8, 0) and root.nth_legal(3) == (-8, 3)
    child = root.copy()
    child.advance(-8, 3)
    assert root.ply == 1 and child.ply == 2 and (-8, 3) in root.legal_moves()
    assert child.current_player == 1 and child.moves_remaining == 1
    # six in a row ends the game with a winner
    p = eng.Position.replay([(0, 0), (0, 5), (0, 6), (1, 0), (2, 0), (0, 7), (0, 8), (3, 0), (4, 0), (0, 9), (-1, 9)])
    assert not p.is_terminal
    p.advance(5, 0)
    assert p.is_terminal and p.winner == 0


def test_chooser_argument_checks():
    with pytest.raises(ValueError):
        search.gumbel_choose(None, 1.0, 0.0, -1)
    with pytest.raises(ValueError):
        search.gumbel_choose(None, 1.0, 0.0, 0, temperature=0.5)
    with pytest.raises(ValueError):
        search.gumbel_choose(None, 1.0, 0.0, 8, temperature=float("nan"))
