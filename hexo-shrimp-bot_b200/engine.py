"""Hexo rules, restated only as far as position generation needs them.

Facts followed (crates/hexo-engine/README.md:8-13, 45-50, 111-115;
crates/hexo-engine/src/coord.rs:7; python/hexo-py/src/lib.rs:146-153):

- P0 opens at the origin; afterwards each player places two stones per turn
  (P0; P1 P1; P0 P0; ...).
- A placement is legal when the cell is empty and within 8 hex steps of a stone;
  legal moves are listed in ascending (q, r) order.
- Six or more in a row on one axis wins, checked after every placement.
- ``moves_remaining`` is 2 before the first stone of a normal turn and 1 before
  the second stone or the opening stone.

Seeded uniform-random playouts that end non-terminal stand in for the
reference's engine-replay fixtures (python/mantisnet/tests/conftest.py:64-86).
"""

from __future__ import annotations

import random
from dataclasses import dataclass

import numpy as np

from .vocab import AXES, LEGAL_RADIUS

DISK = [
    (dq, dr)
    for dq in range(-LEGAL_RADIUS, LEGAL_RADIUS + 1)
    for dr in range(-LEGAL_RADIUS, LEGAL_RADIUS + 1)
    if max(abs(dq), abs(dr), abs(dq + dr)) <= LEGAL_RADIUS
]
assert len(DISK) == 217


def mover_at(ply: int) -> int:
    """Player to place stone number ``ply`` (0-based)."""
    if ply == 0:
        return 0
    return 1 if ((ply - 1) // 2) % 2 == 0 else 0


def moves_remaining_at(ply: int) -> int:
    if ply == 0:
        return 1
    return 2 if ply % 2 == 1 else 1


@dataclass(frozen=True)
class PositionSpec:
    """The builder's input list for one position (§11 of the model spec)."""

    stone_qr: np.ndarray  # (n_s, 2) int64, ascending (q, r)
    stone_owner: np.ndarray  # (n_s,) int64 in {0, 1}
    mover: int
    legal_qr: np.ndarray  # (n_legal, 2) int64, ascending (q, r)
    moves_remaining: int


class Position:
    """Mutable game state with an incrementally maintained legal frontier."""

    def __init__(self) -> None:
        self.board: dict[tuple[int, int], int] = {}
        self.ply = 0
        self.terminal = False
        self.winner = None
        # Frontier as an indexable list with positions, for O(1) random choice.
        self._front: list[tuple[int, int]] = [(0, 0)]
        self._where: dict[tuple[int, int], int] = {(0, 0): 0}

    @classmethod
    def replay(cls, moves) -> "Position":
        """The position after placing ``moves`` ((q, r) pairs) in order."""
        pos = cls()
        for q, r in moves:
            pos.advance(int(q), int(r))
        return pos

    def copy(self) -> "Position":
        other = Position.__new__(Position)
        other.board = dict(self.board)
        other.ply = self.ply
        other.terminal = self.terminal
        other.winner = getattr(self, "winner", None)
        other._front = list(self._front)
        other._where = dict(self._where)
        return other

    @property
    def is_terminal(self) -> bool:
        return self.terminal

    def nth_legal(self, rank: int) -> tuple[int, int]:
        """The legal move of index ``rank`` in engine order (ascending (q, r))."""
        return self.legal_moves()[rank]

    @property
    def current_player(self) -> int:
        return mover_at(self.ply)

    @property
    def moves_remaining(self) -> int:
        return moves_remaining_at(self.ply)

    def legal_moves(self) -> list[tuple[int, int]]:
        if self.terminal:
            return []
        return sorted(self._front)

    def _drop(self, cell) -> None:
        i = self._where.pop(cell)
        last = self._front.pop()
        if i < len(self._front):
            self._front[i] = last
            self._where[last] = i

    def _wins(self, q: int, r: int, who: int) -> bool:
        for dq, dr in AXES.tolist():
            run = 1
            for sign in (1, -1):
                k = 1
                while self.board.get((q + sign * k * dq, r + sign * k * dr)) == who:
                    run += 1
                    k += 1
            if run >= 6:
                return True
        return False

    def advance(self, q: int, r: int) -> None:
        cell = (q, r)
        if self.terminal or cell not in self._where:
            raise ValueError(f"illegal placement {cell}")
        who = self.current_player
        if self.ply == 0:
            self._front.clear()
            self._where.clear()
        else:
            self._drop(cell)
        self.board[cell] = who
        for dq, dr in DISK:
            c = (q + dq, r + dr)
            if c not in self.board and c not in self._where:
                self._where[c] = len(self._front)
                self._front.append(c)
        self.ply += 1
        if self._wins(q, r, who):
            self.terminal = True
            self.winner = who

    def random_legal(self, rng: random.Random) -> tuple[int, int]:
        return self._front[rng.randrange(len(self._front))]

    def spec(self) -> PositionSpec:
        if self.board:
            cells = sorted(self.board)
            qr = np.asarray(cells, dtype=np.int64)
            owner = np.asarray([self.board[c] for c in cells], dtype=np.int64)
        else:
            qr = np.empty((0, 2), dtype=np.int64)
            owner = np.empty(0, dtype=np.int64)
        legal = np.asarray(self.legal_moves(), dtype=np.int64).reshape(-1, 2)
        return PositionSpec(qr, owner, self.current_player, legal, self.moves_remaining)


def random_game(plies: int, seed: int, snapshot_at=None) -> list[PositionSpec]:
    """Play ``plies`` uniform-random placements that leave the game
    non-terminal; return the position specs at ``snapshot_at`` plies (default:
    the final position). Terminal playouts are retried with a new stream."""
    want = sorted(snapshot_at) if snapshot_at is not None else [plies]
    for attempt in range(100):
        rng = random.Random(seed * 1_000_003 + attempt * 1_009 + plies)
        pos = Position()
        out = []
        ok = True
        for ply in range(plies + 1):
            hits = want.count(ply)
            if hits:
                spec = pos.spec()
                out.extend([spec] * hits)
            if ply == plies:
                break
            pos.advance(*pos.random_legal(rng))
            if pos.terminal:
                ok = False
                break
        if ok:
            return out
    raise RuntimeError(f"no non-terminal {plies}-ply playout in 100 attempts")


def random_positions(n: int, lo: int, hi: int, seed: int, per_game: int = 8) -> list[PositionSpec]:
    """``n`` positions with stone counts uniform in [lo, hi], taken as move
    prefixes of seeded random games (``per_game`` prefixes per game)."""
    rng = np.random.default_rng(seed)
    out: list[PositionSpec] = []
    game = 0
    while len(out) < n:
        k = min(per_game, n - len(out))
        plies = sorted(int(x) for x in rng.integers(lo, hi + 1, size=k))
        out.extend(random_game(plies[-1], seed=seed * 7919 + game, snapshot_at=plies))
        game += 1
    return out[:n]
