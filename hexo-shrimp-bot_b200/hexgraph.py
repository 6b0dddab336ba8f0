"""Cell-token graphs of the isolated-op workloads: the hex message-passing op
(neighbour table over cell tokens) and the axial-bias attention op (token
coordinates and valid lengths).

A position's cell tokens are its occupied cells plus the empty cells within
hex distance ``radius`` of a stone, in ascending (q, r) order. Neighbour slot
order follows the reference adjacency walk (builder.py:458-471): for each
engine axis Q, R, QR (builder.py:32) the step -1 then the step +1, so slot
2 * axis + (sign > 0). A slot holds the global token row of that neighbour,
or -1 when the neighbour cell is not a token. Rows past a position's token
count (padding) have every slot -1.
"""

from __future__ import annotations

import numpy as np

from .engine import random_positions
from .vocab import AXES

SLOTS = 6
# (6, 2) unit steps in slot order: axis 0 (-, +), axis 1 (-, +), axis 2 (-, +)
SLOT_STEPS = np.stack([s * AXES[a] for a in range(3) for s in (-1, 1)]).astype(np.int64)


def _pack(qr: np.ndarray) -> np.ndarray:
    """Order-preserving int64 key of (q, r) pairs (|q|, |r| < 2**20)."""
    return (qr[..., 0] + (1 << 20)) * (1 << 21) + (qr[..., 1] + (1 << 20))


def cell_tokens(stone_qr: np.ndarray, radius: int = 2) -> np.ndarray:
    """(n, 2) int64 token coordinates in ascending (q, r): the stones and
    every cell within hex distance ``radius`` of one."""
    offs = np.array([(dq, dr) for dq in range(-radius, radius + 1) for dr in range(-radius, radius + 1)
                     if max(abs(dq), abs(dr), abs(dq + dr)) <= radius], dtype=np.int64)
    cells = (stone_qr[:, None, :] + offs[None, :, :]).reshape(-1, 2)
    keys = np.unique(_pack(cells))  # sorted, unique
    q = keys // (1 << 21) - (1 << 20)
    r = keys % (1 << 21) - (1 << 20)
    return np.stack([q, r], 1)


def neighbour_table(tokens: np.ndarray, length: int, row0: int = 0) -> np.ndarray:
    """(length, 6) int32 neighbour rows for the first ``length`` tokens (the
    rest padding), offset by ``row0``."""
    n = min(len(tokens), length)
    kept = tokens[:n]
    keys = _pack(kept)  # ascending because the tokens are
    out = np.full((length, SLOTS), -1, dtype=np.int32)
    if n:
        nb = _pack(kept[:, None, :] + SLOT_STEPS[None, :, :])  # (n, 6)
        pos = np.searchsorted(keys, nb)
        hit = (pos < n) & (keys[np.minimum(pos, n - 1)] == nb)
        out[:n] = np.where(hit, pos + row0, -1).astype(np.int32)
    return out


def message_graph(n_pos: int, length: int = 256, lo: int = 40, hi: int = 200, seed: int = 0):
    """The message-passing workload's table: ``n_pos`` seeded random-play
    positions (``lo``-``hi`` stones), ``length`` token rows each (tokens at
    hex distance <= 2, truncated or padded). Returns (nbr (n_pos*length, 6)
    int32, tokens per position)."""
    specs = random_positions(n_pos, lo, hi, seed=seed)
    tables, counts = [], []
    for i, s in enumerate(specs):
        tok = cell_tokens(s.stone_qr, 2)
        counts.append(min(len(tok), length))
        tables.append(neighbour_table(tok, length, i * length))
    return np.concatenate(tables), np.asarray(counts)


def attention_layout(n_pos: int, length: int = 256, lo: int = 10, hi: int = 40, seed: int = 0,
                     min_valid: int = 32):
    """The axial-attention workload's token coordinates and valid lengths:
    per position the first ``length`` tokens in ascending (q, r) of a seeded
    random-play position of ``lo``-``hi`` stones (token radius grown from 2
    until there are ``length`` of them), and a valid length uniform in
    [``min_valid``, ``length``]. Returns (coords (n_pos, length, 2) int32,
    valid (n_pos,) int32)."""
    specs = random_positions(n_pos, lo, hi, seed=seed)
    rng = np.random.default_rng(seed + 1)
    coords = np.zeros((n_pos, length, 2), dtype=np.int32)
    for i, s in enumerate(specs):
        radius = 2
        tok = cell_tokens(s.stone_qr, radius)
        while len(tok) < length:
            radius += 1
            tok = cell_tokens(s.stone_qr, radius)
        coords[i] = tok[:length]
    valid = rng.integers(min_valid, length + 1, size=n_pos).astype(np.int32)
    return coords, valid
