"""Positions to graphs, graphs to batches (host side, numpy).

This is the drop-in for the reference builder's public surface
(python/mantisnet/mantisnet/builder.py): ``build`` (486-642), ``collate``
(881-956), ``Batch`` (666-752), ``batch_from_arrays`` (778-811) and the relay
views (relay.py:48-94). Every emitted array — order included — is part of the
representation contract and is checked bit-exact against fixtures produced by
the reference builder.

The construction is vectorised differently from the reference (neighbour
disks are enumerated from the stones, lookups go through sorted packed keys),
but each output follows the reference's ordering rules:

- windows: ascending packed (start_q, start_r, axis) key;
- incidence: window-major, slot-minor;
- decoder rows and action rows: legal-cell-major, then axis, then offset k;
- radius edges: destination cell-major, source stone-minor;
- adjacency: sorted (destination, source, axis) triples.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from .vocab import (
    ACTION_EMPTY,
    ACTION_EMPTY_ORBITS,
    ACTION_MIXED,
    ACTION_OPP,
    ACTION_OWN,
    ACTION_SLOT_ORBIT,
    AXES,
    CELL_NEAREST_UNREACHED,
    GLOBAL_ROWS,
    GLOBAL_THREAT_CAP,
    LEGAL_RADIUS,
    ORBIT48_TABLE,
    ORBIT_SPAN,
    POW3,
    TACTICAL_FEATURES,
    TERN_DEC_CLASS,
    TERN_DEC_CLASSES,
    TERN_OCC_CLASS,
    TERN_POST1_CLASS,
    TERN_RANK,
    WINDOW_LEN,
)

_QSHIFT = 1 << 21


def _pack(qr: np.ndarray) -> np.ndarray:
    """(n, 2) axial coordinates to order-preserving int64 keys."""
    return qr[..., 0] * _QSHIFT + qr[..., 1]


def _lookup(sorted_keys: np.ndarray, keys: np.ndarray) -> np.ndarray:
    """Index of each key in ``sorted_keys`` or -1."""
    if len(sorted_keys) == 0:
        return np.full(keys.shape, -1, dtype=np.int64)
    pos = np.searchsorted(sorted_keys, keys)
    pos = np.minimum(pos, len(sorted_keys) - 1)
    return np.where(sorted_keys[pos] == keys, pos, -1)


_MSG_REACH = "every legal cell must be empty and at most 8 steps from a stone"

# Offsets of the radius-8 disk without its centre, for stone -> cell edges.
_DISK = np.array(
    [
        (dq, dr)
        for dq in range(-LEGAL_RADIUS, LEGAL_RADIUS + 1)
        for dr in range(-LEGAL_RADIUS, LEGAL_RADIUS + 1)
        if 1 <= max(abs(dq), abs(dr), abs(dq + dr)) <= LEGAL_RADIUS
    ],
    dtype=np.int64,
)
_DISK_DIST = np.maximum.reduce([np.abs(_DISK[:, 0]), np.abs(_DISK[:, 1]), np.abs(_DISK.sum(1))])
_DISK_ORBIT = ORBIT48_TABLE[_DISK[:, 0] + ORBIT_SPAN, _DISK[:, 1] + ORBIT_SPAN]
_DISK_ON_AXIS = (
    (_DISK[:, 0] == 0) | (_DISK[:, 1] == 0) | (_DISK[:, 0] + _DISK[:, 1] == 0)
).astype(np.int64)


@dataclass(frozen=True)
class PositionGraph:
    """One position's entities and index tables (reference builder.py:244-289)."""

    stone_own: np.ndarray
    stone_qr: np.ndarray
    window_feat: np.ndarray
    window_id: np.ndarray
    inc_stone: np.ndarray
    inc_window: np.ndarray
    inc_class: np.ndarray
    n_legal: int
    cell_qr: np.ndarray
    cell_nearest: np.ndarray
    radius_src: np.ndarray
    radius_dst: np.ndarray
    radius_orbit: np.ndarray
    radius_own: np.ndarray
    radius_on_axis: np.ndarray
    adjacency_src: np.ndarray
    adjacency_dst: np.ndarray
    adjacency_axis: np.ndarray
    dec_cell: np.ndarray
    dec_window: np.ndarray
    dec_class: np.ndarray
    moves_remaining: int
    action_window_index: np.ndarray
    action_post1_class: np.ndarray
    action_pre_status: np.ndarray
    action_tactical: np.ndarray

    @property
    def n_stones(self) -> int:
        return len(self.stone_own)

    @property
    def n_windows(self) -> int:
        return len(self.window_feat)


def _cell_node_fields(stone_qr, stone_own, legal_qr, legal_key, legal_sorted, legal_rank):
    """Nearest-stone buckets, radius-8 stone->cell edges, and cell adjacency
    (reference builder.py:427-483)."""
    n_legal = len(legal_qr)
    empty = np.empty(0, dtype=np.int64)
    if len(stone_qr):
        cells = stone_qr[:, None, :] + _DISK[None, :, :]  # (n_s, 216, 2)
        hit = _lookup(legal_sorted, _pack(cells))  # index into sorted legal keys
        src, disk = np.nonzero(hit >= 0)
        dst = legal_rank[hit[src, disk]]
        order = np.lexsort((src, dst))  # destination-major, source-minor
        src, disk, dst = src[order], disk[order], dst[order]
        nearest = np.full(n_legal, LEGAL_RADIUS + 1, dtype=np.int64)
        np.minimum.at(nearest, dst, _DISK_DIST[disk])
        if np.any(nearest > LEGAL_RADIUS) or np.any(_lookup(np.sort(_pack(stone_qr)), legal_key) >= 0):
            raise ValueError(_MSG_REACH)
        # The displacement is cell - stone, which is the disk offset itself.
        radius = dict(
            radius_src=src.astype(np.int64),
            radius_dst=dst.astype(np.int64),
            radius_orbit=_DISK_ORBIT[disk],
            radius_own=stone_own[src],
            radius_on_axis=_DISK_ON_AXIS[disk],
        )
    else:
        nearest = np.full(n_legal, CELL_NEAREST_UNREACHED, dtype=np.int64)
        radius = dict(
            radius_src=empty, radius_dst=empty, radius_orbit=empty,
            radius_own=empty, radius_on_axis=empty,
        )

    # Directed distance-one neighbours among legal cells: (dst, src, axis).
    steps = np.concatenate([-AXES, AXES], axis=0)  # (6, 2): axis a at a and a+3
    step_axis = np.array([0, 1, 2, 0, 1, 2], dtype=np.int64)
    nb = _lookup(legal_sorted, _pack(legal_qr[:, None, :] + steps[None, :, :]))
    src, slot = np.nonzero(nb >= 0)
    if len(src):
        dst = legal_rank[nb[src, slot]]
        axis = step_axis[slot]
        order = np.lexsort((axis, src, dst))
        adj = dict(adjacency_src=src[order].astype(np.int64),
                   adjacency_dst=dst[order].astype(np.int64),
                   adjacency_axis=axis[order])
    else:
        adj = dict(adjacency_src=empty, adjacency_dst=empty, adjacency_axis=empty)
    return dict(cell_qr=legal_qr.copy(), cell_nearest=nearest, **radius, **adj)


# ---------------------------------------------------------------- windows
# Format of the window, decoder and action tables (the representation
# contract the checkpoints and the Rust bridge read):
#
# A window is six consecutive cells along one of the three line axes
# (``AXES``: Q, R, QR); slot j of the window (axis a, start s) is the cell
# s + j * AXES[a]. Each slot holds a ternary digit: 0 empty, 1 a stone of
# the player to move, 2 an opponent stone; the window's pattern is
# sum_j digit_j * 3**j. The live windows are those with at least one stone,
# listed by ascending key pack(s) * 4 + a. Each live window has an
# incidence row per occupied slot (window by window, slots ascending) with
# the class of (pattern, slot).
#
# Every legal cell c sits at slot k of the six windows of each axis that
# start k steps before it (k = 0..5): 18 candidate rows per cell, listed
# axis-major then k. A candidate whose window is live is a decoder row
# (class of (pattern, empty slot k)); every candidate also yields an action
# row: the pattern after the mover places a stone at slot k, its status
# (which players the window held before the placement) and the window's
# index when live (-1 otherwise). Eleven tactical scalars per cell summarise
# a cell's 18 candidates.

_SLOT = np.arange(WINDOW_LEN)
_REACH = WINDOW_LEN - 1  # a window through a cell spans 5 cells either side
# line offset of slot j in the window starting k cells before the centre
_WINDOW_AT = (_REACH - _SLOT)[:, None] + _SLOT[None, :]  # (k, j)

_MSG_TERMINAL = "terminal position: no legal move left to evaluate"
_MSG_DUPLICATE = "two stones occupy the same cell"
_MSG_OCCUPIED = "a legal cell holds a stone"


class _Board:
    """Stones by coordinate: the stone row at a cell and its ternary digit
    (0 empty, 1 the mover's stone, 2 an opponent stone)."""

    def __init__(self, stone_qr: np.ndarray, opponent: np.ndarray):
        key = _pack(stone_qr)
        self.order = np.argsort(key, kind="stable")
        self.keys = key[self.order]
        if len(self.keys) > 1 and np.any(self.keys[1:] == self.keys[:-1]):
            raise ValueError(_MSG_DUPLICATE)
        self.digit_of = 1 + opponent

    def rows_at(self, qr: np.ndarray) -> np.ndarray:
        hit = _lookup(self.keys, _pack(qr))
        if len(self.order) == 0:
            return hit
        return np.where(hit >= 0, self.order[np.maximum(hit, 0)], -1)

    def lines(self, centres: np.ndarray):
        """Stone rows and digits on the 11-cell line through each centre along
        each axis: arrays (n, 3, 11), offset o at line index o + 5."""
        offs = np.arange(-_REACH, _REACH + 1)
        qr = centres[:, None, None, :] + AXES[None, :, None, :] * offs[None, None, :, None]
        rows = self.rows_at(qr)
        digits = np.where(rows >= 0, self.digit_of[np.maximum(rows, 0)] if len(self.digit_of) else 0, 0)
        return rows, digits


def _live_windows(board: _Board, stone_qr: np.ndarray):
    """Every live window once, in key order: (axis, start (n, 2), pattern,
    stone row per slot (n, 6), -1 where empty).

    A window is enumerated from its lowest occupied slot only: the stone at
    line offset 0 is slot k of the window starting k cells before it, and it
    is that window's lowest stone when the k cells before it are empty."""
    n_s = len(stone_qr)
    rows, digits = board.lines(stone_qr)
    before = digits[:, :, :_REACH] == 0  # the five cells before the stone
    # clear[..., k]: the k cells right before the stone are empty
    suffix = np.flip(np.logical_and.accumulate(np.flip(before, -1), -1), -1)
    clear = np.concatenate([np.ones((n_s, 3, 1), bool), np.flip(suffix, -1)], axis=-1)
    stone, axis, k = np.nonzero(clear)
    start = stone_qr[stone] - AXES[axis] * k[:, None]
    slots = rows[stone, axis][np.arange(len(k))[:, None], _WINDOW_AT[k]]
    pattern = (digits[stone, axis][np.arange(len(k))[:, None], _WINDOW_AT[k]] * POW3).sum(1)
    key = _pack(start) * 4 + axis
    by_key = np.argsort(key, kind="stable")
    return axis[by_key].astype(np.int64), start[by_key], pattern[by_key], slots[by_key], key[by_key]


# tactical scalar columns (the checkpoint reads them in this order)
(_T_WIN_NOW, _T_OWN_BEST, _T_OPP_BEST, _T_MAKE_FIVE, _T_MAKE_FOUR, _T_BLOCK_FIVE, _T_BLOCK_FOUR,
 _T_FIVES_LEFT, _T_FOURS_LEFT, _T_BLOCKS_ALL_FIVES, _T_LIVE_ROWS) = range(TACTICAL_FEATURES)


def _cell_rows(board: _Board, legal_qr: np.ndarray, win_key: np.ndarray, win_pattern: np.ndarray):
    """Decoder rows and action rows of every legal cell's 18 candidates, and
    the cells' tactical scalars."""
    n_c = len(legal_qr)
    _, digits = board.lines(legal_qr)
    if np.any(digits[:, :, _REACH] != 0):
        raise ValueError(_MSG_OCCUPIED)
    cand = digits[:, :, _WINDOW_AT]  # (n_c, 3, k, j): digits of the window starting k before the cell
    before = (cand * POW3).sum(-1)  # pattern before the placement
    mine = (cand == 1).sum(-1)
    theirs = (cand == 2).sum(-1)
    live = (mine + theirs) > 0
    start = legal_qr[:, None, None, :] - AXES[None, :, None, :] * _SLOT[None, None, :, None]
    window = np.where(live, _lookup(win_key, _pack(start) * 4 + np.arange(3)[None, :, None]), -1)
    if np.any((window >= 0) != live):
        raise ValueError("internal: a window through a stone is missing from the live set")
    status = np.select([live & (theirs == 0), live & (mine == 0), live], [ACTION_OWN, ACTION_OPP, ACTION_MIXED],
                       ACTION_EMPTY)
    placed = TERN_POST1_CLASS[before + POW3[None, None, :], _SLOT[None, None, :]]

    cell, axis, k = np.nonzero(live)  # cell-major, then axis, then k
    dec_window = window[cell, axis, k]
    dec_class = TERN_DEC_CLASS[win_pattern[dec_window], k]

    # tactical scalars
    f32 = np.float32
    per_cell = (1, 2)
    n_rows = f32(3 * WINDOW_LEN)
    clean = theirs == 0
    blocks_five = live & (mine == 0) & (theirs == WINDOW_LEN - 1)
    blocks_four = live & (mine == 0) & (theirs == WINDOW_LEN - 2)
    fives_left = np.unique(window[blocks_five]).size
    fours_left = np.unique(window[blocks_four]).size
    five_hits = blocks_five.sum(per_cell)
    cap = f32(GLOBAL_THREAT_CAP)
    tac = np.empty((n_c, TACTICAL_FEATURES), dtype=f32)
    tac[:, _T_WIN_NOW] = (clean & (mine == WINDOW_LEN - 1)).any(per_cell)
    tac[:, _T_OWN_BEST] = (mine.max(per_cell) + 1).astype(f32) / f32(WINDOW_LEN)
    tac[:, _T_OPP_BEST] = theirs.max(per_cell).astype(f32) / f32(WINDOW_LEN)
    tac[:, _T_MAKE_FIVE] = (clean & (mine == 4)).sum(per_cell).astype(f32) / n_rows
    tac[:, _T_MAKE_FOUR] = (clean & (mine == 3)).sum(per_cell).astype(f32) / n_rows
    tac[:, _T_BLOCK_FIVE] = five_hits.astype(f32) / n_rows
    tac[:, _T_BLOCK_FOUR] = blocks_four.sum(per_cell).astype(f32) / n_rows
    tac[:, _T_FIVES_LEFT] = f32(min(fives_left, GLOBAL_THREAT_CAP)) / cap
    tac[:, _T_FOURS_LEFT] = f32(min(fours_left, GLOBAL_THREAT_CAP)) / cap
    tac[:, _T_BLOCKS_ALL_FIVES] = (fives_left > 0) & (five_hits == fives_left)
    tac[:, _T_LIVE_ROWS] = live.sum(per_cell).astype(f32) / n_rows
    return dict(
        dec_cell=cell.astype(np.int64), dec_window=dec_window.astype(np.int64), dec_class=dec_class.astype(np.int64),
        action_window_index=window.astype(np.int64), action_post1_class=placed.astype(np.int64),
        action_pre_status=status.astype(np.int64), action_tactical=tac,
    )


def build(stone_qr, stone_owner, mover, legal_qr, moves_remaining) -> PositionGraph:
    """One position's graph from the builder input list: stones (q, r) with
    their owners, the player to move, the legal cells in engine order and the
    stones left this turn (reference builder.py:486-642).

    Raises ``ValueError`` for a terminal position (no legal moves), a turn
    that does not place one or two stones, two stones on one cell, or a
    legal cell that holds a stone or lies beyond distance 8 of every stone."""
    stones = np.asarray(stone_qr, dtype=np.int64).reshape(-1, 2)
    owners = np.asarray(stone_owner, dtype=np.int64).reshape(-1)
    cells = np.asarray(legal_qr, dtype=np.int64).reshape(-1, 2)
    if len(cells) == 0:
        raise ValueError(_MSG_TERMINAL)
    if moves_remaining not in (1, 2):
        raise ValueError(f"a turn places one or two stones; got moves_remaining={moves_remaining}")
    opponent = (owners != mover).astype(np.int64)  # stone_own: 0 the mover's, 1 the opponent's

    cell_key = _pack(cells)
    cell_order = np.argsort(cell_key, kind="stable")
    node_fields = _cell_node_fields(stones, opponent, cells, cell_key, cell_key[cell_order], cell_order)
    board = _Board(stones, opponent)

    axis, start, pattern, slots, win_key = _live_windows(board, stones)
    win, slot = np.nonzero(slots >= 0)  # window-major, slot-minor
    inc_class = TERN_OCC_CLASS[pattern[win], slot]
    rows = _cell_rows(board, cells, win_key, pattern)
    return PositionGraph(
        stone_own=opponent, stone_qr=stones,
        window_feat=TERN_RANK[pattern].astype(np.int64),
        window_id=np.column_stack([axis, start[:, 0], start[:, 1]]).astype(np.int64).reshape(-1, 3),
        inc_stone=slots[win, slot].astype(np.int64), inc_window=win.astype(np.int64),
        inc_class=inc_class.astype(np.int64),
        n_legal=len(cells), **node_fields,
        moves_remaining=moves_remaining, **rows,
    )


def from_spec(spec) -> PositionGraph:
    """Build from an :class:`engine.PositionSpec` (reference ``from_position``)."""
    return build(spec.stone_qr, spec.stone_owner, spec.mover, spec.legal_qr, spec.moves_remaining)


@dataclass
class Batch:
    """A collated batch (reference builder.py:666-752); same field names,
    dtypes and meanings, so a reference-built batch can be passed as is."""

    n_pos: int
    stone_own: torch.Tensor
    window_feat: torch.Tensor
    window_id: torch.Tensor
    moves_idx: torch.Tensor
    inc_stone: torch.Tensor
    inc_window: torch.Tensor
    inc_class: torch.Tensor
    max_t: int
    stone_slot: torch.Tensor
    coords: torch.Tensor
    attn_valid: torch.Tensor
    max_w: int
    window_slot: torch.Tensor
    value_valid: torch.Tensor
    n_cells: int
    legal_offsets: torch.Tensor
    cell_pos: torch.Tensor
    cell_nearest: torch.Tensor
    radius_src: torch.Tensor
    radius_dst: torch.Tensor
    radius_orbit: torch.Tensor
    radius_own: torch.Tensor
    radius_on_axis: torch.Tensor
    adjacency_src: torch.Tensor
    adjacency_dst: torch.Tensor
    adjacency_axis: torch.Tensor
    dec_cell: torch.Tensor
    dec_window: torch.Tensor
    dec_class: torch.Tensor
    relay_cell_ptr: torch.Tensor
    relay_window: torch.Tensor
    relay_class: torch.Tensor
    relay_win_ptr: torch.Tensor
    relay_wcell: torch.Tensor
    relay_cls_ptr: torch.Tensor
    relay_ccell: torch.Tensor
    act_class: torch.Tensor
    act_rev: torch.Tensor
    act_empty: torch.Tensor
    act_tactical: torch.Tensor

    def to(self, device, non_blocking: bool = True) -> "Batch":
        moved = {
            k: (v.to(device, non_blocking=non_blocking) if isinstance(v, torch.Tensor) else v)
            for k, v in vars(self).items()
        }
        return Batch(**moved)

    def pin_memory(self) -> "Batch":
        return Batch(**{k: (v.pin_memory() if isinstance(v, torch.Tensor) else v) for k, v in vars(self).items()})

    @property
    def n_stones(self) -> int:
        return int(self.stone_own.shape[0])

    @property
    def n_windows(self) -> int:
        return int(self.window_feat.shape[0])


RELAY_FIELDS = (
    "relay_cell_ptr", "relay_window", "relay_class", "relay_win_ptr",
    "relay_wcell", "relay_cls_ptr", "relay_ccell",
)


def relay_tables(dec_cell, dec_window, dec_class, n_windows: int, n_classes: int):
    """The relay's three CSR views of the decoder incidence (reference
    relay.py:48-94): cell-major with compact covered-cell ids, window-major,
    class-major. Host-side, stable sorts."""
    dc = np.asarray(dec_cell, dtype=np.int64)
    dw = np.asarray(dec_window, dtype=np.int64)
    dk = np.asarray(dec_class, dtype=np.int64)
    if not (dc.shape == dw.shape == dk.shape) or dc.ndim != 1:
        raise ValueError("dec_cell, dec_window, and dec_class must be one length")
    if dw.size:
        if dw.min() < 0 or dw.max() >= n_windows:
            raise ValueError(f"dec_window entries must lie in [0, {n_windows})")
        if dk.min() < 0 or dk.max() >= n_classes:
            raise ValueError(f"dec_class entries must lie in [0, {n_classes})")
    order = np.argsort(dc, kind="stable")
    window, cls, cells = dw[order], dk[order], dc[order]
    head = np.ones(len(cells), dtype=bool)
    head[1:] = cells[1:] != cells[:-1]
    edge_cell = np.cumsum(head) - 1
    cell_ptr = np.concatenate([np.nonzero(head)[0], [len(cells)]]).astype(np.int64)
    worder = np.argsort(window, kind="stable")
    win_ptr = np.searchsorted(window[worder], np.arange(n_windows + 1)).astype(np.int64)
    corder = np.argsort(cls, kind="stable")
    cls_ptr = np.searchsorted(cls[corder], np.arange(n_classes + 1)).astype(np.int64)
    out = (cell_ptr, window, cls, win_ptr, edge_cell[worder], cls_ptr, edge_cell[corder])
    return tuple(torch.from_numpy(np.ascontiguousarray(x, dtype=np.int64)) for x in out)


def _relay_fields(dec_cell, dec_window, dec_class, n_windows):
    return dict(zip(RELAY_FIELDS, relay_tables(dec_cell, dec_window, dec_class, n_windows, TERN_DEC_CLASSES)))


def _cat(parts, dtype=np.int64):
    if not parts:
        return torch.empty(0, dtype=torch.long)
    return torch.from_numpy(np.ascontiguousarray(np.concatenate(parts).astype(dtype)))


def collate(graphs: list[PositionGraph]) -> Batch:
    """Concatenate position graphs into one batch (reference builder.py:881-956)."""
    if not graphs:
        raise ValueError("empty batch")
    p = len(graphs)
    ns = np.array([g.n_stones for g in graphs])
    nw = np.array([g.n_windows for g in graphs])
    nl = np.array([g.n_legal for g in graphs])
    stone_off = np.concatenate([[0], np.cumsum(ns)])
    win_off = np.concatenate([[0], np.cumsum(nw)])
    cell_off = np.concatenate([[0], np.cumsum(nl)])
    max_t = int(ns.max()) + GLOBAL_ROWS
    max_w = int(nw.max()) + 1

    coords = np.zeros((p, max_t, 2), dtype=np.int32)
    attn_valid = np.zeros((p, max_t), dtype=bool)
    attn_valid[:, :GLOBAL_ROWS] = True
    value_valid = np.zeros((p, max_w), dtype=bool)
    value_valid[:, 0] = True
    for i, g in enumerate(graphs):
        coords[i, GLOBAL_ROWS: GLOBAL_ROWS + g.n_stones] = g.stone_qr
        attn_valid[i, GLOBAL_ROWS: GLOBAL_ROWS + g.n_stones] = True
        value_valid[i, 1: 1 + g.n_windows] = True

    dec_cell = _cat([g.dec_cell + cell_off[i] for i, g in enumerate(graphs)])
    dec_window = _cat([g.dec_window + win_off[i] for i, g in enumerate(graphs)])
    dec_class = _cat([g.dec_class for g in graphs])

    # Action-row views: kept rows ride the decoder order; EMPTY rows become
    # per-orbit counts (reference builder.py:840-878).
    classes, counts = [], []
    for g in graphs:
        status = g.action_pre_status.reshape(g.n_legal, -1)
        kept = (status != ACTION_EMPTY).ravel()
        flat = np.nonzero(kept)[0]
        if not np.array_equal(flat // (3 * WINDOW_LEN), g.dec_cell):
            raise ValueError("action-row cells disagree with the decoder walk")
        if not np.array_equal(g.action_window_index.ravel()[kept], g.dec_window):
            raise ValueError("action-row windows disagree with the decoder walk")
        classes.append(g.action_post1_class.ravel()[kept])
        emp = (status == ACTION_EMPTY).reshape(g.n_legal, 3, WINDOW_LEN)
        counts.append(np.stack(
            [emp[:, :, ACTION_SLOT_ORBIT == o].sum(axis=(1, 2)) for o in range(ACTION_EMPTY_ORBITS)],
            axis=1,
        ))

    return Batch(
        n_pos=p,
        stone_own=_cat([g.stone_own for g in graphs]),
        window_feat=_cat([g.window_feat for g in graphs]),
        window_id=_cat([g.window_id for g in graphs]).view(-1, 3),
        moves_idx=torch.tensor([g.moves_remaining - 1 for g in graphs], dtype=torch.long),
        inc_stone=_cat([g.inc_stone + stone_off[i] for i, g in enumerate(graphs)]),
        inc_window=_cat([g.inc_window + win_off[i] for i, g in enumerate(graphs)]),
        inc_class=_cat([g.inc_class for g in graphs]),
        max_t=max_t,
        stone_slot=_cat([i * max_t + GLOBAL_ROWS + np.arange(g.n_stones) for i, g in enumerate(graphs)]),
        coords=torch.from_numpy(coords),
        attn_valid=torch.from_numpy(attn_valid),
        max_w=max_w,
        window_slot=_cat([i * max_w + 1 + np.arange(g.n_windows) for i, g in enumerate(graphs)]),
        value_valid=torch.from_numpy(value_valid),
        n_cells=int(cell_off[-1]),
        legal_offsets=torch.from_numpy(cell_off.astype(np.int64)),
        cell_pos=_cat([np.full(g.n_legal, i) for i, g in enumerate(graphs)]),
        cell_nearest=_cat([g.cell_nearest for g in graphs]),
        radius_src=_cat([g.radius_src + stone_off[i] for i, g in enumerate(graphs)]),
        radius_dst=_cat([g.radius_dst + cell_off[i] for i, g in enumerate(graphs)]),
        radius_orbit=_cat([g.radius_orbit for g in graphs]),
        radius_own=_cat([g.radius_own for g in graphs]),
        radius_on_axis=_cat([g.radius_on_axis for g in graphs]),
        adjacency_src=_cat([g.adjacency_src + cell_off[i] for i, g in enumerate(graphs)]),
        adjacency_dst=_cat([g.adjacency_dst + cell_off[i] for i, g in enumerate(graphs)]),
        adjacency_axis=_cat([g.adjacency_axis for g in graphs]),
        dec_cell=dec_cell,
        dec_window=dec_window,
        dec_class=dec_class,
        **_relay_fields(dec_cell.numpy(), dec_window.numpy(), dec_class.numpy(), int(win_off[-1])),
        act_class=_cat(classes),
        act_rev=torch.from_numpy(np.argsort(dec_window.numpy(), kind="stable").astype(np.int64)),
        act_empty=_cat(counts).view(-1, ACTION_EMPTY_ORBITS),
        act_tactical=torch.from_numpy(
            np.concatenate([g.action_tactical for g in graphs]).astype(np.float32).reshape(-1, TACTICAL_FEATURES)
        ),
    )


def batch_from_arrays(**fields) -> Batch:
    """A ``Batch`` from per-field arrays with the relay views derived here
    (reference builder.py:778-811). Scalar fields may be passed; a value that
    disagrees with the tensor shapes is refused."""
    scalars = {k: int(fields.pop(k)) for k in ("n_pos", "max_t", "max_w", "n_cells") if k in fields}
    t = {k: torch.as_tensor(v) for k, v in fields.items()}
    derived = {
        "n_pos": int(t["attn_valid"].shape[0]),
        "max_t": int(t["attn_valid"].shape[1]),
        "max_w": int(t["value_valid"].shape[1]),
        "n_cells": int(t["cell_pos"].shape[0]),
    }
    for k, v in scalars.items():
        if v != derived[k]:
            raise ValueError(f"{k}={v} disagrees with the derived {derived[k]}")
    for k in RELAY_FIELDS:
        t.pop(k, None)
    return Batch(
        **derived, **t,
        **_relay_fields(t["dec_cell"].numpy(), t["dec_window"].numpy(), t["dec_class"].numpy(),
                        int(t["window_feat"].shape[0])),
    )
