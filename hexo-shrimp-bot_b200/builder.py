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
            raise ValueError("legal cells must be empty and within radius 8 of a stone")
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


def _action_tables(legal_qr, stone_sorted, stone_order, stone_own, live_key):
    """18 hypothetical post-placement rows per legal action plus the tactical
    scalars (reference builder.py:292-424)."""
    n_legal = len(legal_qr)
    offs = np.arange(-(WINDOW_LEN - 1), WINDOW_LEN, dtype=np.int64)
    cells = legal_qr[:, None, None, :] + AXES[None, :, None, :] * offs[None, None, :, None]
    occ = _lookup(stone_sorted, _pack(cells))
    occupant = np.where(occ >= 0, stone_order[np.maximum(occ, 0)] if len(stone_order) else 0, -1)
    digit = np.where(occupant >= 0, np.where(stone_own[np.maximum(occupant, 0)] == 0, 1, 2), 0) \
        if len(stone_own) else np.zeros(occupant.shape, dtype=np.int64)
    line = digit.reshape(n_legal, 3, 2 * WINDOW_LEN - 1)
    if line[:, :, WINDOW_LEN - 1].any():
        raise ValueError("a legal action cell is occupied")
    # slot j of the window starting k steps before the cell sits at line[j + 5 - k]
    j_idx = np.arange(WINDOW_LEN)[None, :] + (WINDOW_LEN - 1) - np.arange(WINDOW_LEN)[:, None]
    win_digits = line[:, :, j_idx]  # (n_legal, 3, k, j)
    pre = (win_digits * POW3).sum(axis=-1)
    own_count = (win_digits == 1).sum(axis=-1)
    opp_count = (win_digits == 2).sum(axis=-1)
    has_own, has_opp = own_count > 0, opp_count > 0
    status = np.where(
        has_own & ~has_opp, ACTION_OWN,
        np.where(has_opp & ~has_own, ACTION_OPP,
                 np.where(has_own & has_opp, ACTION_MIXED, ACTION_EMPTY)),
    )
    k_arr = np.arange(WINDOW_LEN)[None, None, :]
    post1 = TERN_POST1_CLASS[pre + POW3[None, None, :], k_arr]
    if post1.min(initial=0) < 0:
        raise ValueError("a post-placement row lost its own stone")

    starts = legal_qr[:, None, None, :] - AXES[None, :, None, :] * np.arange(WINDOW_LEN)[None, None, :, None]
    wkey = _pack(starts) * 4 + np.arange(3)[None, :, None]
    window_index = _lookup(live_key, wkey)
    kept = status != ACTION_EMPTY
    if ((window_index >= 0) != kept).any():
        raise ValueError("the kept-window set disagrees with the action-row walk")

    opp_only = has_opp & ~has_own
    five_rows = opp_only & (opp_count == 5)
    four_rows = opp_only & (opp_count == 4)
    five_remaining = len(np.unique(window_index[five_rows]))
    four_remaining = len(np.unique(window_index[four_rows]))
    ax = (1, 2)
    opp_five_hit = five_rows.sum(axis=ax)
    rows_total = np.float32(3 * WINDOW_LEN)
    f32 = np.float32

    tactical = np.stack(
        [
            (~has_opp & (own_count == WINDOW_LEN - 1)).any(axis=ax).astype(f32),
            (own_count.max(axis=ax) + 1).astype(f32) / f32(WINDOW_LEN),
            opp_count.max(axis=ax).astype(f32) / f32(WINDOW_LEN),
            (~has_opp & (own_count + 1 == 5)).sum(axis=ax).astype(f32) / rows_total,
            (~has_opp & (own_count + 1 == 4)).sum(axis=ax).astype(f32) / rows_total,
            opp_five_hit.astype(f32) / rows_total,
            four_rows.sum(axis=ax).astype(f32) / rows_total,
            np.full(n_legal, f32(min(five_remaining, GLOBAL_THREAT_CAP)) / f32(GLOBAL_THREAT_CAP), dtype=f32),
            np.full(n_legal, f32(min(four_remaining, GLOBAL_THREAT_CAP)) / f32(GLOBAL_THREAT_CAP), dtype=f32),
            ((five_remaining > 0) & (opp_five_hit == five_remaining)).astype(f32),
            kept.sum(axis=ax).astype(f32) / rows_total,
        ],
        axis=1,
    ).astype(f32)
    return window_index, post1, status, tactical


def build(stone_qr, stone_owner, mover, legal_qr, moves_remaining) -> PositionGraph:
    """One position's graph from the builder input list (reference builder.py:486-642).

    Raises ``ValueError`` for a terminal position (no legal moves), a bad
    ``moves_remaining``, duplicate stones, or legal cells that are occupied
    or out of reach."""
    stone_qr = np.asarray(stone_qr, dtype=np.int64).reshape(-1, 2)
    stone_owner = np.asarray(stone_owner, dtype=np.int64).reshape(-1)
    legal_qr = np.asarray(legal_qr, dtype=np.int64).reshape(-1, 2)
    if len(legal_qr) == 0:
        raise ValueError("terminal position: the builder refuses it")
    if moves_remaining not in (1, 2):
        raise ValueError(f"moves_remaining must be 1 or 2, got {moves_remaining}")
    n_s = len(stone_qr)
    stone_own = (stone_owner != mover).astype(np.int64)

    legal_key = _pack(legal_qr)
    legal_order = np.argsort(legal_key, kind="stable")
    legal_sorted = legal_key[legal_order]
    legal_rank = legal_order  # sorted slot -> legal row
    cell_nodes = _cell_node_fields(stone_qr, stone_own, legal_qr, legal_key, legal_sorted, legal_rank)

    empty = np.empty(0, dtype=np.int64)
    if n_s == 0:
        actions = _action_tables(legal_qr, empty, empty, stone_own, empty)
        return PositionGraph(
            stone_own=stone_own, stone_qr=stone_qr,
            window_feat=empty, window_id=np.empty((0, 3), dtype=np.int64),
            inc_stone=empty, inc_window=empty, inc_class=empty,
            n_legal=len(legal_qr), **cell_nodes,
            dec_cell=empty, dec_window=empty, dec_class=empty,
            moves_remaining=moves_remaining,
            action_window_index=actions[0], action_post1_class=actions[1],
            action_pre_status=actions[2], action_tactical=actions[3],
        )

    stone_key = _pack(stone_qr)
    stone_order = np.argsort(stone_key, kind="stable")
    stone_sorted = stone_key[stone_order]
    if np.any(stone_sorted[1:] == stone_sorted[:-1]):
        raise ValueError("duplicate stone coordinates")

    ks = np.arange(WINDOW_LEN, dtype=np.int64)
    # Every (axis, start) through some stone: 18 candidates per stone.
    starts = stone_qr[:, None, None, :] - AXES[None, :, None, :] * ks[None, None, :, None]
    axis_of = np.broadcast_to(np.arange(3)[None, :, None], starts.shape[:3])
    cand_key = (_pack(starts) * 4 + axis_of).reshape(-1)
    live_key, first = np.unique(cand_key, return_index=True)
    w_start = starts.reshape(-1, 2)[first]
    w_axis = axis_of.reshape(-1)[first].astype(np.int64)

    wcells = w_start[:, None, :] + AXES[w_axis][:, None, :] * ks[None, :, None]
    occ = _lookup(stone_sorted, _pack(wcells))
    occupant = np.where(occ >= 0, stone_order[np.maximum(occ, 0)], -1)  # (n_w, 6)
    own = stone_own[np.maximum(occupant, 0)]
    digit = np.where(occupant >= 0, 1 + own, 0)
    pattern = (digit * POW3[None, :]).sum(axis=1)
    window_feat = TERN_RANK[pattern]
    window_id = np.column_stack([w_axis, w_start[:, 0], w_start[:, 1]])

    w_idx, slot = np.nonzero(occupant >= 0)
    inc_stone = occupant[w_idx, slot]
    inc_class = TERN_OCC_CLASS[pattern[w_idx], slot]
    if inc_class.size and inc_class.min() < 0:
        raise ValueError("incidence entry pairs a window with a slot it does not occupy")

    c_starts = legal_qr[:, None, None, :] - AXES[None, :, None, :] * ks[None, None, :, None]
    c_key = (_pack(c_starts) * 4 + np.arange(3)[None, :, None]).reshape(-1)
    c_win = _lookup(live_key, c_key)
    flat = np.nonzero(c_win >= 0)[0]
    dec_cell = flat // (3 * WINDOW_LEN)
    dec_window = c_win[flat]
    dec_class = TERN_DEC_CLASS[pattern[dec_window], flat % WINDOW_LEN]
    if dec_class.size and dec_class.min() < 0:
        raise ValueError("decoder entry pairs a window with a slot it already occupies")

    actions = _action_tables(legal_qr, stone_sorted, stone_order, stone_own, live_key)
    return PositionGraph(
        stone_own=stone_own, stone_qr=stone_qr,
        window_feat=window_feat, window_id=window_id,
        inc_stone=inc_stone.astype(np.int64), inc_window=w_idx.astype(np.int64),
        inc_class=inc_class,
        n_legal=len(legal_qr), **cell_nodes,
        dec_cell=dec_cell.astype(np.int64), dec_window=dec_window.astype(np.int64),
        dec_class=dec_class,
        moves_remaining=moves_remaining,
        action_window_index=actions[0], action_post1_class=actions[1],
        action_pre_status=actions[2], action_tactical=actions[3],
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
