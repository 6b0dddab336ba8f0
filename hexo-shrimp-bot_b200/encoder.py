"""Positions to a collated ``Batch`` through the library's C++ encoder.

The same batch as ``collate([build(...) for each position])`` (every array
and its order; the builder follows the reference builder,
python/mantisnet/mantisnet/builder.py:486-956), built by native code over
all host threads instead of numpy per position. The reference's production
counterpart is its Rust encoder (crates/models/mantisnet/src/encoder.rs).
The arrays can be written straight into pinned host memory, ready for the
host-to-device copy.
"""

from __future__ import annotations

import ctypes
from typing import Sequence

import numpy as np
import torch

from . import _lib
from .builder import Batch

# (Batch field, dtype, shape from the sizes) in the C-ABI's field order
# (MB_ENC_* in include/mantis_b200.h).
_P, _NS, _NW, _NINC, _NC, _NR, _NA, _ND, _MAXT, _MAXW, _NCOV = range(11)
_FIELDS = (
    ("stone_own", torch.int64, lambda s: (s[_NS],)),
    ("window_feat", torch.int64, lambda s: (s[_NW],)),
    ("window_id", torch.int64, lambda s: (s[_NW], 3)),
    ("moves_idx", torch.int64, lambda s: (s[_P],)),
    ("inc_stone", torch.int64, lambda s: (s[_NINC],)),
    ("inc_window", torch.int64, lambda s: (s[_NINC],)),
    ("inc_class", torch.int64, lambda s: (s[_NINC],)),
    ("stone_slot", torch.int64, lambda s: (s[_NS],)),
    ("coords", torch.int32, lambda s: (s[_P], s[_MAXT], 2)),
    ("attn_valid", torch.bool, lambda s: (s[_P], s[_MAXT])),
    ("window_slot", torch.int64, lambda s: (s[_NW],)),
    ("value_valid", torch.bool, lambda s: (s[_P], s[_MAXW])),
    ("legal_offsets", torch.int64, lambda s: (s[_P] + 1,)),
    ("cell_pos", torch.int64, lambda s: (s[_NC],)),
    ("cell_nearest", torch.int64, lambda s: (s[_NC],)),
    ("radius_src", torch.int64, lambda s: (s[_NR],)),
    ("radius_dst", torch.int64, lambda s: (s[_NR],)),
    ("radius_orbit", torch.int64, lambda s: (s[_NR],)),
    ("radius_own", torch.int64, lambda s: (s[_NR],)),
    ("radius_on_axis", torch.int64, lambda s: (s[_NR],)),
    ("adjacency_src", torch.int64, lambda s: (s[_NA],)),
    ("adjacency_dst", torch.int64, lambda s: (s[_NA],)),
    ("adjacency_axis", torch.int64, lambda s: (s[_NA],)),
    ("dec_cell", torch.int64, lambda s: (s[_ND],)),
    ("dec_window", torch.int64, lambda s: (s[_ND],)),
    ("dec_class", torch.int64, lambda s: (s[_ND],)),
    ("relay_cell_ptr", torch.int64, lambda s: (s[_NCOV] + 1,)),
    ("relay_window", torch.int64, lambda s: (s[_ND],)),
    ("relay_class", torch.int64, lambda s: (s[_ND],)),
    ("relay_win_ptr", torch.int64, lambda s: (s[_NW] + 1,)),
    ("relay_wcell", torch.int64, lambda s: (s[_ND],)),
    ("relay_cls_ptr", torch.int64, lambda s: (727,)),
    ("relay_ccell", torch.int64, lambda s: (s[_ND],)),
    ("act_class", torch.int64, lambda s: (s[_ND],)),
    ("act_rev", torch.int64, lambda s: (s[_ND],)),
    ("act_empty", torch.int64, lambda s: (s[_NC], 3)),
    ("act_tactical", torch.float32, lambda s: (s[_NC], 11)),
)


# The fields the narrow layout writes as int32 (int64 in the batch contract).
INT64_FIELDS = frozenset(name for name, dt, _ in _FIELDS if dt == torch.int64)


def _flat(arrays, cols: int) -> tuple[np.ndarray, np.ndarray]:
    """Concatenated int64 rows and the (n + 1) row offsets."""
    parts = [np.asarray(a, dtype=np.int64).reshape(-1, cols) for a in arrays]
    off = np.zeros(len(parts) + 1, dtype=np.int64)
    np.cumsum([len(p) for p in parts], out=off[1:])
    flat = np.ascontiguousarray(np.concatenate(parts) if parts else np.zeros((0, cols), np.int64))
    return flat, off


def encode(positions: Sequence, threads: int = 0, pin_memory: bool = False, narrow: bool = False) -> Batch:
    """The collated batch of ``positions`` (objects with ``stone_qr``,
    ``stone_owner``, ``mover``, ``legal_qr``, ``moves_remaining``, such as
    ``engine.PositionSpec``). ``threads`` = 0 uses every hardware thread.
    ``narrow`` writes the int64 fields as int32 (the same values; half the
    host memory and host-to-device bytes), which ``network_evaluate`` widens
    on the device. Raises ``ValueError`` for a position the builder refuses,
    naming it."""
    if len(positions) == 0:
        raise ValueError("empty batch")
    stone_qr, stone_off = _flat([p.stone_qr for p in positions], 2)
    owner, _ = _flat([p.stone_owner for p in positions], 1)
    legal_qr, legal_off = _flat([p.legal_qr for p in positions], 2)
    mover = np.ascontiguousarray([int(p.mover) for p in positions], dtype=np.int64)
    moves = np.ascontiguousarray([int(p.moves_remaining) for p in positions], dtype=np.int64)
    if len(owner) != len(stone_qr):
        raise ValueError("stone_owner and stone_qr lengths differ")
    lib = _lib.load()
    handle = ctypes.c_void_p()

    def ptr(a):
        return a.ctypes.data if a.size else None

    _lib.call("mb_encode_positions", len(positions), ptr(stone_off), ptr(stone_qr), ptr(owner), ptr(mover),
              ptr(legal_off), ptr(legal_qr), ptr(moves), int(threads), ctypes.byref(handle))
    try:
        sizes = np.zeros(11, dtype=np.int64)
        _lib.call("mb_encoding_sizes", handle, sizes.ctypes.data)
        s = [int(v) for v in sizes]
        out = {}
        for name, dt, shape in _FIELDS:
            if narrow and dt == torch.int64:
                dt = torch.int32
            t = torch.empty(shape(s), dtype=dt, pin_memory=pin_memory)
            out[name] = t
        # torch.bool is one byte per flag, 0 or 1, as the encoder writes it;
        # a zero-size buffer still needs a valid address.
        keep = [torch.empty(1, dtype=torch.int64) for _ in _FIELDS]
        addrs = (ctypes.c_void_p * len(_FIELDS))(
            *[out[name].data_ptr() if out[name].numel() else keep[i].data_ptr() for i, (name, _, _) in
              enumerate(_FIELDS)])
        _lib.call("mb_encoding_fill_narrow" if narrow else "mb_encoding_fill", handle, addrs, int(threads))
    finally:
        lib.mb_encoding_free(handle)
    return Batch(n_pos=s[_P], max_t=s[_MAXT], max_w=s[_MAXW], n_cells=s[_NC], **out)


def vocab_table(which: int) -> np.ndarray:
    """The encoder's own copy of a vocabulary table (see mb_encoder_table)."""
    n = {0: 729, 1: 729 * 6, 2: 729 * 6, 3: 729 * 6, 4: 25 * 25}[which]
    out = np.zeros(n, dtype=np.int64)
    _lib.call("mb_encoder_table", which, out.ctypes.data, n)
    return out
