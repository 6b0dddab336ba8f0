"""Closed vocabularies of the MantisNet representation (integer tables).

Every table here is part of the representation contract: the class numbering
must equal the reference's exactly, because checkpoints index embedding rows
by it. The tables are derived from first principles (orbits of a reversal or
D6 action, ranked by their smallest representative), not transcribed.

Reference definitions followed:
- window ternary pattern and its reversal rank: python/mantisnet/mantisnet/builder.py:93-115
- joint (pattern, slot) decoder / incidence classes: builder.py:118-155
- per-pattern occupied-class counts: builder.py:158-185
- post-placement (own insert) classes and EMPTY orbits: builder.py:188-229
- D6 displacement orbits (48 classes within radius 12): builder.py:41-90
- radius class composition (orbit + 48 * (own + 2 * on_axis)): model.py:867-869,
  cell_nodes.py:16-17
"""

from __future__ import annotations

import numpy as np

WINDOW_LEN = 6
# Unit steps of the three line axes, canonical order Q, R, QR.
AXES = np.array([[1, 0], [0, 1], [1, -1]], dtype=np.int64)
GLOBAL_ROWS = 4  # state latents per position
LEGAL_RADIUS = 8
CELL_NEAREST_UNREACHED = 9
TACTICAL_FEATURES = 11
GLOBAL_THREAT_CAP = 8
ORBIT48_CLASSES = 48
RADIUS_CLASSES = ORBIT48_CLASSES * 2 * 2
ADJACENCY_CLASSES = 1
NEAREST_BUCKETS = 10
ACTION_EMPTY_ORBITS = 3
ACTION_OWN, ACTION_OPP, ACTION_EMPTY, ACTION_MIXED = 0, 1, 2, 3

POW3 = 3 ** np.arange(WINDOW_LEN, dtype=np.int64)
N_PATTERNS_RAW = 3**WINDOW_LEN  # 729


def _digits() -> np.ndarray:
    return (np.arange(N_PATTERNS_RAW)[:, None] // POW3[None, :]) % 3


TERN_DIGITS = _digits()  # (729, 6): slot k digit, 0 empty, 1 own, 2 opp
TERN_REV = (TERN_DIGITS[:, ::-1] * POW3[None, :]).sum(axis=1)  # reversed pattern


def _pattern_rank() -> np.ndarray:
    """Rank of each raw pattern's reversal class among nonempty classes."""
    canon = np.minimum(np.arange(N_PATTERNS_RAW), TERN_REV)
    reps = np.unique(canon[canon > 0])
    rank = np.full(N_PATTERNS_RAW, -1, dtype=np.int64)
    rank[1:] = np.searchsorted(reps, canon[1:])
    return rank


TERN_RANK = _pattern_rank()
TERN_PATTERNS = int(TERN_RANK.max()) + 1  # 377


def _orbit_rank(mask: np.ndarray) -> np.ndarray:
    """Rank every (pattern, slot) pair in ``mask`` by the smallest member of its
    orbit under (p, s) -> (reverse(p), 5 - s); -1 outside ``mask``.

    The orbit ids of the reference are handed out in ascending (p, s) order of
    each orbit's smallest member, so ranking by that member gives the same
    numbering once restricted to ``mask`` (both members of an orbit share
    membership in every mask used here)."""
    p = np.arange(N_PATTERNS_RAW)[:, None].repeat(WINDOW_LEN, axis=1)
    s = np.arange(WINDOW_LEN)[None, :].repeat(N_PATTERNS_RAW, axis=0)
    key = p * WINDOW_LEN + s
    mirror = TERN_REV[p] * WINDOW_LEN + (WINDOW_LEN - 1 - s)
    rep = np.minimum(key, mirror)
    table = np.full((N_PATTERNS_RAW, WINDOW_LEN), -1, dtype=np.int64)
    reps = np.unique(rep[mask])
    table[mask] = np.searchsorted(reps, rep[mask])
    return table


_EMPTY_SLOT = TERN_DIGITS == 0
TERN_DEC_CLASS = _orbit_rank(_EMPTY_SLOT & (np.arange(N_PATTERNS_RAW) != 0)[:, None])
TERN_OCC_CLASS = _orbit_rank(~_EMPTY_SLOT)
TERN_POST1_CLASS = _orbit_rank(TERN_DIGITS == 1)
TERN_DEC_CLASSES = int(TERN_DEC_CLASS.max()) + 1  # 726
TERN_OCC_CLASSES = int(TERN_OCC_CLASS.max()) + 1  # 1458
TERN_POST1_CLASSES = int(TERN_POST1_CLASS.max()) + 1  # 729
ACTION_EMPTY_CLASSES = tuple(int(TERN_POST1_CLASS[3**k, k]) for k in range(3))
# EMPTY row orbit of candidate slot k: slot k and 5 - k fold together.
ACTION_SLOT_ORBIT = np.minimum(np.arange(WINDOW_LEN), WINDOW_LEN - 1 - np.arange(WINDOW_LEN))


def _pattern_class_counts() -> np.ndarray:
    """(377, 1458) float32 occupied-slot class histogram per pattern class."""
    counts = np.zeros((TERN_PATTERNS, TERN_OCC_CLASSES), dtype=np.float32)
    seen = np.zeros(TERN_PATTERNS, dtype=bool)
    for p in range(1, N_PATTERNS_RAW):
        r = TERN_RANK[p]
        if seen[r]:
            continue
        seen[r] = True
        for s in range(WINDOW_LEN):
            c = TERN_OCC_CLASS[p, s]
            if c >= 0:
                counts[r, c] += 1.0
    return counts


TERN_PATTERN_CLASS_COUNTS = _pattern_class_counts()


# --- D6 displacement orbits.

def _images(q: int, r: int) -> list[tuple[int, int]]:
    out = []
    for seed in ((q, r), (r, q)):  # identity and the reflection
        a, b = seed
        for _ in range(6):  # rotation by 60 degrees: (q, r) -> (-r, q + r)
            out.append((a, b))
            a, b = -b, a + b
    return out


def hex_distance(qr: np.ndarray) -> np.ndarray:
    qr = np.asarray(qr)
    return np.maximum.reduce(
        [np.abs(qr[..., 0]), np.abs(qr[..., 1]), np.abs(qr[..., 0] + qr[..., 1])]
    )


ORBIT_SPAN = 12


def _orbit48_table() -> np.ndarray:
    """(25, 25) orbit id for (dq, dr) in [-12, 12]^2, -1 at distance 0 or > 12.

    Orbits are ordered by (distance, smallest image) which is the reference's
    representative order."""
    reps = {}
    for q in range(-ORBIT_SPAN, ORBIT_SPAN + 1):
        for r in range(-ORBIT_SPAN, ORBIT_SPAN + 1):
            d = max(abs(q), abs(r), abs(q + r))
            if 1 <= d <= ORBIT_SPAN:
                reps[(q, r)] = (d, *min(_images(q, r)))
    order = sorted(set(reps.values()))
    rank = {rep: i for i, rep in enumerate(order)}
    table = np.full((2 * ORBIT_SPAN + 1, 2 * ORBIT_SPAN + 1), -1, dtype=np.int64)
    for (q, r), rep in reps.items():
        table[q + ORBIT_SPAN, r + ORBIT_SPAN] = rank[rep]
    return table


ORBIT48_TABLE = _orbit48_table()


def orbit48_id(dq, dr):
    """Orbit class of displacement(s) with distance 1..12 (vectorised)."""
    dq = np.asarray(dq)
    dr = np.asarray(dr)
    d = hex_distance(np.stack([dq, dr], axis=-1))
    if np.any((d < 1) | (d > ORBIT_SPAN)):
        raise ValueError("displacement outside distance 1..12")
    return ORBIT48_TABLE[dq + ORBIT_SPAN, dr + ORBIT_SPAN]


def radius_class(orbit, own, on_axis):
    """The 192-way radius class: orbit + 48 * (own + 2 * on_axis)."""
    return orbit + ORBIT48_CLASSES * (own + 2 * on_axis)


# Coverage buckets (cell_structure knob): degree 1..18 folded into 8 buckets.
COVERAGE_BUCKETS = 8
COVERAGE_BUCKET_OF = np.array(
    [0, 0, 1, 2, 3, 4, 4, 5, 5, 5, 6, 6, 6, 6, 7, 7, 7, 7, 7], dtype=np.int64
)

assert len(np.unique(np.minimum(np.arange(729), TERN_REV))) == 378
assert TERN_PATTERNS == 377
assert TERN_DEC_CLASSES == 726 and TERN_OCC_CLASSES == 1458 and TERN_POST1_CLASSES == 729
assert int(ORBIT48_TABLE.max()) + 1 == ORBIT48_CLASSES
assert len(set(ACTION_EMPTY_CLASSES)) == ACTION_EMPTY_ORBITS
