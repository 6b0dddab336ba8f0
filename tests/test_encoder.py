"""The native batch encoder (mb_encode_positions, encoder.encode): the
collated batch of the reference builder's golden fixture bit-exact, the same
arrays as the package's numpy builder on seeded random positions (early and
late game, empty board, one stone), the same refusals, and the same result
at any thread count. Host-only: runs without a GPU."""

from __future__ import annotations

from dataclasses import replace

import numpy as np
import pytest
import torch

from golden_io import batch_from, load, mb

enc = mb.encoder
eng = mb.engine
PositionSpec = eng.PositionSpec


def _library_built():
    if not mb._lib.LIB_PATH.exists():
        pytest.skip("library not built (run hexo-shrimp-bot_b200/build.py)")


def _assert_same_batch(got, want):
    for k, v in vars(want).items():
        g = getattr(got, k)
        if isinstance(v, torch.Tensor):
            assert g.dtype == v.dtype and g.shape == v.shape and torch.equal(g, v), k
        else:
            assert g == v, k


def test_vocabulary_tables_match_the_package_derivation():
    _library_built()
    V = mb.vocab
    for i, ref in enumerate([V.TERN_RANK, V.TERN_OCC_CLASS, V.TERN_DEC_CLASS, V.TERN_POST1_CLASS, V.ORBIT48_TABLE]):
        assert np.array_equal(enc.vocab_table(i), ref.ravel()), i


def test_reference_fixture_batch_bit_exact():
    _library_built()
    d = load("builder.npz")
    n = int(d["n_cases"])
    specs = [PositionSpec(d[f"{i}.in.stone_qr"], d[f"{i}.in.stone_owner"], int(d[f"{i}.in.mover"]),
                          d[f"{i}.in.legal_qr"], int(d[f"{i}.in.moves_remaining"])) for i in range(n - 1)]
    _assert_same_batch(enc.encode(specs), batch_from(d))


@pytest.mark.parametrize("lo,hi,count,seed", [(0, 40, 24, 3), (40, 150, 8, 4), (150, 300, 4, 5)])
def test_matches_numpy_builder(lo, hi, count, seed):
    _library_built()
    specs = eng.random_positions(count, lo, hi, seed=seed)
    want = mb.collate([mb.from_spec(s) for s in specs])
    _assert_same_batch(enc.encode(specs), want)
    _assert_same_batch(enc.encode(specs, threads=1), want)
    _assert_same_batch(enc.encode(specs, threads=3), want)


def test_empty_board_and_single_stone():
    _library_built()
    empty = PositionSpec(np.zeros((0, 2), np.int64), np.zeros(0, np.int64), 0, np.array([[0, 0], [1, 0]]), 1)
    one = PositionSpec(np.array([[0, 0]]), np.array([1]), 0, np.array([[1, 0], [0, 1], [-1, 1], [8, 0]]), 2)
    for case in ([empty], [one], [empty, one, empty]):
        _assert_same_batch(enc.encode(case), mb.collate([mb.from_spec(s) for s in case]))


def test_spread_out_position_takes_the_hash_index():
    """Two stone groups 3,000 cells apart: the bounding box exceeds the dense
    grid's 4M cells, so every lookup goes through the hash table instead of
    grid offsets; the arrays must not change. Mixed with a compact position
    (dense path) in one batch."""
    _library_built()
    far = PositionSpec(np.array([[0, 0], [1, 0], [3000, -1500], [3001, -1500], [3000, -1499]]),
                       np.array([0, 1, 0, 1, 1]), 0,
                       np.array([[2, 0], [0, 1], [-1, 0], [-3, 4], [3002, -1500], [2999, -1500], [3003, -1505]]), 1)
    near = eng.random_positions(1, 20, 40, seed=9)[0]
    for case in ([far], [far, near], [near, far]):
        _assert_same_batch(enc.encode(case), mb.collate([mb.from_spec(s) for s in case]))
        _assert_same_batch(enc.encode(case, threads=2), mb.collate([mb.from_spec(s) for s in case]))


def test_refusals_match_the_builder():
    _library_built()
    good = eng.random_positions(1, 10, 20, seed=6)[0]
    cases = [
        PositionSpec(np.array([[0, 0]]), np.array([0]), 0, np.zeros((0, 2), np.int64), 1),  # terminal
        replace(good, moves_remaining=3),
        PositionSpec(np.array([[0, 0], [0, 0]]), np.array([0, 1]), 0, np.array([[1, 0]]), 1),  # duplicate stones
        PositionSpec(np.array([[0, 0]]), np.array([0]), 0, np.array([[0, 0]]), 1),  # legal cell occupied
        PositionSpec(np.array([[0, 0]]), np.array([0]), 0, np.array([[9, 0]]), 1),  # beyond distance 8
    ]
    for c in cases:
        with pytest.raises(ValueError) as py:
            mb.from_spec(c)
        with pytest.raises(ValueError) as native:
            enc.encode([good, c])
        assert "position 1" in str(native.value) and str(py.value) in str(native.value)
    with pytest.raises(ValueError):
        enc.encode([])


@pytest.mark.gpu
def test_pinned_output_matches():
    """pin_memory=True writes the same arrays into page-locked buffers."""
    _library_built()
    specs = eng.random_positions(6, 30, 90, seed=8)
    pinned = enc.encode(specs, pin_memory=True)
    plain = enc.encode(specs)
    for k, v in vars(plain).items():
        if isinstance(v, torch.Tensor):
            p = getattr(pinned, k)
            assert p.is_pinned() and torch.equal(p, v), k


def test_narrow_layout_holds_the_same_values():
    """encode(narrow=True) writes every int64 field as int32 with the same
    values (the layout the evaluator widens on the device)."""
    specs = mb.engine.random_positions(6, 5, 120, seed=41)
    wide = mb.encoder.encode(specs, threads=2)
    narrow = mb.encoder.encode(specs, threads=2, narrow=True)
    for k, v in vars(wide).items():
        if not isinstance(v, torch.Tensor):
            assert getattr(narrow, k) == v, k
            continue
        n = getattr(narrow, k)
        if k in mb.encoder.INT64_FIELDS:
            assert v.dtype == torch.int64 and n.dtype == torch.int32, k
            assert torch.equal(n.long(), v), k
        else:
            assert n.dtype == v.dtype and torch.equal(n, v), k
