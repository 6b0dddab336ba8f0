"""Builder parity: every PositionGraph field and the collated Batch are
bit-exact against the reference builder's output (fixtures from
tests/golden/make_golden.py; reference tests test_builder.py and
test_rust_builder.py check the same field set)."""

from __future__ import annotations

import dataclasses

import numpy as np
import pytest
import torch

from golden_io import batch_from, load, mb


@pytest.fixture(scope="module")
def fixture():
    return load("builder.npz")


def _spec(d, i):
    return (d[f"{i}.in.stone_qr"], d[f"{i}.in.stone_owner"], int(d[f"{i}.in.mover"]),
            d[f"{i}.in.legal_qr"], int(d[f"{i}.in.moves_remaining"]))


def test_every_graph_field_bit_exact(fixture):
    n = int(fixture["n_cases"])
    assert n >= 12
    for i in range(n):
        g = mb.build(*_spec(fixture, i))
        for f in dataclasses.fields(g):
            got = getattr(g, f.name)
            want = fixture[f"{i}.out.{f.name}"]
            if isinstance(got, np.ndarray):
                assert got.dtype == want.dtype, (i, f.name)
                assert got.shape == want.shape and np.array_equal(got, want), (i, f.name)
            else:
                assert got == want, (i, f.name)


def test_collated_batch_bit_exact(fixture):
    n = int(fixture["n_cases"])
    graphs = [mb.build(*_spec(fixture, i)) for i in range(n - 1)]
    got = mb.collate(graphs)
    want = batch_from(fixture)
    for k, v in vars(want).items():
        g = getattr(got, k)
        if isinstance(v, torch.Tensor):
            assert g.dtype == v.dtype and g.shape == v.shape and torch.equal(g, v), k
        else:
            assert g == v, k


def test_batch_from_arrays_rederives_relay_views(fixture):
    want = batch_from(fixture)
    fields = {k: v for k, v in vars(want).items() if not k.startswith("relay_")}
    got = mb.batch_from_arrays(**fields)
    for k in mb.builder.RELAY_FIELDS:
        assert torch.equal(getattr(got, k), getattr(want, k)), k
    with pytest.raises(ValueError):
        mb.batch_from_arrays(**{**fields, "n_pos": want.n_pos + 1})


def test_builder_refusals():
    with pytest.raises(ValueError, match="terminal"):
        mb.build(np.zeros((1, 2)), np.zeros(1), 0, np.empty((0, 2)), 1)
    with pytest.raises(ValueError, match="moves_remaining"):
        mb.build(np.zeros((1, 2)), np.zeros(1), 0, np.array([[1, 0]]), 3)
    with pytest.raises(ValueError):  # legal cell on a stone
        mb.build(np.zeros((1, 2)), np.zeros(1), 0, np.array([[0, 0]]), 1)
    with pytest.raises(ValueError):  # legal cell out of reach
        mb.build(np.zeros((1, 2)), np.zeros(1), 0, np.array([[9, 0]]), 1)
    with pytest.raises(ValueError):
        mb.collate([])


def test_vocab_laws():
    v = mb.vocab
    assert (v.TERN_PATTERNS, v.TERN_DEC_CLASSES, v.TERN_OCC_CLASSES, v.TERN_POST1_CLASSES) == (377, 726, 1458, 729)
    assert v.TERN_PATTERN_CLASS_COUNTS.shape == (377, 1458)
    # each pattern's class counts sum to its occupied-slot count
    occ = (v.TERN_DIGITS != 0).sum(1)
    for p in range(1, 729):
        assert v.TERN_PATTERN_CLASS_COUNTS[v.TERN_RANK[p]].sum() == occ[p]
    assert int(v.ORBIT48_TABLE.max()) == 47
