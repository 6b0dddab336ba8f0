"""Sub-batch split of the evaluator (host logic, CPU): every run of positions
is a self-contained batch whose index fields point into its own stones,
windows, cells and positions, and the runs put back together give the parent
batch (the order the pipelined evaluator concatenates its outputs in)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from golden_io import mb

E = mb.evaluator
INDEX_RANGE = {  # field -> attribute counting the rows its values index
    "inc_stone": "stone_own", "inc_window": "window_feat", "radius_src": "stone_own", "radius_dst": "cell_pos",
    "dec_cell": "cell_pos", "dec_window": "window_feat",
}


@pytest.fixture(scope="module")
def batch():
    specs = mb.engine.random_positions(9, 20, 120, seed=11)
    return mb.collate([mb.from_spec(s) for s in specs])


KNOBS = [dict(cell_latents=True, cell_nodes=True), dict(cell_latents=True, cell_nodes=True, cell_adjacency=True)]


@pytest.mark.parametrize("knobs", KNOBS, ids=["production", "adjacency"])
@pytest.mark.parametrize("part", [1, 2, 3, 5, 100])
def test_runs_reassemble_the_batch(batch, part, knobs):
    cfg = mb.MantisConfig(h=32, blocks=1, heads=2, **knobs)
    fields = E.needed_fields(cfg)
    assert E.split_supported(fields)
    cuts = E.split_points(batch, part)
    assert cuts[0] == 0 and cuts[-1] == batch.n_pos and all(a < b for a, b in zip(cuts, cuts[1:]))
    off = E._offsets(batch, fields)
    parts = [E.part_to_device(batch, fields, off, a, b, "cpu") for a, b in zip(cuts, cuts[1:])]
    for part, p0 in zip(parts, cuts):
        for f, rows in INDEX_RANGE.items():
            v = getattr(part, f)
            assert v.numel() == 0 or (int(v.min()) >= 0 and int(v.max()) < getattr(part, rows).shape[0]), f
        assert int(part.legal_offsets[0]) == 0 and int(part.legal_offsets[-1]) == part.cell_pos.shape[0]
        assert part.n_cells == part.cell_pos.shape[0] and part.n_pos == part.moves_idx.shape[0]
        assert torch.all(part.cell_pos < part.n_pos)
    base = {"stone": off["stone"], "window": off["window"], "cell": off["cell"], "pos": off["pos"],
            "slot": off["pos"] * batch.max_w}
    for f in fields:
        rows, by = E._SPLIT_FIELDS[f]
        pieces = []
        for part, p0 in zip(parts, cuts):
            t = getattr(part, f).clone()
            if rows == "pos+1" and pieces:
                t = t[1:]
            if by is not None:
                t += int(base[by][p0])
            pieces.append(t)
        assert torch.equal(torch.cat(pieces), getattr(batch, f)), f
    # the source batch is untouched by the in-place rebasing
    assert int(batch.radius_src.max()) == int(off["stone"][-1]) - 1 or batch.radius_src.numel() == 0


@pytest.mark.parametrize("cut", [(0, 4), (4, 9), (3, 4)])
def test_relay_runs_derive_their_own_tables(cut):
    """The relay configuration's CSR views are rebuilt per run: a run's
    tables equal those of a batch collated from its positions alone."""
    specs = mb.engine.random_positions(9, 20, 120, seed=11)
    whole = mb.collate([mb.from_spec(s) for s in specs])
    cfg = mb.MantisConfig(h=32, blocks=1, heads=2)
    fields = E.needed_fields(cfg)
    assert E.split_supported(fields) and set(mb.builder.RELAY_FIELDS) <= set(fields)
    off = E._offsets(whole, fields)
    a, b = cut
    run = E.part_to_device(whole, fields, off, a, b, "cpu")
    own = mb.collate([mb.from_spec(s) for s in specs[a:b]])
    # (padded fields keep the parent batch's padding width, so only the
    # incidence and its derived views are compared)
    for f in mb.builder.RELAY_FIELDS + ("dec_cell", "dec_window", "dec_class"):
        assert torch.equal(getattr(run, f), getattr(own, f)), f


def test_range_points():
    assert E.range_points(5, 9, 0) == [5, 9]
    assert E.range_points(5, 9, 4) == [5, 9]
    assert E.range_points(0, 512, 448) == [0, 64, 512]
    pts = E.range_points(100, 1100, 448)
    assert pts[0] == 100 and pts[-1] == 1100 and all(a < b for a, b in zip(pts, pts[1:]))
    assert max(b - a for a, b in zip(pts, pts[1:])) <= 448


def test_narrow_batch_runs_equal_the_wide_ones():
    """Runs cut from a narrow (int32) batch are the wide batch's runs: the
    index fields are widened to int64 on the way to the device."""
    specs = mb.engine.random_positions(9, 20, 120, seed=11)
    wide = mb.encoder.encode(specs, threads=1)
    narrow = mb.encoder.encode(specs, threads=1, narrow=True)
    for knobs in (dict(cell_latents=True, cell_nodes=True), dict()):
        cfg = mb.MantisConfig(h=32, blocks=1, heads=2, **knobs)
        fields = E.needed_fields(cfg)
        ow, on = E._offsets(wide, fields), E._offsets(narrow, fields)
        for a, b in ((0, 4), (4, 9)):
            rw = E.part_to_device(wide, fields, ow, a, b, "cpu")
            rn = E.part_to_device(narrow, fields, on, a, b, "cpu")
            for f in fields:
                assert getattr(rn, f).dtype == getattr(rw, f).dtype, f
                assert torch.equal(getattr(rn, f), getattr(rw, f)), f
        dw, dn = E.to_device(wide, "cpu", fields), E.to_device(narrow, "cpu", fields)
        for f in fields:
            assert torch.equal(getattr(dn, f), getattr(dw, f)), f
