"""Host side of the isolated-op workloads (CPU): the cell-token sets and the
six-slot neighbour table against a direct restatement of the reference
adjacency walk (builder.py:458-471), and the CPU restatements' own identities."""

from __future__ import annotations

import numpy as np
import torch

from golden_io import mb
from oracle import isolated as ISO

HG = mb.hexgraph


def _walk(tokens):
    """The reference adjacency loop restated over tokens: for each token,
    axes Q, R, QR and signs -1, +1 in that order."""
    index = {tuple(map(int, t)): i for i, t in enumerate(tokens)}
    table = []
    for t in tokens:
        row = []
        for axis in range(3):
            for sign in (-1, 1):
                nb = (int(t[0]) + sign * int(mb.vocab.AXES[axis][0]), int(t[1]) + sign * int(mb.vocab.AXES[axis][1]))
                row.append(index.get(nb, -1))
        table.append(row)
    return np.asarray(table, dtype=np.int32).reshape(-1, 6)


def test_tokens_sorted_and_within_radius():
    spec = mb.engine.random_positions(1, 30, 30, seed=4)[0]
    tok = HG.cell_tokens(spec.stone_qr, 2)
    keys = [tuple(t) for t in tok]
    assert keys == sorted(keys) and len(set(keys)) == len(keys)
    d = np.abs(tok[:, None, :] - spec.stone_qr[None, :, :])
    dist = np.maximum(np.maximum(d[..., 0], d[..., 1]), np.abs((tok[:, None, 0] + tok[:, None, 1])
                                                                 - (spec.stone_qr[None, :, 0] + spec.stone_qr[None, :, 1])))
    assert np.all(dist.min(1) <= 2)
    assert {tuple(s) for s in spec.stone_qr} <= set(keys)


def test_neighbour_table_matches_reference_walk():
    for seed, stones in ((1, 40), (2, 120), (3, 200)):
        spec = mb.engine.random_positions(1, stones, stones, seed=seed)[0]
        tok = HG.cell_tokens(spec.stone_qr, 2)
        length = 256
        got = HG.neighbour_table(tok, length, row0=1000)
        kept = tok[:length]
        want = _walk(kept)
        want = np.where(want >= 0, want + 1000, -1)
        n = len(kept)
        assert np.array_equal(got[:n], want)
        assert np.all(got[n:] == -1)
        # symmetry: slot 2a and 2a+1 are opposite steps
        for i in range(n):
            for s in range(6):
                j = got[i, s]
                if j >= 0:
                    assert got[j - 1000, s ^ 1] == i + 1000


def test_message_graph_layout():
    nbr, counts = HG.message_graph(5, 256, 40, 200, seed=9)
    assert nbr.shape == (5 * 256, 6) and nbr.dtype == np.int32
    for p in range(5):
        block = nbr[p * 256:(p + 1) * 256]
        live = block[block >= 0]
        assert np.all((live >= p * 256) & (live < p * 256 + counts[p]))
        assert np.all(block[counts[p]:] == -1)


def test_attention_layout():
    coords, valid = HG.attention_layout(6, 256, seed=3)
    assert coords.shape == (6, 256, 2) and valid.shape == (6,)
    assert np.all((valid >= 32) & (valid <= 256))
    for c in coords:
        keys = [tuple(t) for t in c]
        assert keys == sorted(keys) and len(set(keys)) == 256


def test_oracle_identities():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(20, 8, generator=g, dtype=torch.float64)
    nbr = torch.randint(-1, 20, (20, 6), generator=g)
    w = torch.zeros(8, 8, dtype=torch.float64)
    b = torch.randn(8, generator=g, dtype=torch.float64)
    torch.testing.assert_close(ISO.hex_message_pass(x, nbr, w, b), x + b)
    # the mean over present neighbours, by hand for one row
    w = torch.eye(8, dtype=torch.float64)
    y = ISO.hex_message_pass(x, nbr, w, None)
    r = 3
    pres = [int(j) for j in nbr[r] if j >= 0]
    want = x[r] + (x[pres].mean(0) if pres else 0)
    torch.testing.assert_close(y[r], want)
    # zero bias: the masked softmax attention of torch's SDPA
    p, h, length, d = 2, 3, 16, 32
    q, k, v = (torch.randn(p, h, length, d, generator=g, dtype=torch.float64) for _ in range(3))
    coords = torch.randint(-5, 5, (p, length, 2), generator=g, dtype=torch.int32)
    valid = torch.tensor([16, 9], dtype=torch.int32)
    out = ISO.axial_attention(q, k, v, coords, valid, torch.zeros(33, 33, h, dtype=torch.float64))
    mask = (torch.arange(length)[None, :] < valid[:, None])[:, None, None, :]
    ref = torch.nn.functional.scaled_dot_product_attention(q, k, v, attn_mask=mask)
    live = (torch.arange(length)[None, :] < valid[:, None])[:, None, :, None]
    torch.testing.assert_close(out, torch.where(live, ref, torch.zeros(())))
