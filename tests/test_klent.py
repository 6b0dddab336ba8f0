"""KLENT policy improvement and move draw (mb_klent_improve,
ops.improved_policy): the CPU restatement against the reference's own
outputs (tests/golden/klent.npz, from klent/improve.py and the crate fixture
improvement.json), then the device kernel against both, and the draw against
the restated self-play sampling. Float tolerance: the reference computes in
float32, the kernel sums in float64, so 1e-5 relative (+1e-6 absolute)."""

from __future__ import annotations

import sys

import numpy as np
import pytest
import torch

from golden_io import REPO, load, mb

sys.path.insert(0, str(REPO))
from oracle import klent as K  # noqa: E402

RTOL, ATOL = 1e-5, 1e-6


def _cases():
    d = load("klent.npz")
    for i in range(int(d["n_cases"])):
        yield i, d, {k: d[f"{i}.{k}"] for k in ("logits", "score", "q", "offsets")}, float(d[f"{i}.tau"]), \
            float(d[f"{i}.lam"])


def _close(got, want, rtol=RTOL, atol=ATOL):
    got, want = np.asarray(got, np.float64), np.asarray(want, np.float64)
    assert got.shape == want.shape
    assert np.all(np.abs(got - want) <= atol + rtol * np.abs(want)), float(np.max(np.abs(got - want)))


def test_oracle_matches_reference_outputs():
    for i, d, a, tau, lam in _cases():
        p, v, kl, ne = K.improved_policy(a["logits"], a["score"], a["q"], a["offsets"], tau, lam)
        _close(p, d[f"{i}.probs"])
        _close(v, d[f"{i}.v_hat"])
        _close(kl, d[f"{i}.kl"], atol=1e-5)
        _close(ne, d[f"{i}.norm_entropy"], atol=1e-5)
        if f"{i}.fixture_pi" in d.files:  # the crate fixture's own expected values
            _close(p, d[f"{i}.fixture_pi"])
            _close(v[:1], [d[f"{i}.fixture_v"]])


@pytest.mark.gpu
def test_kernel_matches_reference_outputs():
    dev = torch.device("cuda")
    for i, d, a, tau, lam in _cases():
        t = {k: torch.from_numpy(np.ascontiguousarray(v)).to(dev) for k, v in a.items()}
        r = mb.ops.improved_policy(t["logits"], t["score"], t["q"], t["offsets"], tau, lam)
        torch.cuda.synchronize()
        _close(r.probs.cpu(), d[f"{i}.probs"])
        _close(r.v_hat.cpu(), d[f"{i}.v_hat"])
        _close(r.kl.cpu(), d[f"{i}.kl"], atol=1e-5)
        _close(r.norm_entropy.cpu(), d[f"{i}.norm_entropy"], atol=1e-5)
    mb._lib.check_device_error()


@pytest.mark.gpu
def test_draw_matches_restated_selfplay_sampling():
    """Ranks equal the restated self-play draw on ragged late-game-sized
    segments (cumulative sums per position on the device, over the batch in
    the restatement); stored policies and probabilities to float rounding."""
    dev = torch.device("cuda")
    rng = np.random.default_rng(3)
    widths = rng.integers(1, 9000, size=96)
    widths[:3] = [1, 2, 9000]
    off = np.concatenate([[0], np.cumsum(widths)]).astype(np.int64)
    n = int(off[-1])
    logits = (rng.standard_normal(n) * 2).astype(np.float32)
    score = rng.uniform(-1, 1, n).astype(np.float32)
    q = rng.uniform(-1, 1, n).astype(np.float32)
    u = rng.random(len(widths))
    u[:4] = [0.0, 0.5, 0.999999, 0.25]
    T = lambda x: torch.from_numpy(x).to(dev)  # noqa: E731
    imp, draw = mb.ops.improved_policy(T(logits), T(score), T(q), T(off), 0.1, 0.03, uniforms=torch.from_numpy(u))
    torch.cuda.synchronize()
    stored, ranks, top1, chosen = K.draw(imp.probs.cpu().numpy(), off, u)
    assert np.array_equal(draw.ranks.cpu().numpy(), ranks)
    _close(draw.stored.cpu(), stored, rtol=1e-6, atol=0)
    _close(draw.pi_top1.cpu(), top1, rtol=1e-12, atol=0)
    _close(draw.pi_chosen.cpu(), chosen, rtol=1e-12, atol=0)
    p, v, kl, ne = K.improved_policy(logits, score, q, off, 0.1, 0.03)
    _close(imp.probs.cpu(), p, rtol=2e-5, atol=1e-7)
    _close(imp.v_hat.cpu(), v, rtol=2e-5, atol=1e-6)
    mb._lib.check_device_error()


@pytest.mark.gpu
def test_argument_refusals():
    dev = torch.device("cuda")
    x = torch.zeros(4, device=dev)
    off = torch.tensor([0, 4], device=dev)
    with pytest.raises(ValueError, match="tau"):
        mb.ops.improved_policy(x, x, x, off, 0.0, 0.0)
    with pytest.raises(ValueError, match="same shape"):
        mb.ops.improved_policy(x, x, torch.zeros(3, device=dev), off, 0.1, 0.1)
    with pytest.raises(ValueError, match="one draw per position"):
        mb.ops.improved_policy(x, x, x, off, 0.1, 0.1, uniforms=torch.zeros(2, dtype=torch.float64))
