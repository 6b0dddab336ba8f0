"""CPU restatement of the KLENT policy-improvement step and the self-play
move draw — test infrastructure.

Only tests/ use this module; the product path (the library's
``mb_klent_improve`` kernel) never does.

- ``improved_policy`` follows python/mantisnet/mantisnet/klent/improve.py:27-69
  (eq. 3 of the KLENT note): per position, log pi = log-softmax(logits),
  pi' = softmax((q_score + tau log pi) / (tau + lam)), and the pi'-weighted
  means of the action value, of log pi' - log pi (the KL) and of -log pi'
  (the entropy, normalised by log |A|, zero for a single legal cell), each
  divided by the segment's pi' mass. Computed in float64 here; the
  reference computes in the inputs' float32, so parity is a tolerance.
  Pinned by ``tests/golden/klent.npz`` (the reference function's outputs,
  and its crate fixture's expected values).
- ``draw`` follows the sampling of python/mantisnet/mantisnet/klent/selfplay.py:180-190:
  pi' renormalised per position in float64, one uniform per position, the
  move rank = the first cell whose cumulative probability reaches the
  uniform, clipped to the segment; also the stored float32 policy, the
  largest probability and the chosen one. Parity unpinned by reference
  vectors: the reference draws inside a self-play object, so this step is a
  restatement of those lines. Its cumulative sums run over the whole batch
  as the reference's do.
"""

from __future__ import annotations

import numpy as np


def _segment_log_softmax(x: np.ndarray, offsets: np.ndarray) -> np.ndarray:
    out = np.empty_like(x)
    for a, b in zip(offsets[:-1], offsets[1:]):
        s = x[a:b] - x[a:b].max()
        out[a:b] = s - np.log(np.exp(s).sum())
    return out


def improved_policy(logits, score, q, offsets, tau: float, lam: float):
    """(probs, v_hat, kl, norm_entropy) in float64."""
    offsets = np.asarray(offsets, np.int64)
    log_pi = _segment_log_softmax(np.asarray(logits, np.float64), offsets)
    z = (np.asarray(score, np.float64) + tau * log_pi) / (tau + lam)
    log_imp = _segment_log_softmax(z, offsets)
    probs = np.exp(log_imp)
    p = len(offsets) - 1
    v_hat, kl, ent = np.zeros(p), np.zeros(p), np.zeros(p)
    qq = np.asarray(q, np.float64)
    for i, (a, b) in enumerate(zip(offsets[:-1], offsets[1:])):
        m = probs[a:b].sum()
        v_hat[i] = (probs[a:b] * qq[a:b]).sum() / m
        kl[i] = (probs[a:b] * (log_imp[a:b] - log_pi[a:b])).sum() / m
        ent[i] = (-probs[a:b] * log_imp[a:b]).sum() / m
    counts = np.diff(offsets)
    norm_ent = np.where(counts > 1, ent / np.log(np.maximum(counts, 2)), 0.0)
    return probs, v_hat, kl, norm_ent


def draw(probs, offsets, uniforms):
    """(stored float32 policy, ranks, pi_top1, pi_chosen) from pi' (float32
    as the improvement step returns it) and one uniform per position."""
    offsets = np.asarray(offsets, np.int64)
    flat = np.asarray(probs, np.float32).astype(np.float64)
    widths = np.diff(offsets)
    flat /= np.repeat(np.add.reduceat(flat, offsets[:-1]), widths)
    cdf = np.cumsum(flat)
    base = np.concatenate(([0.0], cdf[offsets[1:-1] - 1]))
    ranks = np.searchsorted(cdf, base + np.asarray(uniforms, np.float64)) - offsets[:-1]
    ranks = np.clip(ranks, 0, widths - 1)
    return flat.astype(np.float32), ranks.astype(np.int64), np.maximum.reduceat(flat, offsets[:-1]), \
        flat[offsets[:-1] + ranks]
