"""Batched Gumbel root sampling with sequential halving over leaf batches
(the evaluation chooser of the reference's KLENT, klent/search.py:92-268),
with every leaf wave evaluated on the GPU.

``gumbel_choose(evaluate, tau, lam, sims, rng, temperature)`` returns a
chooser ``choose(positions, rng) -> moves`` with the reference's contract and
decisions:

- the root batch is evaluated once; ``sims == 0`` picks each root's
  policy-logit argmax; a root with fewer than one candidate
  (``min(16, sims // 2, legal count)``) too;
- each root draws ``temperature * Gumbel(0, 1)`` per legal move from its own
  generator (one uint64 seed per root from the caller's generator, so batched
  and one-at-a-time calls draw the same numbers) and keeps the top
  ``m`` moves of noise + logit as candidate lines, each advanced one move;
- the budget is spent by the halving schedule (``halving_schedule``): each
  round deepens every surviving line ``deepenings`` times, a wave at a time
  over all roots' lines; a line's leaf is evaluated, KLENT-improved and
  advanced along the improved policy's argmax; its value is the improved
  value in the root mover's frame (terminal lines keep +1 / -1); after a
  round the better half of each root's lines (by value) survive;
- the move is the surviving line with the largest
  ``gumbel + logit + (C_VISIT + max visits) * C_SCALE * value``.

B200 specifics: a leaf wave's positions are encoded by the native encoder and
evaluated by an evaluator's ``leaves(batch, tau, lam)`` when it has one
(``evaluator.network_leaf_evaluate``): the forward, the KLENT improvement and
the per-leaf argmax all run on the device and only (rank, value) per leaf
crosses back. A plain ``evaluate(batch)`` returning CPU (logits, q_score,
q_values) is improved with the library's kernels as well.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import numpy as np
import torch

from . import encoder, ops

# Gumbel MuZero's root value transform (the reference's constants).
C_VISIT = 50
C_SCALE = 1.0
MAX_CANDIDATES = 16


def halving_schedule(sims: int, candidates: int) -> list[tuple[int, int]]:
    """``(survivors, deepenings per survivor)`` per round: deepenings double
    between rounds while the budget allows, the last possible round takes
    the remaining equal share, and a remainder smaller than the survivor
    count stays unspent (reference search.py:47-76)."""
    if sims < 0:
        raise ValueError(f"the simulation budget must be >= 0 (got {sims})")
    if candidates < 1:
        raise ValueError(f"a search needs at least one candidate (got {candidates})")
    n_rounds = max(1, math.ceil(math.log2(candidates)))
    left, alive, plan = sims, candidates, []
    for r in range(n_rounds):
        if left < alive:
            break
        share = left // alive
        depth = share if r == n_rounds - 1 else min(1 << r, share)
        if depth < 1:
            break
        plan.append((alive, depth))
        left -= alive * depth
        alive = (alive + 1) // 2
    return plan


@dataclass
class _Line:
    root_rank: int
    root_logit: float
    gumbel: float
    position: object
    value: float
    terminal: bool
    policy_rank: int | None = None
    visits: int = 0


@dataclass
class _Root:
    player: int
    lines: list[_Line]
    survivors: list[int]
    plan: list[tuple[int, int]]
    trace: list[list[int]] = field(default_factory=list)


def _outcome(position, root_player: int) -> float:
    return 1.0 if position.winner == root_player else -1.0


def _specs(positions):
    return [p.spec() for p in positions]


def _leaf_values(evaluate, positions, tau: float, lam: float):
    """(improved-policy argmax rank, improved value) per leaf, on the device."""
    batch = encoder.encode(_specs(positions))
    if hasattr(evaluate, "leaves"):
        return evaluate.leaves(batch, tau, lam)
    logits, q_score, q_values = evaluate(batch)
    dev = torch.device("cuda", torch.cuda.current_device())
    off = batch.legal_offsets.to(dev)
    imp = ops.improved_policy(logits.to(dev), q_score.to(dev), q_values.to(dev), off, tau, lam)
    ranks = ops.segment_argmax(imp.probs, off)
    return ranks.cpu(), imp.v_hat.cpu()


def gumbel_choose(evaluate, tau: float, lam: float, sims: int, rng=None, temperature: float = 1.0, trace=None,
                  root_noise=None):
    """The batched Gumbel chooser (see the module docstring). ``trace``, a
    list, receives each root's surviving candidate ranks after every
    halving (the first entry: the candidates). ``root_noise(k, n)``, when
    given, replaces root k's ``n`` Gumbel draws (before the temperature)."""
    if sims < 0:
        raise ValueError(f"the simulation budget must be >= 0 (got {sims})")
    if not math.isfinite(temperature) or temperature < 0.0:
        raise ValueError(f"temperature must be finite and >= 0 (got {temperature})")
    if sims == 0 and temperature != 1.0:
        raise ValueError(f"temperature={temperature} needs sims > 0: a zero budget is the policy argmax and draws "
                         "no noise to scale")

    def choose(positions, call_rng=None):
        if not positions:
            return []
        parent = call_rng if call_rng is not None else rng
        if parent is None:
            raise ValueError("the Gumbel chooser needs a random generator")
        root_batch = encoder.encode(_specs(positions))
        logits, _, _ = evaluate(root_batch)
        logits = logits.float().cpu()
        off = root_batch.legal_offsets.tolist()
        if sims == 0:
            return [pos.nth_legal(int(logits[off[k]:off[k + 1]].argmax())) for k, pos in enumerate(positions)]
        seeds = parent.integers(0, np.iinfo(np.uint64).max, size=len(positions), dtype=np.uint64)
        roots: list[_Root | None] = []
        fallback: list[int] = []
        for k, pos in enumerate(positions):
            lo, hi = off[k], off[k + 1]
            row = logits[lo:hi].numpy()
            n_legal = hi - lo
            m = min(MAX_CANDIDATES, sims // 2, n_legal)
            if m < 1:
                roots.append(None)
                fallback.append(int(logits[lo:hi].argmax()))
                continue
            noise = (root_noise(k, n_legal) if root_noise is not None
                     else np.random.default_rng(seeds[k]).gumbel(size=n_legal))
            g = np.asarray(noise, dtype=np.float64) * temperature
            picked = np.argsort(-(g + row), kind="stable")[:m]
            lines = []
            for rank in picked:
                child = pos.copy()
                child.advance(*pos.nth_legal(int(rank)))
                lines.append(_Line(int(rank), float(row[rank]), float(g[rank]), child,
                                   _outcome(child, pos.current_player) if child.is_terminal else 0.0,
                                   bool(child.is_terminal)))
            root = _Root(pos.current_player, lines, list(range(m)), halving_schedule(sims, m))
            root.trace.append([lines[i].root_rank for i in root.survivors])
            roots.append(root)
            fallback.append(-1)

        live = [r for r in roots if r is not None]
        for rnd in range(max((len(r.plan) for r in live), default=0)):
            active = [r for r in live if rnd < len(r.plan)]
            for wave in range(max(r.plan[rnd][1] for r in active)):
                pending = []
                for r in active:
                    if wave >= r.plan[rnd][1]:
                        continue
                    for i in r.survivors:
                        line = r.lines[i]
                        if line.terminal:
                            continue
                        if line.policy_rank is not None:  # deepen along the improved policy
                            child = line.position.copy()
                            child.advance(*line.position.nth_legal(line.policy_rank))
                            line.position = child
                            if child.is_terminal:
                                line.terminal = True
                                line.value = _outcome(child, r.player)
                                line.visits += 1
                                continue
                        pending.append((r, line))
                if not pending:
                    continue
                ranks, values = _leaf_values(evaluate, [line.position for _, line in pending], tau, lam)
                for j, (r, line) in enumerate(pending):
                    line.policy_rank = int(ranks[j])
                    sign = 1.0 if line.position.current_player == r.player else -1.0
                    line.value = sign * float(values[j])
                    line.visits += 1
            for r in active:
                ordered = sorted(r.survivors, key=lambda i: r.lines[i].value, reverse=True)
                r.survivors = ordered[:(len(ordered) + 1) // 2]
                r.trace.append([r.lines[i].root_rank for i in r.survivors])

        moves = []
        for k, (pos, r) in enumerate(zip(positions, roots)):
            if r is None:
                moves.append(pos.nth_legal(fallback[k]))
                continue
            top = max(line.visits for line in r.lines)
            best = max(r.survivors, key=lambda i: (r.lines[i].gumbel + r.lines[i].root_logit
                                                   + (C_VISIT + top) * C_SCALE * r.lines[i].value))
            moves.append(pos.nth_legal(r.lines[best].root_rank))
            if trace is not None:
                trace.append(r.trace)
        return moves

    return choose
