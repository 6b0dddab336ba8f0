"""Golden vectors of the KLENT policy-improvement step, from the reference.

Run where the reference checkout is available (the committed ``klent.npz``
travels instead):

    python tests/golden/make_golden_klent.py --reference <path to the reference checkout>

It imports the reference's ``mantisnet.klent.improve.improved_policy``
(python/mantisnet/mantisnet/klent/improve.py:27-69) with the same
``hexo_py`` stub as ``make_golden.py``, and records its outputs for

- the cases of the reference's own fixture
  ``crates/models/mantisnet/tests/fixtures/improvement.json`` (inputs and the
  fixture's expected pi' and v_hat, read from the checkout at generation
  time), each as a one-position batch;
- seeded random batches: ragged segments (1 to 3,000 cells, one single-cell
  segment), logits, acting scores and action values in the ranges the
  evaluator produces, four (tau, lambda) settings.

It also carries the Gumbel search's parity fixture
``crates/hexo-search/tests/fixtures/gumbel_parity.json`` (scripted evaluator
calls, root noise, expected survivors and move) into ``gumbel.npz``.
"""

from __future__ import annotations

import argparse
import importlib
import json
import os
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def _import_improve(checkout: Path):
    stub = types.ModuleType("hexo_py")
    stub.MODEL_REPR_VERSION = 9
    sys.modules["hexo_py"] = stub
    sys.path.insert(0, str(checkout / "python" / "mantisnet"))
    return importlib.import_module("mantisnet.klent.improve")


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("HEXO_REFERENCE"),
                    help="path to the reference checkout (the directory holding python/ and crates/)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference <checkout> or set HEXO_REFERENCE")
    checkout = Path(args.reference)
    imp = _import_improve(checkout)
    out = {}
    cases = json.loads((checkout / "crates/models/mantisnet/tests/fixtures/improvement.json").read_text())["cases"]
    batches = []
    for c in cases:
        n = len(c["policy_logits"])
        q = np.asarray(c["q_values"], np.float32)
        batches.append(dict(name=c["name"], logits=np.asarray(c["policy_logits"], np.float32), score=q, q=q,
                            offsets=np.array([0, n], np.int64), tau=float(c["tau"]), lam=float(c["lambda"]),
                            fixture_pi=np.asarray(c["expected_pi_prime"], np.float64),
                            fixture_v=np.float64(c["expected_v_hat"])))
    rng = np.random.default_rng(7)
    for b, (tau, lam) in enumerate([(0.1, 0.03), (0.03, 0.1), (0.0, 1.0), (1.0, 0.0)]):
        widths = rng.integers(1, 3000, size=12)
        widths[3] = 1
        offsets = np.concatenate([[0], np.cumsum(widths)]).astype(np.int64)
        n = int(offsets[-1])
        batches.append(dict(name=f"random{b}", logits=(rng.standard_normal(n) * 3).astype(np.float32),
                            score=rng.uniform(-1, 1, n).astype(np.float32),
                            q=rng.uniform(-1, 1, n).astype(np.float32), offsets=offsets, tau=tau, lam=lam))
    out["n_cases"] = np.int64(len(batches))
    for i, b in enumerate(batches):
        r = imp.improved_policy(torch.from_numpy(b["logits"]), torch.from_numpy(b["score"]), torch.from_numpy(b["q"]),
                                torch.from_numpy(b["offsets"]), b["tau"], b["lam"])
        for k in ("logits", "score", "q", "offsets"):
            out[f"{i}.{k}"] = b[k]
        out[f"{i}.tau"] = np.float64(b["tau"])
        out[f"{i}.lam"] = np.float64(b["lam"])
        out[f"{i}.probs"] = r.probs.numpy()
        out[f"{i}.v_hat"] = r.v_hat.numpy()
        out[f"{i}.kl"] = r.kl.numpy()
        out[f"{i}.norm_entropy"] = r.norm_entropy.numpy()
        if "fixture_pi" in b:
            out[f"{i}.fixture_pi"] = b["fixture_pi"]
            out[f"{i}.fixture_v"] = b["fixture_v"]
    np.savez_compressed(HERE / "klent.npz", **out)
    print("wrote", HERE / "klent.npz", len(batches), "cases")
    # the Gumbel search's cross-language parity fixture, carried as is
    gumbel = (checkout / "crates/hexo-search/tests/fixtures/gumbel_parity.json").read_text()
    np.savez_compressed(HERE / "gumbel.npz", fixture=np.array(json.dumps(json.loads(gumbel))))
    print("wrote", HERE / "gumbel.npz")


if __name__ == "__main__":
    main()
