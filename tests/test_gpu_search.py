"""The Gumbel search on the GPU: the reference's cross-language parity
fixture (crates/hexo-search/tests/fixtures/gumbel_parity.json, read into
tests/golden/gumbel.npz by make_golden_klent.py) replayed with its scripted
evaluator and root noise — same candidates, same survivors after every
round, same move — and the chooser on a real model through the device leaf
evaluator: batched equals one root at a time, sims = 0 is the argmax."""

from __future__ import annotations

import json

import numpy as np
import pytest
import torch

import golden_io
from golden_io import mb

pytestmark = pytest.mark.gpu
search = mb.search
eng = mb.engine


def _fixture():
    d = golden_io.load("gumbel.npz")
    return json.loads(str(d["fixture"]))


def _scripted(case):
    calls = case["scripted_calls"]
    seen = []

    def evaluate(batch):
        call = calls[len(seen)]
        offsets = batch.legal_offsets.tolist()
        counts = [b - a for a, b in zip(offsets[:-1], offsets[1:])]
        assert counts == call["legal_counts"], (call["phase"], counts)
        raw = call["raw_policy_logits"]
        logits = torch.full((offsets[-1],), raw["fill"], dtype=torch.float32)
        q = torch.empty(offsets[-1], dtype=torch.float32)
        for row, (a, b) in enumerate(zip(offsets[:-1], offsets[1:])):
            for o in raw.get("overrides", []):
                logits[a + o["rank"]] = o["value"]
            q[a:b] = call["raw_q_fill"][row]
        seen.append(call["phase"])
        return logits, q.clone(), q

    return evaluate, seen


class _ZeroSeed:
    def integers(self, low, high, size, dtype):
        return np.zeros(size, dtype=np.uint64)


def test_gumbel_parity_fixture():
    fx = _fixture()
    for case in fx["cases"]:
        cfgc = case["config"]
        evaluate, seen = _scripted(case)
        noise = np.asarray(case["root_gumbel_noise"], dtype=np.float64)
        trace = []
        choose = search.gumbel_choose(evaluate, cfgc["tau"], cfgc["lambda"], cfgc["sims"], trace=trace,
                                      root_noise=lambda k, n: noise[:n])
        root = eng.Position.replay(case["position_prefix"])
        move = choose([root], _ZeroSeed())[0]
        exp = case["expected"]
        assert seen == [c["phase"] for c in case["scripted_calls"]]
        assert trace[0][0] == case["candidate_root_ranks"]
        assert trace[0][1:] == exp["survivor_root_ranks_after_round"]
        assert list(move) == exp["chosen_move"] and root.legal_moves().index(move) == exp["chosen_root_rank"]


@pytest.fixture(scope="module")
def leaf_model():
    cfg = mb.MantisConfig(h=64, blocks=2, heads=2, cell_latents=True, cell_nodes=True)
    torch.manual_seed(4)
    net = mb.MantisNet(cfg)
    with torch.no_grad():
        for head in (net.mlp_p, net.mlp_q):
            head.out.weight.normal_(std=0.5)
            head.out.bias.normal_(std=0.5)
    net = net.cuda().eval()
    return mb.evaluator.network_leaf_evaluate(net, mb.evaluator.EvaluatorConfig(device="cuda", autocast=False))


def _roots(n, seed):
    out = []
    for i, spec_seed in enumerate(range(seed, seed + n)):
        moves = []
        pos = eng.Position()
        rng = __import__("random").Random(spec_seed)
        for _ in range(6 + 3 * i):
            pos.advance(*pos.random_legal(rng))
        out.append(pos)
    return out


def test_leaf_step_matches_the_closure(leaf_model):
    """leaves() = argmax of the improved policy and its value, from the
    closure's own outputs improved by the library."""
    roots = _roots(3, 40)
    batch = mb.encoder.encode([p.spec() for p in roots])
    ranks, values = leaf_model.leaves(batch, 0.1, 0.03)
    logits, q_score, q_values = leaf_model(batch)
    off = batch.legal_offsets.cuda()
    imp = mb.ops.improved_policy(logits.cuda(), q_score.cuda(), q_values.cuda(), off, 0.1, 0.03)
    o = batch.legal_offsets.tolist()
    for k in range(3):
        assert int(ranks[k]) == int(imp.probs[o[k]:o[k + 1]].argmax())
    torch.testing.assert_close(values, imp.v_hat.cpu(), rtol=1e-5, atol=1e-6)


def test_chooser_batched_equals_single_and_argmax(leaf_model):
    roots = _roots(4, 7)
    choose = search.gumbel_choose(leaf_model, 0.1, 0.03, sims=12)
    batched = choose(roots, np.random.default_rng(5))
    seeds = np.random.default_rng(5).integers(0, np.iinfo(np.uint64).max, size=4, dtype=np.uint64)

    class _One:
        def __init__(self, s):
            self.s = s

        def integers(self, low, high, size, dtype):
            return np.asarray([self.s], dtype=np.uint64)

    single = [choose([r], _One(s))[0] for r, s in zip(roots, seeds)]
    assert batched == single
    for r, m in zip(roots, batched):
        assert m in r.legal_moves()
    greedy = search.gumbel_choose(leaf_model, 0.1, 0.03, sims=0)(roots, np.random.default_rng(0))
    batch = mb.encoder.encode([p.spec() for p in roots])
    logits = leaf_model(batch)[0]
    o = batch.legal_offsets.tolist()
    assert greedy == [r.nth_legal(int(logits[o[k]:o[k + 1]].argmax())) for k, r in enumerate(roots)]
    mb._lib.check_device_error()
