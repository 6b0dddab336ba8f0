"""One evaluator call over several devices (``network_evaluate_multi``): the
batch is cut into cost-balanced slices of positions, each evaluated on its own
device, and the host output equals the one-device evaluation (positions are
independent; the contract is the reference's batched == single tolerance).
With one visible GPU the devices are that GPU listed twice (two runners, two
weight replicas' worth of state, serialised by the device's lock). A lost
device is simulated on the host: a runner whose call raises before it
launches anything; its slice must be re-run on the other device."""

from __future__ import annotations

import pytest
import torch

from golden_io import mb

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _devices():
    n = torch.cuda.device_count()
    return [f"cuda:{i}" for i in range(n)] if n > 1 else ["cuda:0", "cuda:0"]


def _net(knobs):
    cfg = mb.MantisConfig(h=64, blocks=2, heads=4, **knobs)
    torch.manual_seed(5)
    net = mb.MantisNet(cfg)
    with torch.no_grad():
        for head in (net.mlp_p, net.mlp_q):
            head.out.weight.normal_(std=0.05)
    return net.to(DEV).eval()


KNOBS = [dict(cell_latents=True, cell_nodes=True), dict()]


@pytest.mark.parametrize("knobs", KNOBS, ids=["production", "relay"])
@pytest.mark.parametrize("autocast", [False, True])
def test_multi_device_equals_one_device(knobs, autocast):
    net = _net(knobs)
    specs = mb.engine.random_positions(23, 20, 160, seed=21)
    batch = mb.collate([mb.from_spec(s) for s in specs])
    cfg = mb.evaluator.EvaluatorConfig(device=DEV, autocast=autocast, part_positions=5)
    want = mb.network_evaluate(net, mb.evaluator.EvaluatorConfig(device=DEV, autocast=autocast, part_positions=0))(batch)
    multi = mb.evaluator.network_evaluate_multi(net, cfg, _devices())
    try:
        got = multi(batch)
        off = mb.evaluator._offsets(batch, multi.fields)
        cuts = mb.sharding.balanced_cuts(multi.costs(batch, off), len(multi.runners))
        assert all(a < b for a, b in zip(cuts, cuts[1:]))  # every device got positions
        for a, b in zip(got, want):
            torch.testing.assert_close(a, b, rtol=0, atol=1e-5 if not autocast else 1e-2)
        assert not multi.lost
    finally:
        multi.close()


def test_lost_device_slice_is_requeued():
    net = _net(KNOBS[0])
    specs = mb.engine.random_positions(12, 20, 120, seed=8)
    batch = mb.collate([mb.from_spec(s) for s in specs])
    cfg = mb.evaluator.EvaluatorConfig(device=DEV, autocast=True, part_positions=0)
    want = mb.network_evaluate(net, cfg)(batch)
    multi = mb.evaluator.network_evaluate_multi(net, cfg, _devices())
    try:
        def lost(*args, **kwargs):
            raise RuntimeError("device lost (host-side injection)")

        multi.runners[1].run_range = lost
        got = multi(batch)
        assert multi.lost == {1}
        for a, b in zip(got, want):
            torch.testing.assert_close(a, b, rtol=0, atol=1e-2)
        got = multi(batch)  # the next call runs on the remaining device alone
        for a, b in zip(got, want):
            torch.testing.assert_close(a, b, rtol=0, atol=1e-2)
    finally:
        multi.close()
