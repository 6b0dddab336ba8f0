"""The reference's own MantisNet and KLENT evaluator (python/mantisnet/
mantisnet/model.py, klent/train.py:100-120, installed in baseline/_ref)
running its mantisnet:: op calls on this library's kernels through the
plug-in (torch_ops.install_into_reference): the config-1 production model,
fp32 against the reference's eager-CPU fp32 outputs at 1e-4 relative, and
bf16 autocast within the north_star bf16 contract."""

from __future__ import annotations

import importlib

import pytest
import torch

import golden_io
import reference_pkg
from golden_io import mb

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not reference_pkg.available(), reason="reference not installed in baseline/_ref")]
torch_ops = importlib.import_module("hexo-shrimp-bot_b200.torch_ops")


@pytest.fixture(scope="module")
def reference_setup():
    mn = reference_pkg.load()
    train = importlib.import_module("mantisnet.klent.train")
    for mod in ("attention", "cell_latents", "window_latents", "message_passing", "row_encoder", "relay"):
        importlib.import_module(f"mantisnet.{mod}")
    taken = torch_ops.install_into_reference()
    assert len(taken) >= 10, taken
    cfg, P, _, want, mf = golden_io.config1_case("prod")
    net = mn.MantisNet(mn.MantisConfig(**{k: v for k, v in cfg.items()})).eval()
    net.load_state_dict(P, strict=True)
    specs = mb.engine.random_positions(16, 10, 40, seed=golden_io.CONFIG1_POSITIONS_SEED)
    graphs = [mn.builder.build(s.stone_qr, s.stone_owner, s.mover, s.legal_qr, s.moves_remaining) for s in specs]
    return train, net.to("cuda"), mn.builder.collate(graphs), want, mf


@pytest.mark.parametrize("autocast", [False, True])
def test_reference_evaluator_on_plugin_kernels(reference_setup, autocast):
    train, net, batch, want, mf = reference_setup
    ev = train.network_evaluate(net, train.KlentConfig(device="cuda", autocast=autocast, mass_floor=mf))
    calls = mb._lib.call_count()
    policy, q_score, q_values = ev(batch)
    assert mb._lib.call_count() > calls, "the plug-in's kernels did not run"
    if autocast:
        assert (policy - want["policy_logits"]).abs().max() <= 2e-2
        assert (q_values - want["q_values"]).abs().max() <= 1e-2
    else:
        for got, k in ((policy, "policy_logits"), (q_values, "q_values"), (q_score, "q_score")):
            scale = want[k].abs().max().clamp(min=1e-6)
            assert (got - want[k]).abs().max() <= 1e-4 * scale, k
    mb._lib.check_device_error()


def test_reference_training_gradients_on_plugin_kernels(reference_setup):
    """The fit path: gradients of a loss on the reference model's policy and
    critic outputs (fp32), through the reference's own autograd formulas
    whose backward ops run on this library's kernels, against the same
    gradients on the reference's eager CPU path."""
    train, net, batch, want, mf = reference_setup
    import copy
    cpu_net = copy.deepcopy(net).to("cpu")

    def loss_grads(model, b):
        model.zero_grad(set_to_none=True)
        w, g, cells = model.trunk(b)
        policy, critic = model.cell_head_logits(w, g, cells, b)
        (policy.float().square().mean() + critic.float().square().mean()).backward()
        return {n: p.grad.detach().float().cpu() for n, p in model.named_parameters() if p.grad is not None}

    got = loss_grads(net, batch.to("cuda"))
    ref = loss_grads(cpu_net, batch)
    assert set(got) == set(ref) and len(got) > 50
    for n in ref:
        scale = ref[n].abs().max().clamp(min=1e-8)
        assert (got[n] - ref[n]).abs().max() <= 1e-3 * scale, n
    mb._lib.check_device_error()
