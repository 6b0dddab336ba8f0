"""The operator-level plug-in on the CPU: the ops defined in a namespace of
their own have the reference's argument lists and fake implementations (so
torch.compile keeps them opaque), and installing into the reference package
takes over every one of its forward ops."""

from __future__ import annotations

import pytest
import torch
from torch._subclasses.fake_tensor import FakeTensorMode

import reference_pkg
from golden_io import mb

torch_ops = __import__("importlib").import_module("hexo-shrimp-bot_b200.torch_ops")


def test_define_registers_every_op_with_fakes():
    names = torch_ops.define()
    assert len(names) == 12
    ns = torch.ops.mantis_b200
    with FakeTensorMode(allow_non_fake_inputs=False) as mode:
        f = lambda *s, dt=torch.bfloat16: torch.empty(*s, dtype=dt, device="cuda")
        i = lambda *s: torch.empty(*s, dtype=torch.long, device="cuda")
        q = f(3, 4, 40, 32)
        out, lse = ns.fused_attention(q, f(3, 4, 40, 32), f(3, 4, 40, 32), torch.empty(3, dtype=torch.int32,
                                                                                        device="cuda"))
        assert out.shape == q.shape and lse.shape == (3, 4, 40) and lse.dtype == torch.float32
        out, lse = ns.fused_attention(f(3, 4, 40, 32, dt=torch.float32), f(3, 4, 40, 32, dt=torch.float32),
                                      f(3, 4, 40, 32, dt=torch.float32), torch.empty(3, dtype=torch.int32,
                                                                                     device="cuda"))
        assert lse.numel() == 0
        o, m, l = ns.cell_attention(f(7, 8, 32), f(5, 8, 32), f(5, 8, 32), f(8, 11, dt=torch.float32),
                                    f(11, 256), i(8), i(9), i(9), i(9), i(6), i(9), i(9), i(12), i(9))
        assert o.shape == (7, 8, 32) and o.dtype == torch.float32 and m.shape == (7, 8)
        o, m, l = ns.window_latent_read(f(2, 4, 8, 32), f(9, 8, 32), f(9, 8, 32), i(9), i(3), i(9))
        assert o.shape == (2, 4, 8, 32) and l.shape == (2, 4, 8)
        r = ns.aggregate_to_stones(f(9, 64), i(20), i(20), i(20), i(20), 13)
        assert r.shape == (13, 64) and r.dtype == torch.float32
        r = ns.action_row_encode(f(9, 64), f(11, 64, dt=torch.float32), i(20), i(20), i(20), i(20), 6)
        assert r.shape == (6, 64)
        off, order = ns.window_latent_layout(i(9), 4)
        assert off.shape == (5,) and order.shape == (9,)
    assert torch_ops.define() == names  # idempotent


def test_compile_keeps_the_ops_opaque():
    """A graph calling a plug-in op traces under the fake implementation."""
    torch_ops.define()

    def fn(values, inc_stone, inc_window, run_stone, run_window):
        return torch.ops.mantis_b200.aggregate_to_windows(values, inc_stone, inc_window, run_stone, run_window, 5) * 2

    from torch._dynamo.testing import CompileCounterWithBackend
    cnt = CompileCounterWithBackend("eager")
    with FakeTensorMode():
        args = (torch.empty(9, 64, device="cuda"),) + tuple(torch.empty(12, dtype=torch.long, device="cuda")
                                                             for _ in range(4))
    gm = torch.fx.experimental.proxy_tensor.make_fx(fn, tracing_mode="fake")(*args)
    assert any("mantis_b200.aggregate_to_windows" in str(n.target) for n in gm.graph.nodes)


@pytest.mark.skipif(not reference_pkg.available(), reason="reference not installed in baseline/_ref")
def test_install_takes_over_the_reference_ops():
    mn = reference_pkg.load()
    for mod in ("attention", "cell_latents", "window_latents", "message_passing", "row_encoder", "relay"):
        __import__(f"mantisnet.{mod}")
    taken = torch_ops.install_into_reference()
    names = {t.split("::")[1] for t in taken}
    assert {"fused_attention", "cell_attention", "cell_attention_plain", "window_latent_read",
            "window_latent_broadcast", "cell_pass", "window_latent_layout"} <= names
    assert mn.MantisConfig  # the package itself imported
