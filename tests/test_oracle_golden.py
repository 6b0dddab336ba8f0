"""Pins the CPU oracle against the reference's own outputs: the fixtures hold
the reference eager-CPU fp32 forward on seeded weights and positions."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import golden_io
from oracle import forward as O


def _cfg(cfg: dict) -> O.Cfg:
    return O.Cfg(**{k: v for k, v in cfg.items() if k != "dropout"})


@pytest.mark.parametrize("name", golden_io.FORWARD_CASES)
def test_oracle_forward_matches_reference(name):
    cfg, P, batch, want, mf = golden_io.forward_case(name)
    got = O.forward(_cfg(cfg), P, batch, mf)
    for k in ("policy_logits", "critic_logits", "q_score", "q_values", "value", "value_dist", "value_logits",
              "trunk_g"):
        torch.testing.assert_close(got[k], want[k], rtol=1e-4, atol=1e-5, msg=f"{name}:{k}")


def test_oracle_ops_match_reference():
    d = golden_io.load("ops.npz")
    t = {k: torch.from_numpy(d[k]) for k in d.files}
    out = O.stone_attention(t["att.q"], t["att.k"], t["att.v"], t["att.seq_lens"].long())
    torch.testing.assert_close(out, t["att.out"], rtol=1e-5, atol=1e-6)
    seg = O.segment_attention(t["seg.q"], t["seg.k"], t["seg.v"], t["seg.bias"], t["seg.vcls"],
                              t["seg.src"], t["seg.cls"], t["seg.qid"])
    torch.testing.assert_close(seg, t["seg.out"], rtol=1e-5, atol=1e-6)
    assert torch.count_nonzero(seg[2]) == 0  # empty run reads zero
    seg = O.segment_attention(t["seg.q"], t["seg.k"], t["seg.v"], t["seg.bias"], None,
                              t["seg.src"], t["seg.cls"], t["seg.qid"])
    torch.testing.assert_close(seg, t["seg.out_plain"], rtol=1e-5, atol=1e-6)
    rd = O.window_read(t["win.rq"], t["win.rk"], t["win.rv"], t["win.pos"])
    torch.testing.assert_close(rd, t["win.read"], rtol=1e-5, atol=1e-6)
    assert torch.count_nonzero(rd[1]) == 0  # empty position reads zero
    bc = O.window_broadcast(t["win.bq"], t["win.bk"], t["win.bv"], t["win.pos"])
    torch.testing.assert_close(bc, t["win.bcast"], rtol=1e-5, atol=1e-6)
    rows = O.encode_rows(t["row.pre"], t["row.table"], t["row.win"], t["row.cls"], t["row.cell"], 5)
    torch.testing.assert_close(rows, t["row.out"], rtol=1e-5, atol=1e-6)


def test_oracle_fresh_decoder_zero_init_gives_zero_values():
    """Reference test_model.py:164-172: zeroed decoder outputs make every
    policy logit and action value exactly zero."""
    cfg, P, batch, _, mf = golden_io.forward_case("cellnodes")
    P = dict(P)
    for k in ("mlp_p.out.weight", "mlp_p.out.bias", "mlp_q.out.weight", "mlp_q.out.bias"):
        P[k] = torch.zeros_like(P[k])
    got = O.forward(_cfg(cfg), P, batch, mf)
    assert torch.count_nonzero(got["policy_logits"]) == 0
    assert torch.count_nonzero(got["q_values"]) == 0


def test_oracle_batched_equals_per_position():
    """Reference test_model.py:34-54 at the oracle level."""
    cfg, P, batch, _, mf = golden_io.forward_case("cellnodes")
    d = golden_io.load("builder.npz")
    wanted = {0, 3, 12, 34, 60}
    graphs = []
    for i in range(int(d["n_cases"])):
        n_s = len(d[f"{i}.in.stone_qr"])
        if n_s in wanted:
            wanted.discard(n_s)
            graphs.append(golden_io.mb.build(d[f"{i}.in.stone_qr"], d[f"{i}.in.stone_owner"],
                                             int(d[f"{i}.in.mover"]), d[f"{i}.in.legal_qr"],
                                             int(d[f"{i}.in.moves_remaining"])))
    c = _cfg(cfg)
    full = O.forward(c, P, golden_io.mb.collate(graphs), mf)
    offset = 0
    for i, g in enumerate(graphs):
        one = O.forward(c, P, golden_io.mb.collate([g]), mf)
        n = g.n_legal
        for k in ("policy_logits", "q_values", "q_score"):
            torch.testing.assert_close(full[k][offset:offset + n], one[k], rtol=0, atol=1e-5)
        torch.testing.assert_close(full["value"][i:i + 1], one["value"], rtol=0, atol=1e-6)
        offset += n
    assert offset == full["policy_logits"].shape[0] == batch.n_cells


@pytest.mark.parametrize("name", golden_io.CONFIG1_CASES)
def test_oracle_config1_matches_reference(name):
    """Config 1 (the reference's default architecture: h=128, 4 blocks, 4
    heads of dim 32) on 16 positions of 10-40 stones, fp32, 1e-4 relative."""
    cfg, P, batch, want, mf = golden_io.config1_case(name)
    assert cfg["h"] == 128 and cfg["blocks"] == 4 and cfg["heads"] == 4 and batch.n_pos == 16
    got = O.forward(_cfg(cfg), P, batch, mf)
    for k in ("policy_logits", "critic_logits", "q_score", "q_values", "value", "value_logits", "trunk_g"):
        scale = want[k].abs().max().clamp(min=1e-6)
        err = (got[k] - want[k]).abs().max()
        assert err <= 1e-4 * scale, f"{name}:{k} max err {err:.3e} vs scale {scale:.3e}"
