"""Generate the golden fixtures from the reference implementation itself.

Run in a container where the reference checkout is available (it is NOT on the
GPU box; the committed ``.npz`` files travel instead):

    python tests/golden/make_golden.py --reference <path to python/mantisnet>

(or set MANTISNET_REFERENCE to that path).

The reference's PyO3 extension ``hexo_py`` needs cargo to build; the only
module-level use is the ``MODEL_REPR_VERSION`` constant (builder.py:26), so a
stub module carrying that constant is installed before importing. Positions
come from this repository's seeded engine restatement (the reference's own
fixtures replay positions through the Rust engine); the reference builder then
builds them, and the reference eager-CPU fp32 forward produces the outputs.

Fixtures written next to this script:

- ``builder.npz``: per-position builder inputs and every PositionGraph field,
  plus the collated Batch of all of them.
- ``forward_<name>.npz``: a model config, its state_dict (seeded; zero-init
  parameters perturbed so every path carries signal), a collated batch, the
  reference outputs of ``MantisNet.forward`` and ``trunk``.
- ``ops.npz``: op-level reference outputs on seeded random inputs.
- ``forward_config1_<relay|prod>.npz``: the config-1 architecture (the
  reference's default ``MantisConfig()``: h=128, 4 blocks, 4 heads of dim 32,
  F=2) on 16 positions of 10-40 stones, relay (default knobs) and production
  knobs (cell_latents + cell_nodes). Weights are seeded N(0, 0.02) everywhere
  (``golden_io.config1_params``), so the fixture stores the seed and one
  checksum per tensor instead of the 4.5-5.2 M parameters; the generator
  checks that the reference's own module, given the same seed, holds exactly
  the weights this repository's module regenerates.
"""

from __future__ import annotations

import argparse
import dataclasses
import importlib
import json
import os
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent

PLIES = [0, 1, 2, 3, 5, 9, 12, 21, 34, 60]  # the reference's fixture depths
EXTRA = [(45, 1234), (150, 99)]

MODELS = {
    "default": dict(),
    "latents": dict(cell_latents=True),
    "cellnodes": dict(cell_latents=True, cell_nodes=True),
    "full": dict(cell_latents=True, cell_nodes=True, cell_adjacency=True,
                 cell_structure=True, action_tactical=True),
    "uncovered": dict(cell_latents=True, cell_nodes=True, cell_node_scope="uncovered"),
}
SMALL = dict(h=32, blocks=2, heads=2, ffn_factor=2, value_queries=2, value_bins=5,
             policy_hidden=24, value_hidden=16)
FORWARD_PLIES = [0, 3, 12, 34, 60]


def _import_reference(path: str):
    stub = types.ModuleType("hexo_py")
    stub.MODEL_REPR_VERSION = 9
    sys.modules["hexo_py"] = stub
    sys.path.insert(0, path)
    return importlib.import_module("mantisnet")


def _engine():
    sys.path.insert(0, str(REPO))
    return importlib.import_module("hexo-shrimp-bot_b200.engine")


def _pack_int(a: np.ndarray) -> np.ndarray:
    a = np.asarray(a)
    if a.dtype == np.int64 and a.size and a.min() >= -32768 and a.max() < 32768:
        return a.astype(np.int16)
    if a.dtype == np.int64:
        return a.astype(np.int32)
    return a


def _batch_arrays(batch, prefix: str) -> dict:
    out = {}
    for k, v in vars(batch).items():
        if isinstance(v, torch.Tensor):
            a = v.numpy()
            out[prefix + k] = _pack_int(a) if a.dtype == np.int64 else a
            out[prefix + k + "__dtype"] = np.array(str(v.dtype))
        else:
            out[prefix + k] = np.array(v)
    return out


def make_builder(mn, eng):
    specs = [eng.random_game(p, seed=7)[0] for p in PLIES] + [eng.random_game(p, seed=s)[0] for p, s in EXTRA]
    arrays = {"n_cases": np.array(len(specs))}
    graphs = []
    for i, sp in enumerate(specs):
        arrays[f"{i}.in.stone_qr"] = sp.stone_qr
        arrays[f"{i}.in.stone_owner"] = sp.stone_owner
        arrays[f"{i}.in.mover"] = np.array(sp.mover)
        arrays[f"{i}.in.legal_qr"] = sp.legal_qr
        arrays[f"{i}.in.moves_remaining"] = np.array(sp.moves_remaining)
        g = mn.builder.build(sp.stone_qr, sp.stone_owner, sp.mover, sp.legal_qr, sp.moves_remaining)
        graphs.append(g)
        for f in dataclasses.fields(g):
            v = getattr(g, f.name)
            arrays[f"{i}.out.{f.name}"] = v
    arrays.update(_batch_arrays(mn.builder.collate(graphs[:-1]), "batch."))
    np.savez_compressed(HERE / "builder.npz", **arrays)
    return specs


def _perturb(model: torch.nn.Module, seed: int) -> None:
    gen = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if torch.count_nonzero(p) == 0:
                p.copy_(torch.randn(p.shape, generator=gen) * 0.3)
        for head in (model.mlp_p, model.mlp_q):
            head.out.weight.copy_(torch.randn(head.out.weight.shape, generator=gen) * 0.5)
            head.out.bias.copy_(torch.randn(head.out.bias.shape, generator=gen) * 0.5)
        # Round every weight to an fp16-representable value before the
        # reference runs, so the fixture stores it losslessly at half size.
        for p in model.parameters():
            p.copy_(p.half().float())


def make_forward(mn, specs, name: str, knobs: dict, seed: int):
    cfg = mn.MantisConfig(**SMALL, **knobs)
    torch.manual_seed(seed)
    model = mn.MantisNet(cfg).eval()
    _perturb(model, seed + 1)
    by_ply = {len(s.stone_qr): s for s in specs}
    graphs = [mn.builder.build(s.stone_qr, s.stone_owner, s.mover, s.legal_qr, s.moves_remaining)
              for s in (by_ply[p] for p in FORWARD_PLIES)]
    batch = mn.builder.collate(graphs)
    with torch.no_grad():
        out = model(batch, 0.2)
        w, g, cells = model.trunk(batch)
        policy, critic = model.cell_head_logits(w, g, cells, batch)
    arrays = {"config": np.array(json.dumps(dataclasses.asdict(cfg))), "mass_floor": np.array(0.2)}
    for k, v in model.state_dict().items():
        arrays["param." + k] = v.half().numpy() if v.is_floating_point() else v.numpy()
    arrays.update(_batch_arrays(batch, "batch."))
    for k, v in vars(out).items():
        arrays["out." + k] = v.numpy()
    arrays["out.critic_logits"] = critic.numpy()
    arrays["out.trunk_g"] = g.numpy()
    np.savez_compressed(HERE / f"forward_{name}.npz", **arrays)


def make_ops(mn):
    att = importlib.import_module("mantisnet.attention")
    cl = importlib.import_module("mantisnet.cell_latents")
    wl = importlib.import_module("mantisnet.window_latents")
    re_ = importlib.import_module("mantisnet.row_encoder")
    gen = torch.Generator().manual_seed(5)
    a = {}
    # stone attention: ragged prefixes, a position with only its latents live
    q, k, v = (torch.randn(3, 2, 37, 16, generator=gen) for _ in range(3))
    seq = torch.tensor([37, 9, 4], dtype=torch.int32)
    a.update({"att.q": q, "att.k": k, "att.v": v, "att.seq_lens": seq,
              "att.out": att._attention_reference(q, k, v, seq)})
    # typed segment attention with an empty run (query 2) and class value rows
    nq, ns, heads, hd, ncls = 5, 7, 2, 8, 11
    qq, kk, vv = torch.randn(nq, heads, hd, generator=gen), torch.randn(ns, heads, hd, generator=gen), \
        torch.randn(ns, heads, hd, generator=gen)
    bias = torch.randn(heads, ncls, generator=gen)
    vcls = torch.randn(ncls, heads * hd, generator=gen)
    qid = torch.tensor([0, 0, 0, 1, 3, 3, 3, 3, 4])
    src = torch.tensor([1, 4, 6, 0, 2, 3, 5, 6, 1])
    cls = torch.tensor([3, 0, 10, 7, 7, 2, 1, 9, 4])
    o, m, l = cl._reference_forward(qq, kk, vv, bias, vcls, src, cls, qid)
    o2, _, _ = cl._reference_forward(qq, kk, vv, bias, None, src, cls, qid)
    a.update({"seg.q": qq, "seg.k": kk, "seg.v": vv, "seg.bias": bias, "seg.vcls": vcls, "seg.qid": qid,
              "seg.src": src, "seg.cls": cls, "seg.out": o, "seg.out_plain": o2})
    # window-latent read / broadcast with an empty position (index 1)
    pos = torch.tensor([0, 0, 0, 2, 2, 3, 3, 3, 3])
    rq = torch.randn(4, 4, heads, hd, generator=gen)
    rk, rv = torch.randn(9, heads, hd, generator=gen), torch.randn(9, heads, hd, generator=gen)
    offsets, order = wl.window_latent_layout(pos, 4)
    ro, _, _ = wl._reference_read_forward(rq, rk, rv, offsets, order)
    bq = torch.randn(9, heads, hd, generator=gen)
    bk, bv = torch.randn(4, 4, heads, hd, generator=gen), torch.randn(4, 4, heads, hd, generator=gen)
    bo, _, _ = wl._reference_broadcast_forward(bq, bk, bv, pos)
    a.update({"win.pos": pos, "win.rq": rq, "win.rk": rk, "win.rv": rv, "win.read": ro,
              "win.bq": bq, "win.bk": bk, "win.bv": bv, "win.bcast": bo})
    # action-row encoder
    pre = torch.randn(6, 16, generator=gen)
    table = torch.randn(9, 16, generator=gen)
    ew = torch.tensor([0, 3, 5, 1, 1, 2, 4])
    ec = torch.tensor([8, 0, 2, 2, 7, 1, 3])
    ecell = torch.tensor([0, 0, 0, 2, 2, 3, 3])
    a.update({"row.pre": pre, "row.table": table, "row.win": ew, "row.cls": ec, "row.cell": ecell,
              "row.out": re_._encode_reference(pre, table, ew, ec, ecell, 5)})
    np.savez_compressed(HERE / "ops.npz", **{k: x.numpy() for k, x in a.items()})


CONFIG1 = {"relay": dict(), "prod": dict(cell_latents=True, cell_nodes=True)}


def make_config1(mn, eng, name: str, knobs: dict):
    """Config 1: the reference's default architecture, 16 positions of 10-40
    stones from seeded random legal play, std-0.02 weights, fp32 eager CPU."""
    sys.path.insert(0, str(REPO / "tests"))
    gio = importlib.import_module("golden_io")
    seed = gio.CONFIG1_SEED[name]
    cfg = mn.MantisConfig(**knobs)
    ours = gio.config1_model(name)  # this repository's module, same seed
    torch.manual_seed(seed)
    model = mn.MantisNet(cfg).eval()
    gio.config1_reinit(model, seed)
    want = ours.state_dict()
    got = model.state_dict()
    assert list(want) == list(got), "parameter names / order differ from the reference"
    for k in want:
        assert torch.equal(want[k], got[k]), f"seeded weights differ from the reference at {k}"
    specs = eng.random_positions(16, 10, 40, seed=gio.CONFIG1_POSITIONS_SEED)
    graphs = [mn.builder.build(s.stone_qr, s.stone_owner, s.mover, s.legal_qr, s.moves_remaining) for s in specs]
    batch = mn.builder.collate(graphs)
    with torch.no_grad():
        out = model(batch, 0.2)
        w, g, cells = model.trunk(batch)
        policy, critic = model.cell_head_logits(w, g, cells, batch)
    arrays = {"config": np.array(json.dumps(dataclasses.asdict(cfg))), "mass_floor": np.array(0.2),
              "seed": np.array(seed)}
    for k, v in got.items():
        arrays["checksum." + k] = np.array(gio.param_checksum(v))
    arrays.update(_batch_arrays(batch, "batch."))
    for k, v in vars(out).items():
        arrays["out." + k] = v.numpy()
    arrays["out.critic_logits"] = critic.numpy()
    arrays["out.trunk_g"] = g.numpy()
    np.savez_compressed(HERE / f"forward_config1_{name}.npz", **arrays)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("MANTISNET_REFERENCE"),
                    help="path to the reference's python/mantisnet directory")
    ap.add_argument("--only", choices=["all", "config1"], default="all")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference <path to python/mantisnet> or set MANTISNET_REFERENCE")
    torch.set_num_threads(max(1, torch.get_num_threads()))
    mn = _import_reference(args.reference)
    importlib.import_module("mantisnet.builder")
    eng = _engine()
    if args.only == "all":
        specs = make_builder(mn, eng)
        for i, (name, knobs) in enumerate(MODELS.items()):
            make_forward(mn, specs, name, knobs, seed=100 + i)
            print("forward", name, "done", flush=True)
        make_ops(mn)
    for name, knobs in CONFIG1.items():
        make_config1(mn, eng, name, knobs)
        print("config1", name, "done", flush=True)
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    main()
