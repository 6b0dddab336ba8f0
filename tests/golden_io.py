"""Loaders for the committed golden fixtures (tests/golden/*.npz)."""

from __future__ import annotations

import importlib
import json
import sys
from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"
REPO = GOLDEN.parent.parent
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

mb = importlib.import_module("hexo-shrimp-bot_b200")

_DT = {"torch.int64": torch.int64, "torch.int32": torch.int32, "torch.bool": torch.bool,
       "torch.float32": torch.float32}


def load(name: str):
    return np.load(GOLDEN / name, allow_pickle=False)


def batch_from(d, prefix: str = "batch."):
    fields = {}
    for k in d.files:
        if not k.startswith(prefix) or k.endswith("__dtype"):
            continue
        name = k[len(prefix):]
        a = d[k]
        dt = prefix + name + "__dtype"
        if dt in d.files:
            fields[name] = torch.from_numpy(np.ascontiguousarray(a)).to(_DT[str(d[dt])])
        else:
            fields[name] = int(a)
    return mb.Batch(**fields)


def forward_case(name: str):
    d = load(f"forward_{name}.npz")
    cfg = json.loads(str(d["config"]))
    params = {k[len("param."):]: torch.from_numpy(d[k].astype(np.float32) if d[k].dtype == np.float16 else d[k])
              for k in d.files if k.startswith("param.")}
    outs = {k[len("out."):]: torch.from_numpy(d[k]) for k in d.files if k.startswith("out.")}
    return cfg, params, batch_from(d), outs, float(d["mass_floor"])


FORWARD_CASES = ["default", "latents", "cellnodes", "full", "uncovered"]


# ------------------------------------------------------------ config 1
# The config-1 fixtures (forward_config1_<name>.npz) hold no weights: both the
# reference's module and this repository's draw them from the same seed (same
# construction order), then every parameter except the LayerNorm affines is
# redrawn as N(0, 0.02) from a seeded generator. The fixture's per-tensor
# checksums guard the regeneration.
CONFIG1_CASES = ["relay", "prod"]
CONFIG1_SEED = {"relay": 301, "prod": 302}
CONFIG1_POSITIONS_SEED = 17
CONFIG1_KNOBS = {"relay": {}, "prod": {"cell_latents": True, "cell_nodes": True}}


def config1_reinit(model: torch.nn.Module, seed: int) -> None:
    """Redraw every weight N(0, 0.02) (LayerNorm weight / bias keep 1 / 0),
    the zero-initialised decoder outputs and class biases included, so every
    path of the forward carries signal at the north_star weight scale."""
    gen = torch.Generator().manual_seed(seed + 1)
    norms = {name for name, m in model.named_modules() if isinstance(m, torch.nn.LayerNorm)}
    with torch.no_grad():
        for name, p in model.named_parameters():
            owner = name.rsplit(".", 1)[0] if "." in name else ""
            if owner in norms:
                continue
            p.copy_(torch.randn(p.shape, generator=gen) * 0.02)


def config1_model(name: str):
    """This repository's module with the config-1 weights (CPU, eval)."""
    torch.manual_seed(CONFIG1_SEED[name])
    net = mb.MantisNet(mb.MantisConfig(**CONFIG1_KNOBS[name])).eval()
    config1_reinit(net, CONFIG1_SEED[name])
    return net


def param_checksum(t: torch.Tensor) -> list:
    t = t.detach().double().reshape(-1)
    return [float(t.sum()), float(t.abs().sum()), float((t * torch.arange(t.numel(), dtype=torch.float64)).sum())]


def config1_case(name: str):
    """(cfg dict, params, batch, reference outputs, mass_floor); the params
    are regenerated and checked against the fixture's checksums."""
    d = load(f"forward_config1_{name}.npz")
    cfg = json.loads(str(d["config"]))
    net = config1_model(name)
    params = {k: v.detach().clone() for k, v in net.state_dict().items()}
    for k, v in params.items():
        want = d["checksum." + k]
        got = np.array(param_checksum(v))
        if not np.allclose(got, want, rtol=1e-9, atol=1e-9):
            raise AssertionError(f"regenerated config-1 weight {k} differs from the fixture's")
    outs = {k[len("out."):]: torch.from_numpy(d[k]) for k in d.files if k.startswith("out.")}
    return cfg, params, batch_from(d), outs, float(d["mass_floor"])
