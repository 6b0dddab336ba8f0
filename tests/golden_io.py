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
