"""B200-native MantisNet evaluator (sm_100a CUDA behind a C-ABI library).

Public surface mirrors the reference package ``mantisnet``: ``MantisConfig``,
``MantisNet``, ``Batch``, ``build``/``collate``/``batch_from_arrays`` and the
KLENT evaluator closure ``network_evaluate``. The package directory name has
hyphens, so import it with ``importlib.import_module("hexo-shrimp-bot_b200")``.
"""

from __future__ import annotations

from .builder import Batch, PositionGraph, batch_from_arrays, build, collate, from_spec, relay_tables
from .config import MantisConfig

__all__ = [
    "Batch", "PositionGraph", "batch_from_arrays", "build", "collate", "from_spec", "relay_tables",
    "MantisConfig",
]


_SUBMODULES = ("_lib", "ops", "model", "evaluator", "vocab", "engine", "builder", "encoder", "config", "build", "sharding",
               "hexgraph", "search", "torch_ops")


def __getattr__(name):
    # The model and evaluator import torch CUDA bindings and the native
    # library lazily, so host-only users (builders, tests) need neither.
    if name in _SUBMODULES:
        import importlib

        return importlib.import_module(f".{name}", __name__)
    if name in ("MantisNet", "ModelOutput", "compose_q", "compose_acting_q", "return_mass", "Engine"):
        from . import model

        return getattr(model, name)
    if name in ("network_evaluate", "network_leaf_evaluate", "Evaluator"):
        from . import evaluator

        return getattr(evaluator, name)
    raise AttributeError(name)
