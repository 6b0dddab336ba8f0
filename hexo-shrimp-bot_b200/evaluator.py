"""The KLENT self-play evaluator closure (reference klent/train.py:100-120).

``network_evaluate(model, cfg)`` returns ``evaluate(batch)`` producing flat
CPU fp32 ``(policy_logits, q_score, q_values)`` in engine legal order, cut by
``batch.legal_offsets`` — the same contract the reference's collector, search
and Rust bridge consume. ``cfg`` needs ``device``, ``autocast`` and
``mass_floor`` attributes (the reference ``KlentConfig`` has them).

B200 specifics: only the batch fields the configured model reads cross PCIe;
copies are issued from pinned memory on the current stream; one lock
serialises device use like the reference's ``_gpu_lock``.
"""

from __future__ import annotations

import threading
from dataclasses import dataclass

import torch

from . import ops
from ._lib import check_device_error
from .builder import Batch
from .config import MantisConfig

_gpu_lock = threading.Lock()

_ALWAYS = (
    "stone_own", "window_feat", "moves_idx", "inc_stone", "inc_window", "inc_class", "attn_valid",
    "window_slot", "value_valid", "legal_offsets", "cell_pos", "dec_cell", "dec_window", "dec_class",
    "act_class", "act_empty",
)


def needed_fields(cfg: MantisConfig) -> tuple[str, ...]:
    """Batch tensors the evaluator forward reads for ``cfg``."""
    f = list(_ALWAYS)
    if cfg.cell_nodes or cfg.cell_structure:
        f.append("cell_nearest")
    if cfg.cell_nodes:
        f += ["radius_src", "radius_dst", "radius_orbit", "radius_own", "radius_on_axis"]
    if cfg.cell_adjacency:
        f += ["adjacency_src", "adjacency_dst"]
    if not cfg.uses_cell_state:
        f += ["relay_cell_ptr", "relay_window", "relay_class", "relay_win_ptr", "relay_wcell", "relay_cls_ptr",
              "relay_ccell"]
    if cfg.action_tactical:
        f.append("act_tactical")
    return tuple(f)


def to_device(batch: Batch, device, fields) -> Batch:
    """Copy only ``fields`` (others become empty placeholders on the device)."""
    moved = {}
    for k, v in vars(batch).items():
        if isinstance(v, torch.Tensor):
            if k in fields:
                moved[k] = v.to(device, non_blocking=True)
            else:
                moved[k] = torch.empty((0,) + tuple(v.shape[1:]), dtype=v.dtype, device=device)
        else:
            moved[k] = v
    # cell_pos is long and needed; keep shapes consistent for size reads
    return Batch(**moved)


@dataclass
class EvaluatorConfig:
    device: str = "cuda"
    autocast: bool = True
    mass_floor: float = 0.2
    gemm: str = "cublas"


def network_evaluate(model, cfg):
    """The self-play evaluator: CPU fp32 (policy, q_score, q_values)."""
    dtype = torch.bfloat16 if getattr(cfg, "autocast", True) else torch.float32
    gemm = getattr(cfg, "gemm", "cublas")
    fields = needed_fields(model.cfg)
    device = torch.device(cfg.device)
    if device.type != "cuda":
        raise RuntimeError("the B200 evaluator runs on CUDA devices only")

    def evaluate(batch: Batch):
        with _gpu_lock, torch.no_grad():
            b = to_device(batch, device, fields)
            eng = model.engine(dtype, gemm=gemm)
            policy, critic = eng.evaluate(b)
            q_score, q_values = ops.compose(critic, b.legal_offsets, cfg.mass_floor)
            out = torch.cat([policy.float(), q_score, q_values]).to("cpu")
            check_device_error(device)
            n = policy.shape[0]
            return out[:n], out[n:2 * n], out[2 * n:]

    return evaluate
