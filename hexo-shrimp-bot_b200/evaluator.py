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

import numpy as np
import torch

from . import ops
from ._lib import check_device_error
from .builder import Batch
from .vocab import GLOBAL_ROWS
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


# ------------------------------------------------------------ sub-batches
# Positions are independent, so a batch can be evaluated as consecutive runs
# of positions, each a self-contained batch whose index fields are rebased to
# its own first stone, window, cell and position. Every per-position block of
# the collated arrays is contiguous and in position order (the builder
# concatenates positions; edge arrays are sorted by their destination), so a
# run is a set of host slices, found by binary search, plus four bases.
#
# field: (row space, value space) -- the row space names the offsets that cut
# the field; the value space, the base its values are rebased by (None: none).
_SPLIT_FIELDS = {
    "stone_own": ("stone", None), "window_feat": ("window", None), "moves_idx": ("pos", None),
    "inc_stone": ("inc", "stone"), "inc_window": ("inc", "window"), "inc_class": ("inc", None),
    "attn_valid": ("pos", None), "window_slot": ("window", "slot"), "value_valid": ("pos", None),
    "legal_offsets": ("pos+1", "cell"), "cell_pos": ("cell", "pos"), "cell_nearest": ("cell", None),
    "radius_src": ("radius", "stone"), "radius_dst": ("radius", "cell"), "radius_orbit": ("radius", None),
    "radius_own": ("radius", None), "radius_on_axis": ("radius", None),
    "dec_cell": ("dec", "cell"), "dec_window": ("dec", "window"), "dec_class": ("dec", None),
    "act_class": ("dec", None), "act_empty": ("cell", None), "act_tactical": ("cell", None),
}


def split_points(batch: Batch, part: int) -> list[int]:
    """Position boundaries of the runs: a short lead run (a quarter of
    ``part``, at most an eighth of the batch), whose copy is the only one
    not hidden behind compute, then runs of ``part`` positions."""
    p = batch.n_pos
    lead = max(1, min(part // 4, p // 8))
    cuts = [0, lead]
    while cuts[-1] + part < p:
        cuts.append(cuts[-1] + part)
    if cuts[-1] < p:
        cuts.append(p)
    return cuts


def _offsets(batch: Batch, fields) -> dict[str, np.ndarray]:
    """Per-position start offsets (length n_pos + 1) of every row space."""
    p = batch.n_pos
    stones = batch.attn_valid.sum(1).numpy() - GLOBAL_ROWS
    off = {"pos": np.arange(p + 1), "stone": np.concatenate([[0], np.cumsum(stones)])}
    off["window"] = np.searchsorted(batch.window_slot.numpy(), np.arange(p + 1) * batch.max_w)
    off["cell"] = batch.legal_offsets.numpy()
    keys = {"inc": ("inc_window", "window"), "radius": ("radius_dst", "cell"), "dec": ("dec_cell", "cell")}
    for space, (key, by) in keys.items():
        if key in fields:
            off[space] = np.searchsorted(getattr(batch, key).numpy(), off[by])
    return off


def split_supported(fields) -> bool:
    return all(f in _SPLIT_FIELDS for f in fields)


def part_to_device(batch: Batch, fields, off, p0: int, p1: int, device) -> Batch:
    """Copy positions [p0, p1) of ``batch`` to ``device`` as a batch of their
    own (host slices copied on the current stream, indices rebased there)."""
    base = {"stone": int(off["stone"][p0]), "window": int(off["window"][p0]), "cell": int(off["cell"][p0]),
            "pos": p0, "slot": p0 * batch.max_w}
    moved = {}
    for k, v in vars(batch).items():
        if not isinstance(v, torch.Tensor):
            moved[k] = v
            continue
        if k not in fields:
            moved[k] = torch.empty((0,) + tuple(v.shape[1:]), dtype=v.dtype, device=device)
            continue
        rows, by = _SPLIT_FIELDS[k]
        if rows == "pos+1":
            a, z = p0, p1 + 1
        else:
            o = off[rows]
            a, z = int(o[p0]), int(o[p1])
        t = v[a:z].to(device, non_blocking=True, copy=True)
        if by is not None and base[by]:
            t.sub_(base[by])
        moved[k] = t
    moved["n_pos"] = p1 - p0
    moved["n_cells"] = int(off["cell"][p1] - off["cell"][p0])
    return Batch(**moved)


@dataclass
class EvaluatorConfig:
    device: str = "cuda"
    autocast: bool = True
    mass_floor: float = 0.2
    gemm: str = "tcgen05-ln"
    # Batches of more than part_positions positions are evaluated as a short
    # lead run, then runs of part_positions positions, whose host-to-device copies overlap
    # the previous run's compute; 0 turns this off. 448 measured best for
    # 512-position calls (a 64-position lead run, then one run of 448).
    part_positions: int = 448


def network_evaluate(model, cfg):
    """The self-play evaluator: CPU fp32 (policy, q_score, q_values)."""
    dtype = torch.bfloat16 if getattr(cfg, "autocast", True) else torch.float32
    gemm = getattr(cfg, "gemm", "tcgen05-ln")
    fields = needed_fields(model.cfg)
    device = torch.device(cfg.device)
    if device.type != "cuda":
        raise RuntimeError("the B200 evaluator runs on CUDA devices only")

    part = int(getattr(cfg, "part_positions", 448) or 0)
    pipelined = part > 0 and split_supported(fields)
    # One copy stream for the closure's lifetime: the caching allocator keeps
    # per-stream pools, so a fresh stream per call would allocate every run's
    # device buffers anew.
    streams = {}

    def run_parts(batch: Batch, eng):
        """Copy run k + 1 in on a side stream while run k computes, and copy
        run k's outputs out on it while run k + 1 computes, into one pinned
        host buffer (the caching host allocator recycles it between calls)."""
        cuts = split_points(batch, part)
        off = _offsets(batch, fields)
        compute = torch.cuda.current_stream(device)
        copy = streams.get("copy")
        if copy is None:
            copy = streams["copy"] = torch.cuda.Stream(device)
        n = int(off["cell"][-1])
        host_out = torch.empty(3 * n, dtype=torch.float32, pin_memory=True)

        def issue(k):
            copy.wait_stream(compute)  # buffers the allocator hands out may still be read by compute
            with torch.cuda.stream(copy):
                b = part_to_device(batch, fields, off, cuts[k], cuts[k + 1], device)
                done = torch.cuda.Event()
                done.record(copy)
            return b, done

        nxt = issue(0)
        for k in range(len(cuts) - 1):
            b, done = nxt
            compute.wait_event(done)
            for t in vars(b).values():
                if isinstance(t, torch.Tensor):
                    t.record_stream(compute)
            if k + 2 < len(cuts):
                nxt = issue(k + 1)
            policy, critic = eng.evaluate(b)
            q_score, q_values = ops.compose(critic, b.legal_offsets, cfg.mass_floor)
            res = (policy.float(), q_score, q_values)
            ready = torch.cuda.Event()
            ready.record(compute)
            copy.wait_event(ready)
            c0, c1 = int(off["cell"][cuts[k]]), int(off["cell"][cuts[k + 1]])
            with torch.cuda.stream(copy):
                for j, t in enumerate(res):
                    t.record_stream(copy)
                    host_out[j * n + c0:j * n + c1].copy_(t, non_blocking=True)
        copy.synchronize()
        return host_out[:n], host_out[n:2 * n], host_out[2 * n:]

    def evaluate(batch: Batch):
        with _gpu_lock, torch.no_grad():
            eng = model.engine(dtype, gemm=gemm)
            if pipelined and batch.n_pos > part:
                out = run_parts(batch, eng)
                check_device_error(device)
                return out
            b = to_device(batch, device, fields)
            policy, critic = eng.evaluate(b)
            q_score, q_values = ops.compose(critic, b.legal_offsets, cfg.mass_floor)
            policy = policy.float()
            out = torch.cat([policy, q_score, q_values]).to("cpu")
            check_device_error(device)
            n = policy.shape[0]
            return out[:n], out[n:2 * n], out[2 * n:]

    return evaluate


class _LeafEvaluator:
    """``network_evaluate``'s closure plus ``leaves(batch, tau, lam)``: per
    position the rank of the KLENT-improved policy's largest entry and the
    improved value (klent/search.py:231-253's per-leaf step), computed on the
    device so that two numbers per position cross back instead of three
    floats per legal cell."""

    def __init__(self, model, cfg):
        self._full = network_evaluate(model, cfg)
        self._model, self._cfg = model, cfg
        self._dtype = torch.bfloat16 if getattr(cfg, "autocast", True) else torch.float32
        self._gemm = getattr(cfg, "gemm", "tcgen05-ln")
        self._fields = needed_fields(model.cfg)
        self._device = torch.device(cfg.device)

    def __call__(self, batch: Batch):
        return self._full(batch)

    def leaves(self, batch: Batch, tau: float, lam: float):
        with _gpu_lock, torch.no_grad():
            eng = self._model.engine(self._dtype, gemm=self._gemm)
            b = to_device(batch, self._device, self._fields)
            policy, critic = eng.evaluate(b)
            q_score, q_values = ops.compose(critic, b.legal_offsets, self._cfg.mass_floor)
            imp = ops.improved_policy(policy.float(), q_score, q_values, b.legal_offsets, tau, lam)
            ranks = ops.segment_argmax(imp.probs, b.legal_offsets)
            ranks, values = ranks.cpu(), imp.v_hat.cpu()
            check_device_error(self._device)
        return ranks, values


def network_leaf_evaluate(model, cfg):
    """The evaluator closure with the device-side leaf step the Gumbel search
    (search.gumbel_choose) uses for its leaf waves."""
    if torch.device(cfg.device).type != "cuda":
        raise RuntimeError("the B200 evaluator runs on CUDA devices only")
    return _LeafEvaluator(model, cfg)
