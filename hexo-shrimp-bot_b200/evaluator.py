"""The KLENT self-play evaluator closure (reference klent/train.py:100-120).

``network_evaluate(model, cfg)`` returns ``evaluate(batch)`` producing flat
CPU fp32 ``(policy_logits, q_score, q_values)`` in engine legal order, cut by
``batch.legal_offsets`` — the same contract the reference's collector, search
and Rust bridge consume. ``cfg`` needs ``device``, ``autocast`` and
``mass_floor`` attributes (the reference ``KlentConfig`` has them).

``network_evaluate_multi(model, cfg, devices)`` is the same closure over
several GPUs of one process: each call is cut into contiguous slices of
positions balanced by cells + windows + radius edges, each slice is
evaluated on its own device (a weight replica each), and the host output is
assembled in position order; a device whose slice fails is dropped and the
slice re-run on another.

B200 specifics: only the batch fields the configured model reads cross PCIe;
copies are issued from pinned memory on the current stream; one lock per
device serialises its use like the reference's ``_gpu_lock``.
"""

from __future__ import annotations

import threading
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass

import numpy as np
import torch

from . import ops, sharding
from ._lib import check_device_error
from .builder import RELAY_FIELDS, Batch, relay_tables
from .encoder import INT64_FIELDS
from .vocab import GLOBAL_ROWS, TERN_DEC_CLASSES
from .config import MantisConfig

_locks: dict = {}
_locks_guard = threading.Lock()


def device_lock(device) -> threading.Lock:
    """The lock serialising evaluator calls on ``device`` (the reference's
    single ``_gpu_lock``, klent/train.py:85, one per device here so that
    different GPUs run concurrently)."""
    d = torch.device(device)
    if d.type == "cuda" and d.index is None:
        d = torch.device("cuda", torch.cuda.current_device())
    with _locks_guard:
        return _locks.setdefault(d, threading.Lock())

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


def _device_dtype(k: str, v: torch.Tensor) -> torch.dtype:
    """The batch contract's dtype of field ``k`` (int64 for an index field
    of a narrow batch, whose host copy is int32)."""
    return torch.int64 if (v.dtype == torch.int32 and k in INT64_FIELDS) else v.dtype


def _widened(k: str, t: torch.Tensor) -> torch.Tensor:
    """An index field copied from a narrow batch, widened on the device."""
    return t.long() if (t.dtype == torch.int32 and k in INT64_FIELDS) else t


def to_device(batch: Batch, device, fields) -> Batch:
    """Copy only ``fields`` (others become empty placeholders on the device);
    int32 index fields of a narrow batch are widened to int64 there."""
    moved = {}
    for k, v in vars(batch).items():
        if isinstance(v, torch.Tensor):
            if k in fields:
                moved[k] = _widened(k, v.to(device, non_blocking=True))
            else:
                moved[k] = torch.empty((0,) + tuple(v.shape[1:]), dtype=_device_dtype(k, v), device=device)
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
    "adjacency_src": ("adj", "cell"), "adjacency_dst": ("adj", "cell"), "adjacency_axis": ("adj", None),
}
# The relay's CSR views are derived from the decoder incidence of the run's
# own positions (builder.relay_tables) instead of being cut.
_DERIVED_FIELDS = frozenset(RELAY_FIELDS)


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
    keys = {"inc": ("inc_window", "window"), "radius": ("radius_dst", "cell"), "dec": ("dec_cell", "cell"),
            "adj": ("adjacency_dst", "cell")}
    for space, (key, by) in keys.items():
        if key in fields:
            off[space] = np.searchsorted(getattr(batch, key).numpy(), off[by])
    return off


def split_supported(fields) -> bool:
    return all(f in _SPLIT_FIELDS or f in _DERIVED_FIELDS for f in fields)


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
        if k not in fields or k in _DERIVED_FIELDS:
            moved[k] = torch.empty((0,) + tuple(v.shape[1:]), dtype=_device_dtype(k, v), device=device)
            continue
        rows, by = _SPLIT_FIELDS[k]
        if rows == "pos+1":
            a, z = p0, p1 + 1
        else:
            o = off[rows]
            a, z = int(o[p0]), int(o[p1])
        t = _widened(k, v[a:z].to(device, non_blocking=True, copy=True))
        if by is not None and base[by]:
            t.sub_(base[by])
        moved[k] = t
    if _DERIVED_FIELDS & set(fields):
        a, z = int(off["dec"][p0]), int(off["dec"][p1])
        n_win = int(off["window"][p1] - off["window"][p0])
        views = relay_tables(batch.dec_cell[a:z].numpy() - base["cell"], batch.dec_window[a:z].numpy() - base["window"],
                             batch.dec_class[a:z].numpy(), n_win, TERN_DEC_CLASSES)
        for k, t in zip(RELAY_FIELDS, views):
            moved[k] = t.to(device, non_blocking=True)
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


def range_points(p0: int, p1: int, part: int) -> list[int]:
    """``split_points`` for positions [p0, p1): one run when the range fits
    in ``part`` positions (or ``part`` is 0), else a short lead run and runs
    of ``part``."""
    n = p1 - p0
    if part <= 0 or n <= part:
        return [p0, p1]
    lead = max(1, min(part // 4, n // 8))
    cuts = [p0, p0 + lead]
    while cuts[-1] + part < p1:
        cuts.append(cuts[-1] + part)
    if cuts[-1] < p1:
        cuts.append(p1)
    return cuts


class _DeviceRunner:
    """Evaluates position ranges of host batches on one device: the runs'
    host-to-device copies on a side stream overlap the previous run's
    compute, and each run's outputs are copied out on it while the next run
    computes, into the caller's pinned host buffer."""

    def __init__(self, model, cfg, device):
        self.model = model
        self.device = torch.device(device)
        self.dtype = torch.bfloat16 if getattr(cfg, "autocast", True) else torch.float32
        self.gemm = getattr(cfg, "gemm", "tcgen05-ln")
        self.mass_floor = cfg.mass_floor
        self.fields = needed_fields(model.cfg)
        self.part = int(getattr(cfg, "part_positions", 448) or 0)
        # One copy stream for the runner's lifetime: the caching allocator
        # keeps per-stream pools, so a fresh stream per call would allocate
        # every run's device buffers anew.
        self._copy = None

    def run_range(self, batch: Batch, off, p0: int, p1: int, host_out: torch.Tensor, n: int, part=None) -> None:
        """Positions [p0, p1) of ``batch`` (``off``: its ``_offsets``) into
        ``host_out[j * n + c0 : j * n + c1]`` for j = policy, q_score,
        q_values, where [c0, c1) are the range's cells."""
        with device_lock(self.device), torch.no_grad(), torch.cuda.device(self.device):
            eng = self.model.engine(self.dtype, gemm=self.gemm)
            cuts = range_points(p0, p1, self.part if part is None else part)
            compute = torch.cuda.current_stream(self.device)
            if self._copy is None:
                self._copy = torch.cuda.Stream(self.device)
            copy = self._copy

            def issue(k):
                copy.wait_stream(compute)  # buffers the allocator hands out may still be read by compute
                with torch.cuda.stream(copy):
                    b = part_to_device(batch, self.fields, off, cuts[k], cuts[k + 1], self.device)
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
                q_score, q_values = ops.compose(critic, b.legal_offsets, self.mass_floor)
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
            check_device_error(self.device)


def network_evaluate(model, cfg):
    """The self-play evaluator: CPU fp32 (policy, q_score, q_values)."""
    dtype = torch.bfloat16 if getattr(cfg, "autocast", True) else torch.float32
    gemm = getattr(cfg, "gemm", "tcgen05-ln")
    fields = needed_fields(model.cfg)
    device = torch.device(cfg.device)
    if device.type != "cuda":
        raise RuntimeError("the B200 evaluator runs on CUDA devices only")

    runner = _DeviceRunner(model, cfg, device)
    pipelined = runner.part > 0 and split_supported(fields)

    def evaluate(batch: Batch):
        if pipelined and batch.n_pos > runner.part:
            off = _offsets(batch, fields)
            n = int(off["cell"][-1])
            host_out = torch.empty(3 * n, dtype=torch.float32, pin_memory=True)
            runner.run_range(batch, off, 0, batch.n_pos, host_out, n)
            return host_out[:n], host_out[n:2 * n], host_out[2 * n:]
        with device_lock(device), torch.no_grad():
            eng = model.engine(dtype, gemm=gemm)
            b = to_device(batch, device, fields)
            policy, critic = eng.evaluate(b)
            q_score, q_values = ops.compose(critic, b.legal_offsets, cfg.mass_floor)
            policy = policy.float()
            out = torch.cat([policy, q_score, q_values]).to("cpu")
            check_device_error(device)
            n = policy.shape[0]
            return out[:n], out[n:2 * n], out[2 * n:]

    return evaluate


def _replica(model, device):
    """``model`` itself on its own device, else a copy of its weights on
    ``device`` (loaded once, evaluation mode)."""
    dev = next(model.parameters()).device
    if dev == device:
        return model
    twin = type(model)(model.cfg)
    twin.load_state_dict(model.state_dict())
    return twin.to(device).eval()


class MultiDeviceEvaluator:
    """``network_evaluate`` over several GPUs (the reference's evaluator
    closure, klent/train.py:100-120, sharded by positions): see
    ``network_evaluate_multi``. ``lost`` holds the indices of devices
    dropped after a failure."""

    def __init__(self, model, cfg, devices):
        devs = [torch.device(d) for d in devices]
        if not devs or any(d.type != "cuda" for d in devs):
            raise RuntimeError("the multi-device evaluator needs one or more CUDA devices")
        devs = [torch.device("cuda", d.index if d.index is not None else torch.cuda.current_device()) for d in devs]
        self.fields = needed_fields(model.cfg)
        if not split_supported(self.fields):
            raise NotImplementedError(f"batches of this configuration cannot be cut by positions: "
                                      f"{sorted(set(self.fields) - set(_SPLIT_FIELDS) - _DERIVED_FIELDS)}")
        replicas = {}
        for d in devs:
            if d not in replicas:
                replicas[d] = _replica(model, d)
        self.devices = devs
        self.runners = [_DeviceRunner(replicas[d], cfg, d) for d in devs]
        self.lost: set[int] = set()
        self._pool = ThreadPoolExecutor(len(devs))

    def costs(self, batch: Batch, off) -> np.ndarray:
        """Per position: cells + windows + radius edges."""
        edges = np.diff(off["radius"]) if "radius" in off else None
        return sharding.position_costs(np.diff(off["cell"]), np.diff(off["window"]), edges)

    def __call__(self, batch: Batch):
        off = _offsets(batch, self.fields)
        n = int(off["cell"][-1])
        host_out = torch.empty(3 * n, dtype=torch.float32, pin_memory=True)
        live = len(self.runners) - len(self.lost)
        if live < 1:
            raise sharding.WorkerLost("every device of this evaluator has failed")
        cuts = sharding.balanced_cuts(self.costs(batch, off), live)

        def run(runner, p0, p1):
            runner.run_range(batch, off, p0, p1, host_out, n)

        sharding.run_slices(cuts, self.runners, run, self.lost, self._pool)
        return host_out[:n], host_out[n:2 * n], host_out[2 * n:]

    def close(self) -> None:
        self._pool.shutdown(wait=True)


def network_evaluate_multi(model, cfg, devices=None):
    """The self-play evaluator over ``devices`` (default: every visible GPU):
    CPU fp32 (policy, q_score, q_values) for the whole batch, in position
    order, as ``network_evaluate`` returns them. Each call cuts the batch
    into one contiguous slice per live device, balanced by cells + windows +
    radius edges per position; each device holds a weight replica and
    evaluates its slice (pipelined like ``network_evaluate`` when larger than
    ``cfg.part_positions``) into its rows of the shared host output. A slice
    whose device raises is re-run on a live device and the failed device is
    left out of later calls; when none is left the call raises
    ``sharding.WorkerLost``."""
    if devices is None:
        devices = [f"cuda:{i}" for i in range(torch.cuda.device_count())]
    return MultiDeviceEvaluator(model, cfg, devices)


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
        with device_lock(self._device), torch.no_grad():
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
