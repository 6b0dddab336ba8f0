#!/usr/bin/env python
"""Benchmark: MantisNet evaluator positions/s (bf16, B=4096 per GPU) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (the metric's own configuration; it fits one
GPU in chunks): per GPU, B=4096 late-game positions of 150-300 stones from
seeded uniform-random legal play, evaluated by the config-4 architecture
(h=256, 8 blocks, 8 heads, F=4, cell_latents + cell_nodes, the production
knobs) with random weights (std 0.02), bf16. A step is one pass of the
evaluator forward over the 4096 positions, processed as chunks of ``--chunk``
positions (the reference's cell-budget chunking). Positions are independent:
N GPUs evaluate N x 4096 positions with no collective (weak scaling); the
only cross-rank traffic is the timing barrier and the max-over-ranks reduce.

Printed JSON line keys follow the driver contract; ``value`` is device-resident
throughput (inputs already in HBM), ``e2e`` the same metric through the
reference-facing evaluator call (host batch, H2D + D2H inside the timed
region), ``roofline`` the dominant native kernel, ``cpu_baseline`` the CPU
oracle port of the reference forward on a bounded sample, ``encoder`` the
host rate of the native batch encoder that builds the inputs.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

ARCH = dict(h=256, blocks=8, heads=8, ffn_factor=4, cell_latents=True, cell_nodes=True)
METRIC = "positions/sec evaluated (bf16, B=4096) at 1/2/4/8 B200; p50 batch-64 latency"


def _pkg():
    import importlib

    return importlib.import_module("hexo-shrimp-bot_b200")


def make_specs(n, lo, hi, seed):
    return _pkg().engine.random_positions(n, lo, hi, seed=seed)


def batch_bytes(batch, fields):
    import torch

    return sum(getattr(batch, f).numel() * getattr(batch, f).element_size() for f in fields
               if isinstance(getattr(batch, f), torch.Tensor))


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]
        return False

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in getattr(self, "lines", []):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def peaks():
    try:
        return json.loads((REPO / "MEASURED_PEAKS.json").read_text()), "measured"
    except (OSError, ValueError):
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


# --------------------------------------------------------------- CPU side

def cpu_forward_rate(specs, sample, threads):
    """The CPU oracle (restatement of the reference's eager fp32 forward) on
    ``sample`` positions: positions/s with ``threads`` torch threads."""
    import torch

    from oracle import forward as O

    mb = _pkg()
    torch.set_num_threads(threads)
    cfg = mb.MantisConfig(**ARCH)
    torch.manual_seed(0)
    net = mb.MantisNet(cfg)
    params = {k: v.detach().clone() for k, v in net.state_dict().items()}
    c = O.Cfg(**{k: v for k, v in cfg.to_dict().items() if k != "dropout"})
    batch = mb.collate([mb.from_spec(s) for s in specs[:sample]])
    O.forward(c, params, mb.collate([mb.from_spec(specs[0])]), 0.2, value=False)  # warm
    t0 = time.perf_counter()
    O.forward(c, params, batch, 0.2, value=False)
    dt = time.perf_counter() - t0
    return sample / dt, dt


def _reference_pkg():
    """The loader of the reference installed in baseline/_ref, or None."""
    sys.path.insert(0, str(Path(__file__).resolve().parent / "tests"))
    try:
        import reference_pkg
    except ImportError:
        return None
    return reference_pkg if reference_pkg.available() else None


def reference_cpu_rate(specs, sample, threads):
    """The reference's own KLENT evaluator (klent/train.py:100-120, eager,
    fp32, stock KlentConfig otherwise) on the host cores, on ``sample``
    positions: positions/s. None when the reference is not installed in
    baseline/_ref."""
    reference_pkg = _reference_pkg()
    if reference_pkg is None:
        return None
    import importlib
    import torch

    mn = reference_pkg.load()
    train = importlib.import_module("mantisnet.klent.train")
    mb = _pkg()
    torch.set_num_threads(threads)
    torch.manual_seed(0)
    net = mn.MantisNet(mn.MantisConfig(**ARCH)).eval()
    ev = train.network_evaluate(net, train.KlentConfig(device="cpu", autocast=False, mass_floor=0.2))
    batch = mn.builder.Batch(**vars(mb.collate([mb.from_spec(s) for s in specs[:sample]])))
    t0 = time.perf_counter()
    ev(batch)
    return sample / (time.perf_counter() - t0)


def run_reference(args, rank):
    """The reference arm, on rank 0 only: the reference's own eager CPU
    evaluator from baseline/_ref on the host cores (the reference is Python;
    its CPU path is eager torch), else the CPU restatement of that path."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    sample = args.ref_sample
    specs = make_specs(max(sample, 1), args.lo, args.hi, seed=1234)
    own = _reference_pkg() is not None
    rates = []
    for i in range(args.warmup + args.steps):
        r = reference_cpu_rate(specs, sample, threads) if own else cpu_forward_rate(specs, sample, threads)[0]
        if i >= args.warmup:
            rates.append(r)
    v = statistics.median(rates)
    what = ("reference mantisnet network_evaluate, eager fp32 on CPU (baseline/_ref)" if own
            else "fp32 eager torch-CPU restatement of the reference forward (oracle port)")
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "positions/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * sample / v,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"{sample} late positions ({args.lo}-{args.hi} stones) per step, "
                               "config-4 architecture (h256/8 blocks/8 heads/F4, cell_latents+cell_nodes)",
                   "positions_per_step": sample},
        "cpu_baseline": {"value": v, "unit": "positions/s", "cores": threads, "kind": "reference" if own else "port",
                         "sample": f"{sample} positions per step, {what}"},
        "e2e": {"value": v, "unit": "positions/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------- GPU side

def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    mb = _pkg()
    ops = mb.ops
    lib = mb._lib
    lib.load()

    # Inputs: encoded on the host (the native encoder, all host threads)
    # straight into pinned host memory, ready for the host-to-device copy;
    # its rate on the distinct positions, in the narrow layout that the
    # end-to-end input uses, is reported (the second call: the first one also
    # sets up the vocabulary tables and the pinned blocks).
    n_chunks = math.ceil(args.positions / args.chunk)
    specs = make_specs(args.unique, args.lo, args.hi, seed=1000 + rank)
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    for _ in range(2):
        t0 = time.perf_counter()
        mb.encoder.encode(specs, pin_memory=True, narrow=True)
        enc_s = time.perf_counter() - t0
    encoder = {"value": len(specs) / enc_s, "unit": "positions/s", "threads": os.cpu_count() or 1,
               "sample": f"{len(specs)} distinct late positions ({args.lo}-{args.hi} stones), collated batch "
                         "in the narrow layout the end-to-end input uses (int32 index fields), written into "
                         "pinned host memory"}
    reps = math.ceil(args.chunk / len(specs))
    host = mb.encoder.encode((specs * reps)[: args.chunk])
    fields = mb.evaluator.needed_fields(mb.MantisConfig(**ARCH))
    # the end-to-end input: the encoder's narrow layout (int32 index fields,
    # widened on the device), in pinned memory
    host_pinned = mb.encoder.encode((specs * reps)[: args.chunk], narrow=True, pin_memory=True)

    if world > 1:
        dist.init_process_group("nccl", device_id=device, timeout=__import__("datetime").timedelta(seconds=600))

    cfg = mb.MantisConfig(**ARCH)
    torch.manual_seed(0)
    net = mb.MantisNet(cfg)
    with torch.no_grad():
        for head in (net.mlp_p, net.mlp_q):
            head.out.weight.normal_(std=0.02)
            head.out.bias.normal_(std=0.02)
    net = net.to(device).eval()
    eng = net.engine(torch.bfloat16, gemm=args.gemm)
    dev_batch = mb.evaluator.to_device(host, device, fields)
    torch.cuda.synchronize()

    def step_device():
        for _ in range(n_chunks):
            policy, critic = eng.evaluate(dev_batch)
            ops.compose(critic, dev_batch.legal_offsets, 0.2)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        return mb.sharding.max_over_ranks(x, device)

    for _ in range(args.warmup):
        step_device()
    barrier()
    calls0 = lib.call_count()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    eng.probe = {}
    with ClockSampler(local_rank) as clocks:
        torch.cuda.nvtx.range_push("timed")  # lets a profiler select the timed steps' launches
        start.record()
        for _ in range(args.steps):
            step_device()
        end.record()
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
    probe, eng.probe = eng.probe, None
    tables = eng.tables
    launches = (lib.call_count() - calls0) // max(args.steps, 1)
    ms = max_over_ranks(start.elapsed_time(end) / args.steps)
    positions_per_step = n_chunks * args.chunk
    value = world * positions_per_step / (ms / 1000.0)

    # e2e through the evaluator closure (host batch, H2D + D2H per chunk)
    ev = mb.network_evaluate(net, mb.evaluator.EvaluatorConfig(device=str(device), autocast=True, mass_floor=0.2,
                                                                gemm=args.gemm))

    def step_e2e():
        for _ in range(n_chunks):
            ev(host_pinned)

    for _ in range(max(1, args.warmup)):
        step_e2e()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        step_e2e()
    e1.record()
    torch.cuda.synchronize()
    ms_e2e = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    e2e_value = world * positions_per_step / (ms_e2e / 1000.0)
    # The whole box's host encoder rate (the ranks encoded concurrently on the
    # shared host cores): a self-play pipeline that encodes what the GPUs
    # evaluate runs at the smaller of it and the end-to-end rate.
    enc_box = encoder["value"]
    if world > 1:
        t = torch.tensor([enc_box], dtype=torch.float64, device=device)
        dist.all_reduce(t)
        enc_box = float(t.item())
    h2d = batch_bytes(host_pinned, fields) * n_chunks
    d2h = 3 * host.n_cells * 4 * n_chunks

    # Roofline of the dominant native kernel (the larger total time inside the
    # timed region): the fused projection launches or the radius read.
    roof = None
    if rank == 0:
        n_dec = int(tables.dec_window.numel())
        roof = dominant_roofline([
            resid_ln_roofline(probe), radius_roofline(probe, tables, cfg),
            segment_roofline(probe, "cell_read", "radius_read_kernel (block-diagonal read: cells<-windows, class rows)"
                             if tables.cr_slots is not None else "segment_attention_kernel (cells<-windows, class rows)",
                             tables.N_c, tables.N_w, n_dec, cfg, 726, packed=tables.cr_slots is not None),
            segment_roofline(probe, "window_read", "radius_read_kernel (block-diagonal read: windows<-cells)"
                             if tables.wr_slots is not None else "segment_attention_kernel (windows<-cells)",
                             tables.N_w, tables.N_c, n_dec, cfg, 726, packed=tables.wr_slots is not None)])

    # p50 batch-64 latency (config-4 distribution: 40-150 stones), end to end
    p50 = None
    if rank == 0 and args.latency:
        lat_specs = make_specs(64, 40, 150, seed=77)
        lat_batch = mb.encoder.encode(lat_specs, pin_memory=True, narrow=True)
        times = []
        for i in range(3 + 20):
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            ev(lat_batch)
            dt = time.perf_counter() - t0
            if i >= 3:
                times.append(dt * 1000.0)
        p50 = statistics.median(times)

    # The reference's own GPU path on the same chunk (its KLENT evaluator,
    # Triton kernels JIT-compiled for this GPU, bf16 autocast, host batch in
    # and CPU outputs back, as network_evaluate does), when the reference is
    # installed in baseline/_ref.
    ref_gpu = None
    if rank == 0 and world == 1 and args.ref_gpu:
        ref_gpu = reference_gpu_rate(host, n_chunks, device)

    cpu = None
    if rank == 0 and world == 1 and args.cpu_sample > 0:
        threads = os.cpu_count() or 1
        rate, dt = cpu_forward_rate(specs, args.cpu_sample, threads)
        cpu = {"value": rate, "unit": "positions/s", "cores": threads, "kind": "port",
               "sample": f"{args.cpu_sample} late positions ({args.lo}-{args.hi} stones), fp32 eager torch-CPU "
                         f"oracle forward, {dt:.1f} s"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "positions/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {
                "workload": (f"config 5: {positions_per_step} late positions per GPU ({args.lo}-{args.hi} stones), "
                             f"{n_chunks} chunks of {args.chunk} ({len(specs)} distinct seeded positions per rank, "
                             "repeated to fill a chunk); config-4 architecture"),
                "arch": ARCH, "positions_per_gpu": positions_per_step, "chunk": args.chunk, "gemm": args.gemm,
                "cells_per_chunk": host.n_cells, "windows_per_chunk": host.n_windows,
                "radius_edges_per_chunk": int(host.radius_src.numel()),
                "l2": "inputs larger than L2 (one chunk's device tables exceed 126 MB)",
            },
            "e2e": {"value": e2e_value, "unit": "positions/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "gpu_launches": launches,
            "roofline": roof,
            "cpu_baseline": cpu,
            "clocks": clocks.summary(),
            "p50_batch64_ms": p50,
            "encoder": encoder,
            "pipeline": {"value": min(enc_box, e2e_value), "unit": "positions/s", "encoder_box": enc_box,
                         "bound": "host encoder" if enc_box < e2e_value else "gpus",
                         "note": "encode + evaluate on this box: the smaller of the summed concurrent encoder "
                                 "rates of the ranks and the end-to-end rate"},
            "reference_gpu": ref_gpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def reference_gpu_rate(host, n_chunks, device, repeats=3):
    """Positions/s of the reference's KLENT evaluator (klent/train.py:100-120)
    on one chunk of the benchmark's batch (the same arrays, as the
    reference's Batch), on this GPU: its Triton kernels JIT-compile on the
    first call (untimed); the median of ``repeats`` timed calls. None when
    the reference is not installed in baseline/_ref."""
    reference_pkg = _reference_pkg()
    if reference_pkg is None:
        return None
    import importlib
    import torch

    mn = reference_pkg.load()
    train = importlib.import_module("mantisnet.klent.train")
    batch = mn.builder.Batch(**vars(host))
    torch.manual_seed(0)
    net = mn.MantisNet(mn.MantisConfig(**ARCH))
    with torch.no_grad():
        for head in (net.mlp_p, net.mlp_q):
            head.out.weight.normal_(std=0.02)
            head.out.bias.normal_(std=0.02)
    net = net.to(device).eval()
    ev = train.network_evaluate(net, train.KlentConfig(device=str(device), autocast=True, mass_floor=0.2))
    ev(batch)  # JIT compilation and autotuning
    times = []
    for _ in range(repeats):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        ev(batch)
        torch.cuda.synchronize()
        times.append(time.perf_counter() - t0)
    sec = statistics.median(times)
    return {"value": host.n_pos / sec, "unit": "positions/s", "ms_per_chunk": sec * 1000.0,
            "impl": "reference mantisnet network_evaluate (Triton kernels for this GPU, bf16 autocast, host batch "
                    "in, CPU outputs out)", "positions": host.n_pos, "timed_calls": repeats}


def radius_read_bytes(T, cfg):
    """Algorithmic HBM bytes of one radius read (cells <- stones): per cell its
    bf16 query row in and output row out, its run bound and its slot in the
    edge-count order (one 16-byte slot); per edge the packed int32 stone | class; each stone's
    bf16 K and V rows once; the bf16 class value rows and fp32 bias rows once."""
    h, n_cls = cfg.h, 192
    return (T.N_c * h * 2 * 2 + T.N_c * 16 + int(T.r_src.numel()) * 4 + T.N_s * 2 * h * 2
            + n_cls * h * 2 + cfg.heads * n_cls * 4)


# DRAM bytes per cell of one radius read, from an ncu capture of the same
# kernel (dram__bytes_read.sum + dram__bytes_write.sum = 445.8 MB over 438,658
# cells; profiles/radius_read_64pos.md), scaled to the timed launch by its
# cell count.
RADIUS_DRAM_BYTES_PER_CELL = 445_866_240 / 438_658


def radius_roofline(probe, T, cfg):
    """The radius read's launches inside the timed region (CUDA events on the
    launching stream around each launch, recorded by the engine's probe)."""
    ev = probe.get("radius_read", [])
    if not ev:
        return None
    ms = [s.elapsed_time(e) for s, e in ev]
    sec = statistics.mean(ms) / 1000.0
    algo = radius_read_bytes(T, cfg)
    pk, kind = peaks()
    achieved = algo / sec / 1e9
    return {"kernel": "radius_read_kernel (packed edges, cells<-stones)", "bound": "hbm",
            "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
            "traffic": RADIUS_DRAM_BYTES_PER_CELL * T.N_c, "traffic_source": "ncu capture at 64 positions, scaled by cells",
            "peak_kind": kind, "algorithmic_bytes": algo, "launch_ms": sec * 1000.0,
            "launches_timed": len(ms), "edges": int(T.r_src.numel()), "total_ms": sum(ms)}


def segment_roofline(probe, name, kernel, n_q, n_src, n_edges, cfg, n_cls, packed=True):
    """An incidence read's launches inside the timed region: algorithmic
    bytes per launch (per query row its bf16 query and output rows and its
    16-byte slot, per edge its packed int32 source | class; or, on the generic
    kernel, the run bound and the int64 source and class; each source's bf16
    K and V rows once, class value rows and bias once) over the mean
    CUDA-event duration."""
    ev = probe.get(name, [])
    if not ev:
        return None
    h = cfg.h
    per_row, per_edge = (16, 4) if packed else (8, 16)
    algo = (n_q * (2 * h * 2 + per_row) + n_edges * per_edge + n_src * 2 * h * 2 + n_cls * (h * 2 + cfg.heads * 4))
    ms = [s.elapsed_time(e) for s, e in ev]
    sec = statistics.mean(ms) / 1000.0
    pk, kind = peaks()
    achieved = algo / sec / 1e9
    return {"kernel": kernel, "bound": "hbm", "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s",
            "frac": achieved / pk["hbm_gbs"], "traffic": None, "peak_kind": kind, "algorithmic_bytes": algo,
            "launch_ms": sec * 1000.0, "launches_timed": len(ms), "edges": n_edges, "total_ms": sum(ms)}


# DRAM bytes (read + write) over algorithmic bytes of the fused projection +
# residual + LayerNorm launch, from the ncu capture of
# `bench.py --op resid_ln --rows 262144` (2 outputs): 886.1 MB over 939.5 MB.
# Below 1 because part of the last writes is still in L2 when the kernel ends.
RESID_LN_TRAFFIC_RATIO = 886.1 / 939.5


def resid_ln_roofline(probe):
    """The fused projection + residual + LayerNorm launches inside the timed
    region: algorithmic bytes over CUDA-event time, per launch on average."""
    ev = probe.get("resid_ln", [])
    byt = probe.get("resid_ln_bytes", [])
    if not ev or len(ev) != len(byt):
        return None
    ms = [s.elapsed_time(e) for s, e in ev]
    sec = statistics.mean(ms) / 1000.0
    algo = statistics.mean(byt)
    pk, kind = peaks()
    achieved = algo / sec / 1e9
    return {"kernel": "rowgemm_kernel<COPY, RESID_LN> (projection + residual + LayerNorms, tcgen05)", "bound": "hbm",
            "achieved": achieved, "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": achieved / pk["hbm_gbs"],
            "traffic": algo * RESID_LN_TRAFFIC_RATIO,
            "traffic_source": "ncu capture of bench.py --op resid_ln --rows 262144, DRAM/algorithmic ratio",
            "peak_kind": kind, "algorithmic_bytes": algo, "launch_ms": sec * 1000.0, "launches_timed": len(ms),
            "total_ms": sum(ms)}


def dominant_roofline(cands):
    """The candidate with the largest total time in the timed region, with the
    runner-up under ``next`` (None when there is no candidate)."""
    cands = sorted((r for r in cands if r is not None), key=lambda r: -r["total_ms"])
    if not cands:
        return None
    roof = dict(cands[0])
    if len(cands) > 1:
        roof["next"] = cands[1]
    if len(cands) > 2:
        roof["others"] = cands[2:]
    return roof


def _time_launches(fn, steps, warmup):
    """Mean CUDA-event time of ``fn`` over ``steps`` launches after ``warmup``."""
    import torch

    for _ in range(max(warmup, 3)):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / steps


def run_op(args):
    """One JSON line for an isolated-op workload on one GPU (inputs resident;
    both inputs are larger than L2): ``hex`` = the fused hex message pass over
    4096 x 256 cell tokens, ``axial`` = the axial-bias attention over 4096
    positions x 8 heads x 256 tokens. Not the headline metric."""
    import numpy as np
    import torch

    mb = _pkg()
    ops = mb.ops
    dev = torch.device("cuda", 0)
    pk, kind = peaks()
    g = torch.Generator(device=dev).manual_seed(0)
    p = args.positions
    if args.op == "resid_ln":
        # x += a W^T + b, then LayerNorms of x: the trunk's residual updates
        m, n_out = args.rows, args.ln_outputs
        a = torch.randn(m, 256, device=dev, generator=g).to(torch.bfloat16)
        img = ops.weight_image(torch.randn(256, 256, device=dev, generator=g) * 0.05)
        b = torch.randn(256, device=dev, generator=g) * 0.1
        x = torch.randn(m, 256, device=dev, generator=g)
        outs = [(torch.randn(256, device=dev, generator=g) * 0.1 + 1, torch.randn(256, device=dev, generator=g) * 0.1,
                 torch.empty(m, 256, dtype=torch.bfloat16, device=dev)) for _ in range(n_out)]
        ms = _time_launches(lambda: ops.gemm_rows_ln(a, img, b, x, outs), args.steps, args.warmup)
        algo = m * (512 + 2048 + 512 * n_out)
        line = {"metric": "fused projection + residual + LayerNorm rows/s", "value": m / (ms / 1000.0),
                "unit": "rows/s", "ms_per_step": ms,
                "config": {"workload": f"{m} rows x 256, bf16 input, fp32 residual, {n_out} bf16 LayerNorm outputs"},
                "roofline": {"kernel": "rowgemm_kernel<COPY, RESID_LN>", "bound": "hbm", "achieved": algo / ms / 1e6,
                             "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": algo / ms / 1e6 / pk["hbm_gbs"],
                             "peak_kind": kind, "algorithmic_bytes": algo}}
    elif args.op == "radius":
        # the radius read of one trunk block over encoder-built late positions
        # (tables derived as the engine derives them, packed edges shared)
        specs = make_specs(min(p, 256), args.lo, args.hi, seed=1000)
        host = mb.encoder.encode((specs * math.ceil(p / len(specs)))[:p])
        cfg = mb.MantisConfig(**ARCH)
        b = mb.evaluator.to_device(host, dev, mb.evaluator.needed_fields(cfg))
        T = mb.model._Tables(cfg, b, torch.bfloat16)
        q = torch.randn(T.N_c, cfg.h, device=dev, generator=g).to(torch.bfloat16)
        kv = torch.randn(T.N_s, 2 * cfg.h, device=dev, generator=g).to(torch.bfloat16)
        bias = torch.randn(cfg.heads, 192, device=dev, generator=g) * 0.02
        vcls = (torch.randn(192, cfg.h, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        h, stage = cfg.h, T.max_t - 4
        out = torch.empty_like(q)
        ms = _time_launches(lambda: ops.radius_read(q, kv[:, :h], kv[:, h:], bias, vcls, T.r_ptr, T.r_pack_slots,
                                                    T.cell_off, T.stone_off, stage, order=T.r_order, out=out,
                                                    slots=T.r_slots),
                            args.steps, args.warmup)
        algo = radius_read_bytes(T, cfg)
        line = {"metric": "radius read cells/s", "value": T.N_c / (ms / 1000.0), "unit": "cells/s", "ms_per_step": ms,
                "config": {"workload": f"radius read of {p} late positions ({args.lo}-{args.hi} stones)",
                           "cells": T.N_c, "edges": int(T.r_src.numel())},
                "roofline": {"kernel": "radius_read_kernel", "bound": "hbm", "achieved": algo / ms / 1e6,
                             "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": algo / ms / 1e6 / pk["hbm_gbs"],
                             "peak_kind": kind, "algorithmic_bytes": algo}}
    elif args.op == "hex":
        nbr, _ = mb.hexgraph.message_graph(p, 256, 40, 200, seed=1)
        n = nbr.shape[0]
        x = torch.randn(n, 256, device=dev, generator=g).to(torch.bfloat16)
        w = (torch.randn(256, 256, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        b = torch.randn(256, device=dev, generator=g) * 0.02
        nb = torch.from_numpy(nbr).to(dev)
        img = ops.weight_image(w)
        out = torch.empty_like(x)
        ms = _time_launches(lambda: ops.hex_message_pass(x, nb, img, b, out=out), args.steps, args.warmup)
        algo = 2 * n * 256 * 2 + n * 6 * 4 + 256 * 256 * 2 + 256 * 4
        flops = 2 * n * 256 * 256
        # the fp32 eager CPU restatement on the first 16 positions (all host threads), scaled per node
        from oracle import isolated as ISO
        torch.set_num_threads(os.cpu_count() or 1)
        sub = 16 * 256
        xs, ns, ws, bs = x[:sub].float().cpu(), nb[:sub].cpu().clone(), w.float().cpu(), b.cpu()
        ns[ns >= sub] = -1
        ISO.hex_message_pass(xs, ns, ws, bs)
        t0 = time.perf_counter()
        ISO.hex_message_pass(xs, ns, ws, bs)
        cpu_ms = (time.perf_counter() - t0) * 1000.0
        line = {"metric": "hex message-pass nodes/s (config 3)", "value": n / (ms / 1000.0), "unit": "nodes/s",
                "ms_per_step": ms, "config": {"workload": f"config 3: {p} x 256 cell tokens, F=256, bf16", "nodes": n},
                "cpu_baseline": {"kind": "port", "sample": f"{sub} nodes (16 positions), fp32 eager CPU restatement",
                                 "ms": cpu_ms, "cores": os.cpu_count() or 1,
                                 "value": sub / (cpu_ms / 1000.0), "unit": "nodes/s"},
                "roofline": {"kernel": "hex_window_kernel" if x.stride(0) == 256 else "rowgemm_kernel<HEXMEAN, ADD_X>",
                             "bound": "hbm",
                             "achieved": algo / ms / 1e6, "peak": pk["hbm_gbs"], "unit": "GB/s",
                             "frac": algo / ms / 1e6 / pk["hbm_gbs"], "peak_kind": kind, "algorithmic_bytes": algo,
                             "tflops": flops / ms / 1e9}}
    else:
        coords, valid = mb.hexgraph.attention_layout(p, 256, seed=2)
        q, k, v = (torch.randn(p, 8, 256, 32, device=dev, generator=g).to(torch.bfloat16) for _ in range(3))
        c = torch.from_numpy(coords).to(dev)
        vl = torch.from_numpy(valid).to(dev)
        bias = torch.randn(33, 33, 8, device=dev, generator=g) * 0.02
        out = torch.empty_like(q)
        ms = _time_launches(lambda: ops.axial_attention(q, k, v, c, vl, bias, out=out), args.steps, args.warmup)
        lv = valid.astype(np.float64)
        flops = float((8 * 4 * 32 * lv ** 2).sum())
        algo = float(((3 * lv + 256) * 8 * 32 * 2 + 256 * 8 + 4).sum() + 33 * 33 * 8 * 4)
        # the fp32 eager CPU restatement on the first 16 positions (all host threads)
        from oracle import isolated as ISO
        torch.set_num_threads(os.cpu_count() or 1)
        qs, ks, vs = (t[:16].float().cpu() for t in (q, k, v))
        cs, vls, bs = c[:16].cpu(), vl[:16].cpu(), bias.cpu()
        ISO.axial_attention(qs[:2], ks[:2], vs[:2], cs[:2], vls[:2], bs)
        t0 = time.perf_counter()
        ISO.axial_attention(qs, ks, vs, cs, vls, bs)
        cpu_ms = (time.perf_counter() - t0) * 1000.0
        line = {"metric": "axial-bias attention positions/s (config 2)", "value": p / (ms / 1000.0),
                "unit": "positions/s", "ms_per_step": ms,
                "cpu_baseline": {"kind": "port", "sample": "16 positions, fp32 eager CPU restatement", "ms": cpu_ms,
                                 "cores": os.cpu_count() or 1, "value": 16 / (cpu_ms / 1000.0),
                                 "unit": "positions/s"},
                "config": {"workload": f"config 2: {p} positions x 8 heads x 256 tokens, d=32, bf16"},
                "roofline": {"kernel": "axial_attention_kernel", "bound": "hbm", "achieved": algo / ms / 1e6,
                             "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": algo / ms / 1e6 / pk["hbm_gbs"],
                             "peak_kind": kind, "algorithmic_bytes": algo, "algorithmic_flops": flops,
                             "tflops": flops / ms / 1e9, "tensor_frac": flops / ms / 1e9 / pk["bf16_tflops"]}}
    line.update({"n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "dtype": "bf16",
                 "data": "synthetic", "gpu_launches": 1})
    print(json.dumps(line))


def run_config1(args):
    """One JSON line per knob set for the config-1 baseline: 16 positions of
    10-40 stones at the reference's default architecture (h=128, 4 blocks, 4
    heads), the default (relay) knobs and the production knobs (cell_latents +
    cell_nodes). This build's full forward (every head) on the GPU in fp32
    and bf16, the batch resident, CUDA events (median of 20 after 3 warm-ups),
    against the reference's own eager CPU `MantisNet.forward` from
    baseline/_ref on all host threads (median of --steps after one warm-up),
    and the reference's Python builder (build + collate) on the same
    positions."""
    import torch

    mb = _pkg()
    specs = make_specs(16, 10, 40, seed=17)
    host = mb.collate([mb.from_spec(s) for s in specs])
    dev = torch.device("cuda", 0)
    ref = _reference_pkg()
    mn = ref.load() if ref is not None else None
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    builder_ms = None
    if mn is not None:
        times = []
        for _ in range(3):
            t0 = time.perf_counter()
            mn.builder.collate([mn.builder.build(s.stone_qr, s.stone_owner, s.mover, s.legal_qr, s.moves_remaining)
                                for s in specs])
            times.append((time.perf_counter() - t0) * 1000.0)
        builder_ms = statistics.median(times)
    for name, knobs in (("relay", {}), ("production", {"cell_latents": True, "cell_nodes": True})):
        cfg = mb.MantisConfig(**knobs)
        torch.manual_seed(0)
        net = mb.MantisNet(cfg).to(dev).eval()
        b = mb.evaluator.to_device(host, dev, tuple(k for k, v in vars(host).items() if isinstance(v, torch.Tensor)))
        ours = {}
        for dtype, key in ((torch.float32, "fp32"), (torch.bfloat16, "bf16")):
            for _ in range(3):
                net.forward(b, 0.2, dtype)
            ms = []
            for _ in range(20):
                s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s0.record()
                net.forward(b, 0.2, dtype)
                s1.record()
                torch.cuda.synchronize()
                ms.append(s0.elapsed_time(s1))
            ours[key] = statistics.median(ms)
        ref_ms = None
        if mn is not None:
            torch.manual_seed(0)
            rnet = mn.MantisNet(mn.MantisConfig(**knobs)).eval()
            rb = mn.builder.Batch(**vars(host))
            times = []
            with torch.no_grad():
                for i in range(1 + max(args.steps, 5)):
                    t0 = time.perf_counter()
                    rnet(rb, 0.2)
                    if i > 0:
                        times.append((time.perf_counter() - t0) * 1000.0)
            ref_ms = statistics.median(times)
        print(json.dumps({
            "metric": "config 1 forward ms (16 positions, 10-40 stones, h128/4 blocks/4 heads)", "knobs": name,
            "b200_ms": ours, "b200_positions_per_s": {k: 16 / (v / 1000.0) for k, v in ours.items()},
            "reference_cpu_ms": ref_ms,
            "reference_cpu_positions_per_s": (16 / (ref_ms / 1000.0)) if ref_ms else None,
            "reference_builder_ms": builder_ms, "host_cores": threads, "torch_threads": torch.get_num_threads(),
            "data": "synthetic", "unit": "ms"}), flush=True)


def run_multi(args):
    """One JSON line: ``network_evaluate_multi`` over ``--devices`` GPUs of
    this process (default: all visible), each call one batch of ``--chunk``
    late positions per device, cut into cost-balanced slices; host batch in
    (pinned), CPU outputs back. Not the headline metric (the headline runs
    one process per GPU)."""
    import torch

    mb = _pkg()
    n_dev = args.devices or torch.cuda.device_count()
    specs = make_specs(args.unique, args.lo, args.hi, seed=1000)
    reps = math.ceil(args.chunk * n_dev / len(specs))
    host = mb.encoder.encode((specs * reps)[: args.chunk * n_dev], pin_memory=True)
    torch.manual_seed(0)
    net = mb.MantisNet(mb.MantisConfig(**ARCH))
    with torch.no_grad():
        for head in (net.mlp_p, net.mlp_q):
            head.out.weight.normal_(std=0.02)
            head.out.bias.normal_(std=0.02)
    net = net.to("cuda:0").eval()
    cfg = mb.evaluator.EvaluatorConfig(device="cuda:0", autocast=True, mass_floor=0.2, gemm=args.gemm)
    ev = mb.evaluator.network_evaluate_multi(net, cfg, [f"cuda:{i}" for i in range(n_dev)])
    try:
        for _ in range(args.warmup):
            ev(host)
        times = []
        for _ in range(args.steps):
            t0 = time.perf_counter()
            ev(host)
            times.append(time.perf_counter() - t0)
    finally:
        ev.close()
    sec = statistics.median(times)
    off = mb.evaluator._offsets(host, ev.fields)
    cuts = mb.sharding.balanced_cuts(ev.costs(host, off), n_dev)
    print(json.dumps({
        "metric": "positions/s, one network_evaluate_multi call over the devices (host batch in, CPU outputs out)",
        "value": host.n_pos / sec, "unit": "positions/s", "devices": n_dev, "ms_per_call": sec * 1000.0,
        "positions_per_call": host.n_pos, "slice_positions": [b - a for a, b in zip(cuts, cuts[1:])],
        "steps": args.steps, "warmup": args.warmup, "dtype": "bf16", "data": "synthetic", "lost": sorted(ev.lost)}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--positions", type=int, default=4096)
    ap.add_argument("--chunk", type=int, default=512)
    ap.add_argument("--unique", type=int, default=256)
    ap.add_argument("--lo", type=int, default=150)
    ap.add_argument("--hi", type=int, default=300)
    ap.add_argument("--cpu-sample", type=int, default=4)
    ap.add_argument("--ref-sample", type=int, default=1,
                    help="positions per step of the reference arm (its eager CPU path takes seconds per position)")
    ap.add_argument("--latency", type=int, default=1)
    ap.add_argument("--gemm", default="tcgen05-ln", help="dense projection path (see model.Engine)")
    ap.add_argument("--devices", type=int, default=0, help="GPUs of --op multi (default: all visible)")
    ap.add_argument("--op", default=None, choices=["hex", "axial", "resid_ln", "radius", "multi", "config1"],
                    help="time one isolated-op workload instead of the evaluator (config 3 / config 2 / the "
                         "fused projection + residual + LayerNorm launch)")
    ap.add_argument("--rows", type=int, default=1814720, help="rows of --op resid_ln (default: one chunk's windows)")
    ap.add_argument("--ref-gpu", type=int, default=1,
                    help="also time the reference's own GPU evaluator on one chunk (needs baseline/_ref)")
    ap.add_argument("--ln-outputs", type=int, default=2, help="LayerNorm outputs of --op resid_ln (1-3)")
    args = ap.parse_args()
    if args.op == "multi":
        run_multi(args)
        return
    if args.op == "config1":
        run_config1(args)
        return
    if args.op:
        run_op(args)
        return
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local_rank = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
