"""Benchmark of the B200 FP16 matmul path on the 96-shape grid (and the other configurations).

Which configuration runs:

* plain ``python bench.py`` (one process): the 96-shape grid, the configuration the headline
  metric is quoted on; ``--workload`` picks another (decode, sweep, colpar, rmsnorm);
* under ``torch.distributed.run`` (any number of ranks, one included): the column-parallel GEMM
  (M=8192, K=8192, N=57344 split N-wise over the ranks, slices exchanged over NVLink), the one
  configuration that is sharded over GPUs; the grid shapes are one-GPU problems.

Grid flow, as the reference's protocol (bank 1 selects, bank 2 scores):

1. tuning (untimed): the Thompson-sampling bandit probes ``--budget`` candidates per shape
   with live timed launches (every probe's output is checked against an FP32 reference);
2. ``--warmup`` untimed passes, then ``--steps`` timed passes over the 96 shapes with each
   shape's recommended variant through the public API (``action_expansion.launch``: output and
   workspace allocated per call). Before every launch a 256 MiB write flushes L2; each launch is
   bracketed by CUDA events on the launching stream. The same passes with cuBLAS
   ``torch.matmul`` give the comparison;
3. the bank-2 output of every chosen candidate is checked against the FP32 product, beside
   cuBLAS's error on the same inputs;
4. an end-to-end pass: host->device copies of the pass's distinct A and B tensors from pinned
   memory, the launches, and the device->host copy of every C, inside the events;
5. on rank 0 at N=1, the CPU baseline: FP16 ``torch.matmul`` on all host cores.

``value`` is the grid's aggregate TFLOP/s (total FLOPs of one pass / sum of per-shape median
latencies), ``geomean_latency_vs_cublas`` the headline ratio.

``--impl reference`` times the reference's CPU path (FP16 ``torch.matmul`` on the host cores,
through the oracle) on the same configuration.
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

import numpy as np

ROOT = Path(__file__).resolve().parent
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

METRIC = "geomean latency/cuBLAS torch.matmul, 96-shape FP16 grid; TFLOP/s & % roofline"
COLPAR_METRIC = "column-parallel FP16 GEMM M=8192 K=8192 N=57344: TFLOP/s (whole job)"


def _metric(args, count: int) -> str:
    """The headline metric's name for the grid; the same form naming the shape set otherwise."""
    if args.workload == "colpar" and not args.shapes:
        return COLPAR_METRIC
    if args.workload == "grid" and not args.shapes:
        return METRIC
    name = "custom shapes" if args.shapes else args.workload
    return METRIC.replace("96-shape FP16 grid", f"{count}-shape FP16 {name}")
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}


def _peaks() -> tuple[dict[str, float], str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {k: float(data[k]) for k in FALLBACK_PEAKS if k in data}, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def _distributed_launch() -> bool:
    """Whether ``torch.distributed.run`` started this process (it sets these for every rank)."""
    return "TORCHELASTIC_RUN_ID" in os.environ or "LOCAL_WORLD_SIZE" in os.environ


def _config(args, workloads) -> dict[str, object]:
    """The ``config`` object of the JSON line; both arms print the same one."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if args.workload == "colpar":
        from heliostune_b200.column_parallel import column_parallel_candidate, default_peer_writes

        (w,) = workloads
        exchange = (
            f"fused: GEMM epilogue writes every tile to all ranks over NVLink ({getattr(args, 'peer_writes', None) or default_peer_writes(world)})"
            if args.exchange == "fused" and world > 1
            else "NCCL all-gather + column assembly" if world > 1 else "none (one rank holds all of N)"
        )
        return {
            "workload": f"colpar M={w.m} N={w.n} K={w.k}",
            "parallelism": f"column-parallel x{world}",
            "gemm": column_parallel_candidate(w.m, w.n // world).key,
            "exchange": exchange,
            "l2": "operands larger than L2",
        }
    workload = f"{args.workload}: {len(workloads)} shapes" if not args.shapes else f"shapes {args.shapes}"
    selection = f"Thompson bandit ({getattr(args, 'features', 'v2')} features), {args.budget} probes per shape on bank-1 tensors"
    if args.force:
        selection = f"forced: {args.force}"
    elif args.choices:
        selection = f"choices of {Path(args.choices).name}"
    elif args.confirm > 1:
        selection += (
            f"; the best {args.confirm} probes within {args.confirm_within:.2f}x re-timed side by side in"
            " 5 passes on bank-1 tensors"
        )
    return {
        "workload": workload,
        "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
        "l2": "256 MiB write before every launch",
        "selection": selection + "; scored on bank-2 tensors",
        "timing": "per-launch CUDA events on the launching stream; per-shape median over steps",
    }


def _workloads(name: str, shapes: str | None):
    from heliostune_b200.configs import (
        COLUMN_PARALLEL_WORKLOAD,
        DECODE_WORKLOAD,
        GRID_WORKLOADS,
        SWEEP_WORKLOADS,
        Workload,
    )

    if shapes:
        out = []
        for spec in shapes.split(","):
            m, n, k = (int(v) for v in spec.lower().split("x"))
            out.append(Workload(m=m, n=n, k=k, model="custom", projection="custom", regime=f"m{m}"))
        return tuple(out)
    return {
        "grid": GRID_WORKLOADS,
        "sweep": SWEEP_WORKLOADS,
        "decode": (DECODE_WORKLOAD,),
        "colpar": (COLUMN_PARALLEL_WORKLOAD,),
    }[name]


# ----------------------------------------------------------------------------------------------
# Clock sampling during the timed region
# ----------------------------------------------------------------------------------------------


class ClockSampler:
    QUERY = (
        "timestamp,index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
        "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
        "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    )

    def __init__(self, device: int) -> None:
        self.device = device
        self.proc: subprocess.Popen[str] | None = None

    def __enter__(self) -> ClockSampler:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits", "-lms", "25"],
                stdout=subprocess.PIPE,
                stderr=subprocess.DEVNULL,
                text=True,
            )
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc: object) -> None:
        self.output = ""
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.output, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.output, _ = self.proc.communicate()

    def summary(self, start: float | None = None, end: float | None = None) -> dict[str, object]:
        """Median SM clock and throttle reasons of the samples inside [start, end] (epoch s)."""
        from datetime import datetime

        clocks, max_clock, reasons = [], None, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in getattr(self, "output", "").splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 10:
                continue
            try:
                stamp = datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                clock = float(parts[2])
                max_clock = float(parts[3])
            except ValueError:
                continue
            if start is not None and not start - 0.03 <= stamp <= end + 0.03:
                continue
            clocks.append(clock)
            for name, flag in zip(names, parts[6:10], strict=True):
                if flag.lower() == "active":
                    reasons.add(name)
        return {
            "sm_mhz": statistics.median(clocks) if clocks else None,
            "sm_max_mhz": max_clock,
            "reasons": sorted(reasons),
            "samples": len(clocks),
        }


# ----------------------------------------------------------------------------------------------
# Our arm
# ----------------------------------------------------------------------------------------------


def _make_operands(workloads, device, seed_base: int):
    """A per (K, M) and B per (K, N), shared across the shapes that use them."""
    import torch

    a_cache: dict[tuple[int, int], torch.Tensor] = {}
    b_cache: dict[tuple[int, int], torch.Tensor] = {}
    for w in workloads:
        if (w.k, w.n) not in b_cache:
            g = torch.Generator(device=device).manual_seed(seed_base + 7919 * w.k + w.n)
            b_cache[(w.k, w.n)] = (torch.randn((w.k, w.n), generator=g, device=device) / math.sqrt(w.k)).to(torch.float16)
        if (w.k, w.m) not in a_cache:
            g = torch.Generator(device=device).manual_seed(seed_base + 104729 * w.k + w.m)
            a_cache[(w.k, w.m)] = (torch.randn((w.m, w.k), generator=g, device=device) / math.sqrt(w.k)).to(torch.float16)
    return {w.key: (a_cache[(w.k, w.m)], b_cache[(w.k, w.n)]) for w in workloads}


def _kernel_family(candidate) -> str:
    """Roofline family of a candidate: its launch family, with the 256 x 512 pair tile and the
    128-deep 256 x 256 pair tile apart."""
    config = candidate.config
    if candidate.family == "pair" and config.block_n == 512:
        return "pair_wide"
    if candidate.family == "pair" and config.block_n == 256 and config.block_k == 128:
        return "pair_deep_k"
    return candidate.family


def _launch_count(candidate, workload, sm_count: int) -> int:
    from heliostune_b200.action_configs import SplitKConfig, StreamConfig, split_plan, stream_splits

    config = candidate.config
    if isinstance(config, SplitKConfig):
        bk = 64 if config.block_k <= 64 else 128
        return 1 + (split_plan(workload.k, bk, config.split_k)[1] > 1)
    return 1  # tile, persistent, pair and stream (in-cluster reduction) are one launch


def run_ours(args: argparse.Namespace) -> dict[str, object] | None:
    import torch
    import torch.distributed as dist

    from heliostune_b200 import _native
    from heliostune_b200.action_configs import b200_candidates_for
    from heliostune_b200.action_expansion import fp32_reference, launch
    from heliostune_b200.kernel import get_hardware_profile, require_b200
    from heliostune_b200.timing import do_bench, flush_buffer
    from heliostune_b200.tuner import thompson_probe

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=device)
    _native.library()  # fails loudly if the native path is missing
    hardware = get_hardware_profile("B200", device)
    require_b200(hardware)
    sm_count = hardware.multiprocessor_count
    workloads = _workloads(args.workload, args.shapes)
    operands = _make_operands(workloads, device, seed_base=2)  # bank 2 tensors for scoring
    tune_operands = _make_operands(workloads, device, seed_base=1)  # bank 1 tensors for tuning
    flush = flush_buffer(device)

    # ---- 1. tuning (bank 1) ------------------------------------------------------------
    def measure(workload, candidate) -> float:
        a, b = tune_operands[workload.key]
        out = launch(a, b, candidate)
        expected = fp32_reference(a, b)
        scale = expected.abs().max().item()
        err = (out.float() - expected).abs().max().item() / max(scale, 1e-30)
        ok = bool(torch.all((out.float() - expected).abs() <= 1e-2 + 1e-2 * expected.abs()).item())
        del expected, out
        if not ok or not err <= 1e-2:
            raise ValueError(f"parity failure (normwise {err:.3g})")
        return do_bench(lambda: launch(a, b, candidate), warmup_ms=2.0, rep_ms=args.probe_ms, quantiles=(0.5,))[0]

    # ---- 0. the pre-timing correctness gate: every pool candidate on a small sample --------
    from heliostune_b200.configs import validation_workloads
    from heliostune_b200.hopper_kernel import assert_candidate_kernels_correct

    gate = assert_candidate_kernels_correct(
        "B200", candidates_for=b200_candidates_for, workloads=validation_workloads(workloads)
    )

    t0 = time.perf_counter()
    chosen = {}
    if args.force:
        from heliostune_b200.action_configs import PAIR_SPLIT_CANDIDATES, PAIR_STREAM_K_CANDIDATE

        for w in workloads:
            by_key = {c.key: c for c in (*b200_candidates_for(w), *PAIR_SPLIT_CANDIDATES, PAIR_STREAM_K_CANDIDATE)}
            chosen[w.key] = by_key[args.force]
        from heliostune_b200.tuner import ProbeResult

        tuning = ProbeResult(probes={}, recommendations=dict(chosen))
    elif args.choices:
        # Reuse the selection of an earlier run (profiling runs skip the tuning launches).
        saved = {row["workload"]: row["choice"] for row in json.loads(Path(args.choices).read_text())["shapes"]}
        for w in workloads:
            by_key = {c.key: c for c in b200_candidates_for(w)}
            chosen[w.key] = by_key[saved[w.key]]
        from heliostune_b200.tuner import ProbeResult

        tuning = ProbeResult(probes={}, recommendations=dict(chosen))
    else:
        tuning = thompson_probe(
            workloads, b200_candidates_for, measure, hardware, budget=args.budget, policy_seed=args.seed, basis=args.features
        )
        for w in workloads:
            if w.key not in tuning.recommendations:
                raise RuntimeError(f"no valid candidate for {w.key}")
            chosen[w.key] = tuning.recommendations[w.key]
    # ---- 2. scored passes (bank 2) ---------------------------------------------------------
    def one_pass(fn_for, events) -> None:
        for i, w in enumerate(workloads):
            a, b = operands[w.key]
            fn = fn_for(w)
            flush.zero_()
            events[i][0].record()
            fn(a, b)
            events[i][1].record()

    def ours_fn(w):
        cand = chosen[w.key]
        return lambda a, b: launch(a, b, cand)

    def cublas_fn(w):
        return lambda a, b: torch.matmul(a, b)

    n = len(workloads)

    def timed(fn_for, steps: int, warmup: int, sample_clocks: bool = False):
        for _ in range(warmup):
            one_pass(fn_for, [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)])
        torch.cuda.synchronize()
        events = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)] for _ in range(steps)]
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        sampler = ClockSampler(local_rank) if sample_clocks else None
        if sampler:
            sampler.__enter__()
            time.sleep(0.5)  # nvidia-smi needs a moment before its first sample
        wall0 = time.perf_counter()
        epoch0 = time.time()
        for s in range(steps):
            one_pass(fn_for, events[s])
        torch.cuda.synchronize()
        wall = time.perf_counter() - wall0
        epoch1 = time.time()
        if sampler:
            sampler.__exit__(None, None, None)
        if world > 1:
            dist.barrier()
        per_shape = [[events[s][i][0].elapsed_time(events[s][i][1]) for s in range(steps)] for i in range(n)]
        return per_shape, wall, (sampler.summary(epoch0, epoch1) if sampler else None)

    # ---- 1b. confirmation (bank 1): the probes ran one candidate in a loop; the best ones are
    # re-timed side by side, each after an L2 flush, in passes over all shapes (a different
    # shape before every group), so clock drift over the passes hits every finalist alike ------
    confirmed = 0
    if args.confirm > 1 and not (args.force or args.choices):
        finalists = {w.key: _finalists(tuning.probes[w.key], args.confirm, args.confirm_within) for w in workloads}
        samples = {w.key: [[] for _ in finalists[w.key]] for w in workloads}
        failed: set[tuple[str, int]] = set()  # a finalist that raises drops out (the probe passed)
        if world > 1:
            dist.barrier()
        for rnd in range(6):  # the first pass warms up
            events = []
            for w in workloads:
                a, b = tune_operands[w.key]
                count = len(finalists[w.key])
                for j in range(count):
                    f = (j + rnd) % count  # rotate the order from pass to pass
                    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    flush.zero_()
                    start.record()
                    try:
                        launch(a, b, finalists[w.key][f])
                    except (ValueError, RuntimeError):
                        failed.add((w.key, f))
                    end.record()
                    events.append((w.key, f, start, end))
            torch.cuda.synchronize()
            if rnd > 0:
                for key, f, start, end in events:
                    samples[key][f].append(start.elapsed_time(end))
        if world > 1:
            dist.barrier()
        for w in workloads:
            medians = [
                math.inf if (w.key, f) in failed else statistics.median(t) for f, t in enumerate(samples[w.key])
            ]
            if min(medians) == math.inf:
                continue  # keep the bandit's recommendation
            best = finalists[w.key][medians.index(min(medians))]
            confirmed += best.key != chosen[w.key].key
            chosen[w.key] = best
    tuning_s = time.perf_counter() - t0
    del tune_operands
    torch.cuda.empty_cache()

    ours_times, ours_wall, clocks = timed(ours_fn, args.steps, args.warmup, sample_clocks=True)
    cublas_times, _, _ = timed(cublas_fn, args.steps, args.warmup) if not args.skip_cublas else (ours_times, 0.0, None)
    ours_ms = [statistics.median(t) for t in ours_times]
    cublas_ms = [statistics.median(t) for t in cublas_times]
    total_flops = sum(w.flops for w in workloads)
    pass_ms = sum(ours_ms)
    ratios = [o / c for o, c in zip(ours_ms, cublas_ms, strict=True)]
    geomean = math.exp(sum(math.log(r) for r in ratios) / len(ratios))

    # ---- roofline of the dominant kernel family -------------------------------------------------
    peaks, peak_source = _peaks()
    fam_time: dict[str, float] = {}
    fam_flops: dict[str, float] = {}
    fam_bytes: dict[str, float] = {}
    fam_launches: dict[str, int] = {}
    for w, ms in zip(workloads, ours_ms, strict=True):
        fam = _kernel_family(chosen[w.key])
        fam_time[fam] = fam_time.get(fam, 0.0) + ms
        fam_flops[fam] = fam_flops.get(fam, 0.0) + w.flops
        fam_bytes[fam] = fam_bytes.get(fam, 0.0) + w.ideal_bytes
        fam_launches[fam] = fam_launches.get(fam, 0) + 1
    dominant = max(fam_time, key=fam_time.get)

    floor_us = _after_flush_floor_us(flush)

    def family_roofline(fam: str) -> dict[str, object]:
        seconds = fam_time[fam] / 1e3
        hbm_bound = fam in ("split_k", "stream")
        units = fam_bytes[fam] / 1e9 if hbm_bound else fam_flops[fam] / 1e12
        achieved = units / seconds
        peak = peaks["hbm_gbs"] if hbm_bound else peaks["bf16_tflops"]
        entry = {
            "bound": "hbm" if hbm_bound else "tensor",
            "achieved": round(achieved, 2),
            "peak": peak,
            "unit": "GB/s" if hbm_bound else "TFLOP/s",
            "frac": round(achieved / peak, 4),
            "peak_source": f"{peak_source} (burst)",
            "launches_per_pass": fam_launches[fam],
            "share_of_pass": round(fam_time[fam] / pass_ms, 4),
        }
        above = seconds - fam_launches[fam] * floor_us / 1e6
        if hbm_bound and above > 0:
            # Diagnostic: the same bytes over the time above the floor every launch pays after the
            # L2-flush write (the event time of a trivial launch after the same flush).
            entry["frac_above_after_flush_floor"] = round(units / above / peak, 4)
        return entry

    roofline = family_roofline(dominant)
    roofline["kernel"] = {
        "tile": "tile_gemm_kernel",
        "persistent": "tile_gemm_kernel (persistent grid)",
        "split_k": "stream_gemm_kernel + splitk_reduce_kernel",
        "stream": "stream_cluster_kernel (in-cluster split-K)",
        "pair": "pair_gemm_kernel (cta_group::2)",
        "pair_wide": "pair_gemm_kernel<512, 64> (cta_group::2, 256 x 512 tiles)",
        "pair_deep_k": "pair_gemm_kernel<256, 128> (cta_group::2, 256 x 256 tiles, 128-deep K blocks)",
    }[dominant]
    roofline.update(_traffic_from_profiles(dominant))

    # per-shape roofline fraction (slower of tensor and HBM bound)
    shape_frac = []
    for w, ms in zip(workloads, ours_ms, strict=True):
        t_roof = max(w.flops / (peaks["bf16_tflops"] * 1e12), w.ideal_bytes / (peaks["hbm_gbs"] * 1e9))
        shape_frac.append(t_roof / (ms / 1e3))

    # ---- 2b. parity of the scored outputs: every chosen candidate on its bank-2 tensors ---------
    parity = _grid_parity(workloads, operands, chosen)

    # ---- 3. end to end through the public API with host buffers ------------------------------
    if args.e2e_steps > 0:
        e2e_ms, h2d_bytes, d2h_bytes = _e2e_pass(workloads, operands, chosen, device, args.e2e_steps)
    else:
        e2e_ms, h2d_bytes, d2h_bytes = list(ours_ms), 0, 0

    launches = sum(_launch_count(chosen[w.key], w, sm_count) for w in workloads) * args.steps

    value = total_flops / (pass_ms / 1e3) / 1e12
    e2e_value = total_flops / (sum(e2e_ms) / 1e3) / 1e12
    if world > 1:
        t = torch.tensor([pass_ms, sum(e2e_ms)], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        value = world * total_flops / (t[0].item() / 1e3) / 1e12
        e2e_value = world * total_flops / (t[1].item() / 1e3) / 1e12

    result: dict[str, object] = {
        "metric": _metric(args, len(workloads)),
        "value": round(value, 3),
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(pass_ms, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f16 (fp32 accumulate)",
        "data": "synthetic: seeded N(0,1)/sqrt(K) FP16 operands",
        "config": _config(args, workloads),
        "confirm_changed_shapes": confirmed,
        "pre_timing_gate": f"{len(gate)} candidate checks on {len(validation_workloads(workloads))} sampled shapes, all correct",
        "parity": parity,
        "geomean_latency_vs_cublas": round(geomean, 4),
        "cublas_tflops": round(total_flops / (sum(cublas_ms) / 1e3) / 1e12, 3),
        "shapes_faster_than_cublas": sum(r < 1.0 for r in ratios),
        "geomean_roofline_frac": round(math.exp(sum(math.log(f) for f in shape_frac) / len(shape_frac)), 4),
        "roofline": roofline,
        "roofline_by_family": {f: family_roofline(f) for f in fam_time},
        "e2e": {
            "value": round(e2e_value, 3),
            "unit": "TFLOP/s",
            "h2d_bytes_per_step": h2d_bytes,
            "d2h_bytes_per_step": d2h_bytes,
            "note": (
                "one pass: every distinct input tensor of the pass (8 B, 48 A) copied H2D once from pinned memory "
                "(copy-in stream), each GEMM launched when its A and B have landed, each C copied D2H (copy-out "
                "stream); timed from the first copy to the last D2H"
            ),
        },
        "gpu_launches": launches,
        "clocks": clocks,
        "after_flush_floor_us": round(floor_us, 2),
        "wall_s_timed_region": round(ours_wall, 3),
        "tuning_s": round(tuning_s, 1),
        "status_bits": _native.status(local_rank),
    }
    if args.detail and rank == 0:
        detail = Path(args.detail)
        detail.parent.mkdir(parents=True, exist_ok=True)
        detail.write_text(
            json.dumps(
                {
                    "shapes": [
                        {
                            "workload": w.key,
                            "m": w.m, "n": w.n, "k": w.k,
                            "choice": chosen[w.key].key,
                            "ours_ms": o,
                            "cublas_ms": c,
                            "ratio": o / c,
                            "roofline_frac": f,
                            "tflops": w.flops / (o / 1e3) / 1e12,
                        }
                        for w, o, c, f in zip(workloads, ours_ms, cublas_ms, shape_frac, strict=True)
                    ],
                    "tuning": tuning.to_dict(),
                },
                indent=1,
            )
        )
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        baseline = CpuBaseline(workloads)
        baseline.run(args.cpu_budget_s)
        result["cpu_baseline"] = baseline.summary()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return result if rank == 0 else None


def _after_flush_floor_us(flush, reps: int = 25) -> float:
    """Median event time of a trivial launch of this library (a one-chunk column assembly)
    after the same 256 MiB L2-flush write that precedes every scored launch: the share of any
    launch's time that the protocol, not the kernel, sets."""
    import torch

    from heliostune_b200.column_parallel import assemble_columns

    src = torch.zeros((1, 1, 8), dtype=torch.float16, device=flush.device)
    dst = torch.empty((1, 8), dtype=torch.float16, device=flush.device)
    times = []
    for _ in range(reps):
        flush.zero_()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        assemble_columns(src, dst)
        end.record()
        torch.cuda.synchronize()
        times.append(start.elapsed_time(end) * 1e3)
    return statistics.median(times[5:])


def _grid_parity(workloads, operands, chosen) -> dict[str, object]:
    """Check the scored (bank-2) output of every shape's chosen candidate against the FP32 product
    (elementwise 1e-2 + 1e-2|C|, normwise 1e-2) beside cuBLAS ``torch.matmul``'s normwise error on
    the same inputs. Raises if any shape fails the tolerance."""
    import torch

    from heliostune_b200.action_expansion import fp32_reference, launch

    worst, worst_cublas, worse, failures = 0.0, 0.0, [], []
    for w in workloads:
        a, b = operands[w.key]
        expected = fp32_reference(a, b)
        scale = max(expected.abs().max().item(), 1e-30)
        out = launch(a, b, chosen[w.key]).float()
        err = (out - expected).abs().max().item() / scale
        ok = bool(torch.all((out - expected).abs() <= 1e-2 + 1e-2 * expected.abs()).item()) and err <= 1e-2
        del out
        cublas = (torch.matmul(a, b).float() - expected).abs().max().item() / scale
        del expected
        worst, worst_cublas = max(worst, err), max(worst_cublas, cublas)
        if err > cublas:
            worse.append(f"{w.key}: {err:.3g} vs {cublas:.3g}")
        if not ok:
            failures.append(f"{chosen[w.key].key} on {w.key}: normwise {err:.3g}")
    torch.cuda.empty_cache()
    if failures:
        raise AssertionError("parity failure on the scored tensors: " + "; ".join(failures))
    return {
        "status": "ok",
        "checked": f"bank-2 output of the chosen candidate of all {len(workloads)} shapes vs the FP32 product",
        "max_normwise": float(f"{worst:.4g}"),
        "max_normwise_cublas": float(f"{worst_cublas:.4g}"),
        "shapes_with_error_above_cublas": len(worse),
        "above_cublas": worse[:8],
    }


def run_colpar(args: argparse.Namespace) -> dict[str, object] | None:
    """Config 5: C[M, N] = A[M, K] B[K, N] with B split N-wise over the ranks. Each rank's slice
    is computed by the CTA-pair GEMM; with several ranks the slices reach every rank either from
    the GEMM epilogue over NVLink (fused, the default) or by an NCCL all-gather and a column
    assembly. After the timed steps each rank checks sampled rows of its full C, spanning every
    rank's column slice, against the FP32 product of the same seeded operands."""
    import torch
    import torch.distributed as dist

    from heliostune_b200 import _native
    from heliostune_b200.action_expansion import launch
    from heliostune_b200.column_parallel import ColumnShard, column_parallel_candidate, column_parallel_matmul

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)
    _native.library()
    workloads = _workloads("colpar", args.shapes)
    (w,) = workloads
    shard = ColumnShard(w.n, world, rank)
    a = _colpar_a(w, device)
    b_shard = _colpar_b_slice(w, shard.cols, rank, device)
    candidate = column_parallel_candidate(w.m, shard.cols)

    if args.exchange == "fused" and world > 1:
        from heliostune_b200.column_parallel import FusedColumnParallel

        fused = FusedColumnParallel(w.m, w.n, device=device, peer_writes=args.peer_writes)

        def step_on(x, y, events):
            return fused(x, y, phase_events=events)
    else:
        fused = None

        def step_on(x, y, events):
            return column_parallel_matmul(x, y, phase_events=events)

    def step(events):
        return step_on(a, b_shard, events)

    for _ in range(args.warmup):
        step(None)
    torch.cuda.synchronize()
    events = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    sampler = ClockSampler(local_rank)
    sampler.__enter__()
    time.sleep(0.5)
    epoch0 = time.time()
    out = None
    for s_ in range(args.steps):
        out = step(events[s_])
    torch.cuda.synchronize()
    epoch1 = time.time()
    sampler.__exit__(None, None, None)
    if world > 1:
        dist.barrier()
    phase1_ms = statistics.median(e[0].elapsed_time(e[1]) for e in events)
    phase2_ms = statistics.median(e[1].elapsed_time(e[2]) for e in events)
    step_ms = statistics.median(e[0].elapsed_time(e[2]) for e in events)

    # The slice GEMM alone (no exchange), for the GEMM-phase roofline.
    gemm_events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(4)]
    for start, end in gemm_events:
        start.record()
        launch(a, b_shard, candidate)
        end.record()
    torch.cuda.synchronize()
    gemm_ms = statistics.median(start.elapsed_time(end) for start, end in gemm_events[1:])

    parity = _colpar_parity(w, a, out, world, shard.cols, device)
    del out
    e2e_ms = _colpar_e2e(a, b_shard, shard, step_on, device, args.e2e_steps) if args.e2e_steps > 0 else step_ms
    times = torch.tensor([step_ms, gemm_ms, phase1_ms, phase2_ms, e2e_ms], device=device, dtype=torch.float64)
    checks = torch.tensor(
        [parity["normwise"], parity["normwise_cublas"], 0.0 if parity["ok"] else 1.0], device=device, dtype=torch.float64
    )
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
        dist.all_reduce(checks, op=dist.ReduceOp.MAX)
    step_ms, gemm_ms, phase1_ms, phase2_ms, e2e_ms = (float(t) for t in times.tolist())
    normwise, normwise_cublas, failed = (float(t) for t in checks.tolist())
    peaks, source = _peaks()
    flops = 2.0 * w.m * w.n * w.k
    gemm_tflops = flops / world / (gemm_ms / 1e3) / 1e12
    gather_bytes = 2.0 * w.m * w.n * (world - 1) / world
    # Roofline of the whole step: the slower of the per-GPU GEMM at the sustained tensor peak and
    # the bytes every GPU receives at the measured 770 GB/s peer bandwidth.
    t_roof = max(flops / world / (peaks["bf16_tflops_sustained"] * 1e12), gather_bytes / 770e9)
    limiter = "tensor cores (slice GEMM)" if flops / world / (peaks["bf16_tflops_sustained"] * 1e12) >= gather_bytes / 770e9 else "NVLink receive bytes per GPU"
    result: dict[str, object] = {
        "metric": _metric(args, 1),
        "value": round(flops / (step_ms / 1e3) / 1e12, 3),
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(step_ms, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f16 (fp32 accumulate)",
        "data": "synthetic: seeded N(0,1)/sqrt(K) FP16 operands",
        "config": _config(args, workloads),
        "note": (
            "under torch.distributed.run bench.py runs this column-parallel configuration at every rank "
            "count, one rank included; plain `python bench.py` runs the 96-shape grid"
        ),
        "parity": {
            "status": "fail" if failed else "ok",
            "checked": f"{parity['rows']} rows of the full C on every rank (all {world} column slices) vs the FP32 product",
            "max_normwise": float(f"{normwise:.4g}"),
            "max_normwise_cublas": float(f"{normwise_cublas:.4g}"),
        },
        "gemm_ms": round(gemm_ms, 4),
        "roofline": {
            "bound": "tensor",
            "achieved": round(gemm_tflops, 2),
            "peak": peaks["bf16_tflops_sustained"],
            "unit": "TFLOP/s",
            "frac": round(gemm_tflops / peaks["bf16_tflops_sustained"], 4),
            "peak_source": f"{source} (sustained)",
            "kernel": f"pair_gemm_kernel<{candidate.config.block_n},{candidate.config.block_k}> (slice GEMM alone, per GPU)",
            "traffic": None,
        },
        "step_roofline_frac": round(t_roof / (step_ms / 1e3), 4),
        "step_roofline_limiter": limiter,
        "exchange_bytes_per_gpu": int(gather_bytes),
        "e2e": {
            "value": round(flops / (e2e_ms / 1e3) / 1e12, 3),
            "unit": "TFLOP/s",
            "h2d_bytes_per_step": world * 2 * (w.m * w.k + w.k * shard.cols),
            "d2h_bytes_per_step": 2 * w.m * w.n,
            "note": (
                "one step with host buffers: every rank copies A and its B slice in from pinned memory, runs "
                "the step, and copies its own column slice of C out (the ranks return all of C once); bytes are "
                "the whole job's; time from the first copy to the last, max over ranks"
            ),
        },
        # Per step: barrier, fused GEMM, barrier; or the GEMM and the assembly; or the GEMM alone.
        "gpu_launches": (3 if fused is not None else 1 if world == 1 else 2) * args.steps,
        "clocks": sampler.summary(epoch0, epoch1),
        "status_bits": _native.status(local_rank),
    }
    if world > 1:
        if fused is not None:
            result["phases_ms"] = {"barrier+fused_gemm": round(phase1_ms, 4), "trailing_barrier": round(phase2_ms, 4)}
            result["exchange_gbs"] = round(gather_bytes / (step_ms / 1e3) / 1e9, 1)
            result["exchange_gbs_note"] = "bytes each GPU receives / step time (the exchange overlaps the GEMM)"
        else:
            result["phases_ms"] = {"gemm": round(phase1_ms, 4), "all_gather+assembly": round(phase2_ms, 4)}
            result["exchange_gbs"] = round(gather_bytes / (phase2_ms / 1e3) / 1e9, 1)
    if fused is not None:
        fused.close()
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        baseline = CpuBaseline(workloads)
        baseline.run(args.cpu_budget_s)
        result["cpu_baseline"] = baseline.summary()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if failed:
        print(json.dumps(result), flush=True) if rank == 0 else None
        raise SystemExit("column-parallel parity failure")
    return result if rank == 0 else None


def _colpar_e2e(a, b_shard, shard, step_on, device, steps: int) -> float:
    """Milliseconds of one config-5 step with host buffers on this rank (the slowest rank's is
    the job's): H2D of A and of this rank's B slice from pinned memory into device buffers
    allocated beforehand, the step (GEMM and exchange), D2H of this rank's column slice of C into
    pinned memory; the first of ``steps + 1`` passes warms up."""
    import torch

    a_host, b_host = a.cpu().pin_memory(), b_shard.cpu().pin_memory()
    a_dev, b_dev = torch.empty_like(a), torch.empty_like(b_shard)
    c_host = torch.empty((a.shape[0], shard.cols), dtype=torch.float16).pin_memory()
    total = 0.0
    for rep in range(steps + 1):
        torch.cuda.synchronize(device)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        a_dev.copy_(a_host, non_blocking=True)
        b_dev.copy_(b_host, non_blocking=True)
        c = step_on(a_dev, b_dev, None)
        c_host.copy_(c[:, shard.start : shard.stop], non_blocking=True)
        end.record()
        torch.cuda.synchronize(device)
        if rep > 0:
            total += start.elapsed_time(end) / steps
    return total


def _colpar_a(w, device):
    import torch

    g = torch.Generator(device=device).manual_seed(5)
    return (torch.randn((w.m, w.k), generator=g, device=device) / math.sqrt(w.k)).to(torch.float16)


def _colpar_b_slice(w, cols: int, q: int, device):
    """Column slice ``q`` of B (``cols`` columns), from its own seed, so that any rank can
    regenerate every slice."""
    import torch

    g = torch.Generator(device=device).manual_seed(1000 + q)
    return (torch.randn((w.k, cols), generator=g, device=device) / math.sqrt(w.k)).to(torch.float16)


def _colpar_parity(w, a, out, world: int, cols: int, device) -> dict[str, object]:
    """Sampled rows of the full C against the FP32 product: two rows of every 256-row tile band
    (at offsets that move from band to band), all N columns, so every rank's slice and every
    tile row is covered. Elementwise 1e-2 + 1e-2|C| and normwise 1e-2, plus cuBLAS's normwise
    error on the same rows."""
    import torch

    from heliostune_b200.action_expansion import fp32_reference

    b_full = torch.cat([_colpar_b_slice(w, cols, q, device) for q in range(world)], dim=1)
    bands = -(-w.m // 256)
    rows = sorted({min(w.m - 1, band * 256 + off) for band in range(bands) for off in ((band * 37) % 128, 128 + (band * 101) % 128)})
    index = torch.tensor(rows, device=device)
    a_rows = a.index_select(0, index)
    expected = fp32_reference(a_rows, b_full)
    scale = max(expected.abs().max().item(), 1e-30)
    got = out.index_select(0, index).float()
    diff = (got - expected).abs()
    normwise = diff.max().item() / scale
    ok = bool(torch.all(diff <= 1e-2 + 1e-2 * expected.abs()).item()) and normwise <= 1e-2 and bool(torch.isfinite(got).all().item())
    cublas = (torch.matmul(a_rows, b_full).float() - expected).abs().max().item() / scale
    del b_full, expected, got, diff
    torch.cuda.empty_cache()
    return {"ok": ok, "normwise": normwise, "normwise_cublas": cublas, "rows": len(rows)}


def run_rmsnorm(args: argparse.Namespace) -> dict[str, object] | None:
    """Config 4: standalone RMSNorm over M in {1, 4096, 65536} x hidden in {4096, 8192}, and the
    RMSNorm feeding the (4096 -> 6144) QKV GEMM at M in {1, 128, 4096}. FP16, eps 1e-6,
    x ~ N(0, 1), gamma ~ 1 + 0.1 N(0, 1). Compared with the same math in eager torch. Beside
    them, the reference's own fusion suites: the residual RMSNorm (BF16, 128 x 4096) and the
    gated-MLP projection with its epilogue (BF16, 11008 x 4096 weights)."""
    import torch

    from heliostune_b200 import _native
    from heliostune_b200.action_configs import b200_candidates_for
    from heliostune_b200.configs import Workload
    from heliostune_b200.fusion import rmsnorm, rmsnorm_matmul
    from heliostune_b200.timing import do_bench

    torch.cuda.set_device(0)
    device = torch.device("cuda", 0)
    _native.library()
    peaks, source = _peaks()
    eps = 1e-6

    def inputs(rows: int, hidden: int, seed: int):
        g = torch.Generator(device=device).manual_seed(seed)
        x = torch.randn((rows, hidden), generator=g, device=device).to(torch.float16)
        gamma = (1.0 + 0.1 * torch.randn((hidden,), generator=g, device=device)).to(torch.float16)
        return x, gamma

    def eager(x, gamma):
        xf = x.float()
        return (xf * torch.rsqrt((xf * xf).mean(dim=-1, keepdim=True) + eps) * gamma.float()).to(torch.float16)

    cases = []
    fracs = []
    for rows in (1, 4096, 65536):
        for hidden in (4096, 8192):
            x, gamma = inputs(rows, hidden, rows + hidden)
            ours = do_bench(lambda: rmsnorm(x, gamma, eps), quantiles=(0.5,))[0]
            ref = do_bench(lambda: eager(x, gamma), quantiles=(0.5,))[0]
            nbytes = 4 * rows * hidden + 2 * hidden
            gbs = nbytes / (ours / 1e3) / 1e9
            fracs.append(gbs / peaks["hbm_gbs"])
            cases.append({"op": "rmsnorm", "rows": rows, "hidden": hidden, "ours_us": round(ours * 1e3, 2),
                          "eager_us": round(ref * 1e3, 2), "gbs": round(gbs, 1),
                          "hbm_frac": round(gbs / peaks["hbm_gbs"], 4)})
    w_gen = torch.Generator(device=device).manual_seed(11)
    w = (torch.randn((4096, 6144), generator=w_gen, device=device) / 64).to(torch.float16)
    for rows in (1, 128, 4096):
        x, gamma = inputs(rows, 4096, rows)
        workload = Workload(m=rows, n=6144, k=4096, model="llama-3-8b", projection="attention-qkv", regime=f"m{rows}")
        best = None
        for cand in b200_candidates_for(workload):
            try:
                t = do_bench(lambda: rmsnorm_matmul(x, gamma, w, cand, eps), warmup_ms=2, rep_ms=10, quantiles=(0.5,))[0]
            except Exception:  # noqa: BLE001 -- a candidate that fails is skipped
                continue
            if best is None or t < best[0]:
                best = (t, cand)
        ours = do_bench(lambda: rmsnorm_matmul(x, gamma, w, best[1], eps), quantiles=(0.5,))[0]
        ref = do_bench(lambda: torch.matmul(eager(x, gamma), w), quantiles=(0.5,))[0]
        flops = 2 * rows * 6144 * 4096
        nbytes = 2 * (rows * 4096 + 4096 * 6144 + rows * 6144) + 2 * 4096
        t_roof = max(flops / (peaks["bf16_tflops"] * 1e12), nbytes / (peaks["hbm_gbs"] * 1e9))
        fracs.append(t_roof / (ours / 1e3))
        cases.append({"op": "rmsnorm->qkv gemm", "rows": rows, "hidden": 4096, "n": 6144,
                      "gemm": best[1].key, "ours_us": round(ours * 1e3, 2), "eager_us": round(ref * 1e3, 2),
                      "roofline_frac": round(t_roof / (ours / 1e3), 4)})
    geo = math.exp(sum(math.log(f) for f in fracs) / len(fracs))
    speedups = [c["eager_us"] / c["ours_us"] for c in cases]
    residual_cases = _residual_rmsnorm_cases(device, peaks)
    gated_cases = _gated_mlp_cases(device, peaks)
    return {
        "metric": "RMSNorm fp16 (eps 1e-6) standalone and feeding the QKV GEMM: geomean fraction of roofline",
        "value": round(geo, 4),
        "unit": "fraction of roofline",
        "n_gpus": 1,
        "steps": 0,
        "warmup": 0,
        "ms_per_step": None,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f16 in/out, fp32 row sums",
        "data": "synthetic: x ~ N(0,1), gamma ~ 1 + 0.1 N(0,1), seeded",
        "config": {"workload": "config 4: rmsnorm M x H in {1,4096,65536} x {4096,8192}; rmsnorm->qkv at M in {1,128,4096}",
                   "l2": "256 MiB write before every launch", "peak_source": source},
        "geomean_speedup_vs_eager_torch": round(math.exp(sum(map(math.log, speedups)) / len(speedups)), 3),
        "cases": cases,
        "residual_rmsnorm": residual_cases,
        "gated_mlp": gated_cases,
    }


def _gated_mlp_cases(device, peaks) -> list[dict[str, object]]:
    """The gated-MLP epilogue suite's case (BF16 x [8, 4096], Wg and Wu [11008, 4096]) through
    ``fusion.gated_mlp`` (one launch), beside the reference's formula in eager torch (two FP32
    matmuls, silu, product), each after an L2 flush. HBM-bound: the two weights are read once."""
    import torch

    from heliostune_b200.fusion import gated_mlp
    from heliostune_b200.timing import do_bench

    out = []
    for m in (1, 8, 32, 64):
        g = torch.Generator(device=device).manual_seed(17)
        x = torch.randn((m, 4096), generator=g, device=device).to(torch.bfloat16)
        gate = (torch.randn((11008, 4096), generator=g, device=device) / 64).to(torch.bfloat16)
        up = (torch.randn((11008, 4096), generator=g, device=device) / 64).to(torch.bfloat16)

        def eager():
            return (torch.nn.functional.silu(torch.mm(x.float(), gate.float().T)) * torch.mm(x.float(), up.float().T)).to(torch.bfloat16)

        def eager_bf16():
            return (torch.nn.functional.silu(torch.mm(x, gate.T)) * torch.mm(x, up.T)).to(torch.bfloat16)

        ours = do_bench(lambda: gated_mlp(x, gate, up), quantiles=(0.5,))[0]
        nbytes = 2 * (2 * 11008 * 4096 + m * 4096 + m * 11008)
        out.append({
            "batch": m, "hidden": 4096, "intermediate": 11008,
            "ours_us": round(ours * 1e3, 2),
            "eager_fp32_us": round(do_bench(eager, quantiles=(0.5,))[0] * 1e3, 2),
            "eager_bf16_cublas_us": round(do_bench(eager_bf16, quantiles=(0.5,))[0] * 1e3, 2),
            "gbs": round(nbytes / (ours / 1e3) / 1e9, 1),
            "hbm_frac": round(nbytes / (ours / 1e3) / 1e9 / peaks["hbm_gbs"], 4),
        })
        del x, gate, up
    return out


def _residual_rmsnorm_cases(device, peaks) -> list[dict[str, object]]:
    """The reference's own residual RMSNorm (BF16, 128 x 4096, z = x + r, eps 1e-5) through its
    four entry points. ``call_us``: per-call latency with the reference's protocol (CUDA events
    around each call from the host, L2 flushed before it), comparable with its published H100
    medians; ``device_us``: kernel time alone, from a CUDA graph of 20 (flush, call) pairs minus
    a graph of the 20 flushes."""
    import torch

    from heliostune_b200.fusion import RESIDUAL_RMSNORM_ENTRYPOINTS, load_residual_rmsnorm
    from heliostune_b200.timing import do_bench, flush_buffer

    g = torch.Generator(device=device).manual_seed(17)
    x = torch.randn((128, 4096), generator=g, device=device).to(torch.bfloat16)
    r = torch.randn((128, 4096), generator=g, device=device).to(torch.bfloat16)
    gamma = (1.0 + 0.02 * torch.randn((4096,), generator=g, device=device)).to(torch.bfloat16)
    flush = flush_buffer(device)

    def eager():
        z = x.float() + r.float()
        ms = torch.mean(z * z, dim=-1, keepdim=True, dtype=torch.float32)
        return (z * torch.rsqrt(ms + 1e-5) * gamma.float()).to(torch.bfloat16)

    def graph_us(fn) -> float:
        reps = 20
        side = torch.cuda.Stream(device)
        side.wait_stream(torch.cuda.current_stream(device))
        with torch.cuda.stream(side):  # warm the allocator before capture
            fn()
        torch.cuda.current_stream(device).wait_stream(side)
        torch.cuda.synchronize(device)
        both, flushes = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
        with torch.cuda.graph(both):
            for _ in range(reps):
                flush.zero_()
                fn()
        with torch.cuda.graph(flushes):
            for _ in range(reps):
                flush.zero_()
        times = []
        for graph in (both, flushes):
            samples = []
            for _ in range(7):
                start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                start.record()
                graph.replay()
                end.record()
                torch.cuda.synchronize(device)
                samples.append(start.elapsed_time(end))
            times.append(statistics.median(samples[2:]))
        del both, flushes
        return (times[0] - times[1]) / reps * 1e3

    nbytes = 3 * 128 * 4096 * 2 + 4096 * 2
    out = []
    for name in RESIDUAL_RMSNORM_ENTRYPOINTS:
        fn = load_residual_rmsnorm(name)
        call_us = do_bench(lambda: fn(x, r, gamma), quantiles=(0.5,))[0] * 1e3
        device_us = graph_us(lambda: fn(x, r, gamma))
        out.append({
            "entrypoint": name,
            "call_us": round(call_us, 2),
            "device_us": round(device_us, 2),
            "device_gbs": round(nbytes / (device_us / 1e6) / 1e9, 1),
            "device_hbm_frac": round(nbytes / (device_us / 1e6) / 1e9 / peaks["hbm_gbs"], 4),
        })
    out.append({
        "entrypoint": "eager torch (the reference's formula)",
        "call_us": round(do_bench(eager, quantiles=(0.5,))[0] * 1e3, 2),
        "device_us": round(graph_us(eager), 2),
    })
    return out


def _traffic_from_profiles(family: str) -> dict[str, object]:
    """DRAM bytes of one ncu-captured launch of the family's kernel (profiles/traffic.json),
    beside the algorithmic bytes of that same launch."""
    path = ROOT / "profiles" / "traffic.json"
    entry = json.loads(path.read_text()).get(family) if path.exists() else None
    if entry is None:
        return {"traffic": None}
    m, n, k = (int(part.split("=")[1]) for part in entry["workload"].split())
    return {
        "traffic": entry["bytes_per_launch"],
        "traffic_launch": f"{entry['kernel']} at {entry['workload']}",
        "traffic_algorithmic_bytes": 2 * (m * k + k * n + m * n),
    }


def _finalists(probes, count: int, within: float):
    """Up to ``count`` probed candidates, fastest first, whose latency is within ``within`` x the
    fastest probe's (the fastest alone if nothing else qualifies)."""
    valid = sorted((p for p in probes if p.latency_ms is not None), key=lambda p: p.latency_ms)
    if not valid:
        raise RuntimeError("no valid probe")
    best = valid[0].latency_ms
    return [p.candidate for p in valid if p.latency_ms <= best * within][:count]


def _e2e_pass(workloads, operands, chosen, device, steps: int):
    """Milliseconds of one pass over the workloads through the public API with host buffers.

    A step's inputs are the distinct operand tensors of its shapes (the 96 grid shapes share 8
    weight matrices B and 48 matrices A). Every step copies each of them host to device once,
    from pinned memory, on a copy-in stream, into device buffers allocated before the timing; a
    shape's GEMM runs on the current stream as soon as the copies of its A and B have landed
    (per-tensor events), shapes ordered so that each B is copied right before the shapes using
    it, and each C goes back to pinned memory on a copy-out stream while later inputs arrive.
    Timed from the first copy to the last device-to-host copy; returns ``[pass_ms]``, h2d, d2h.
    """
    import torch

    from heliostune_b200.action_expansion import launch

    order = sorted(workloads, key=lambda w: (w.k, w.n, w.m))
    tensors: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}  # id of the operand -> (host, device copy)
    needs = []
    for w in order:
        a, b = operands[w.key]
        for t in (a, b):
            if id(t) not in tensors:
                tensors[id(t)] = (t.cpu().pin_memory(), torch.empty_like(t))
        needs.append((w, id(a), id(b), torch.empty((w.m, w.n), dtype=torch.float16).pin_memory()))
    main = torch.cuda.current_stream(device)
    copy_in = torch.cuda.Stream(device)
    copy_out = torch.cuda.Stream(device)
    total = 0.0
    for step in range(steps + 1):  # the first pass warms up
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(main)
        copy_in.wait_event(start)
        landed: dict[int, torch.cuda.Event] = {}
        for w, key_a, key_b, c_host in needs:
            for key in (key_a, key_b):
                if key not in landed:
                    host, dev = tensors[key]
                    with torch.cuda.stream(copy_in):
                        dev.copy_(host, non_blocking=True)
                    landed[key] = torch.cuda.Event()
                    landed[key].record(copy_in)
                main.wait_event(landed[key])
            c = launch(tensors[key_a][1], tensors[key_b][1], chosen[w.key])
            copy_out.wait_stream(main)
            with torch.cuda.stream(copy_out):
                c_host.copy_(c, non_blocking=True)
            c.record_stream(copy_out)
        main.wait_stream(copy_out)
        end.record(main)
        torch.cuda.synchronize()
        if step > 0:
            total += start.elapsed_time(end) / steps
    h2d = sum(host.numel() * host.element_size() for host, _ in tensors.values())
    d2h = sum(2 * w.m * w.n for w in workloads)
    return [total], h2d, d2h


# ----------------------------------------------------------------------------------------------
# CPU baseline / reference arm
# ----------------------------------------------------------------------------------------------


def _cpu_model() -> str:
    try:
        out = subprocess.run(["lscpu"], capture_output=True, text=True, timeout=10).stdout
        for line in out.splitlines():
            if line.lower().startswith("model name:"):
                return line.split(":", 1)[1].strip()
    except (OSError, subprocess.SubprocessError):
        pass
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


class CpuBaseline:
    """FP16 ``torch.matmul`` of the workload's shapes on the host cores (through the oracle), with
    ``torch.set_num_threads(os.cpu_count())``.

    The work is cut into pieces: whole shapes, or blocks of ``rows`` rows of shapes taller than
    that (each block against the full B). ``run(budget_s)`` times pieces one after another,
    continuing where the previous call stopped and wrapping around, until ``budget_s`` seconds
    of products are spent; a piece's latency is the median of its samples. ``summary()`` gives
    FLOPs of the measured pieces / the sum of their median latencies: for a workload whose every
    piece was measured, its whole-workload rate on the CPU.
    """

    def __init__(self, workloads, rows: int = 2048, seed: int = 0) -> None:
        import torch

        torch.set_num_threads(os.cpu_count() or 1)
        self.workloads = tuple(workloads)
        self.pieces = [(w, r0, min(w.m, r0 + rows)) for w in self.workloads for r0 in range(0, w.m, rows)]
        self.samples: list[list[float]] = [[] for _ in self.pieces]
        self.cursor = 0
        self.seed = seed
        self._b: dict[tuple[int, int], object] = {}
        self._a: dict[tuple[int, int], object] = {}

    def _operands(self, w, rows: int):
        import torch

        if (w.k, w.n) not in self._b:
            g = torch.Generator().manual_seed(self.seed + 7919 * w.k + w.n)
            self._b[(w.k, w.n)] = (torch.randn((w.k, w.n), generator=g) / math.sqrt(w.k)).to(torch.float16)
        if (w.k, rows) not in self._a:
            g = torch.Generator().manual_seed(self.seed + 104729 * w.k + rows)
            self._a[(w.k, rows)] = (torch.randn((rows, w.k), generator=g) / math.sqrt(w.k)).to(torch.float16)
        return self._a[(w.k, rows)], self._b[(w.k, w.n)]

    def run(self, budget_s: float) -> None:
        from oracle import oracle

        spent = 0.0
        while True:
            w, r0, r1 = self.pieces[self.cursor]
            a, b = self._operands(w, r1 - r0)
            t0 = time.perf_counter()
            oracle.gemm_fp16_torch_cpu(a, b)
            dt = time.perf_counter() - t0
            self.samples[self.cursor].append(dt)
            spent += dt
            self.cursor = (self.cursor + 1) % len(self.pieces)
            if spent >= budget_s:
                return

    def summary(self) -> dict[str, object]:
        import torch

        measured = [(p, statistics.median(t)) for p, t in zip(self.pieces, self.samples, strict=True) if t]
        flops = sum(2.0 * (r1 - r0) * w.n * w.k for (w, r0, r1), _ in measured)
        seconds = sum(t for _, t in measured)
        complete = len(measured) == len(self.pieces)
        cover = (
            f"all {len(self.pieces)} pieces"
            if complete
            else f"{len(measured)} of {len(self.pieces)} pieces (the rest not reached within the budget)"
        )
        shapes = len(self.workloads)
        return {
            "value": round(flops / seconds / 1e12, 4),
            "unit": "TFLOP/s",
            "cores": torch.get_num_threads(),
            "os_cpu_count": os.cpu_count(),
            "cpu_model": _cpu_model(),
            "kind": "port",
            "sample": (
                f"FP16 torch.matmul on the host ({torch.get_num_threads()} threads) over the {shapes}-shape "
                f"workload cut into shapes and 2048-row blocks; {cover} timed, median per piece; "
                "value = their FLOPs / sum of their medians"
            ),
            "full_workload": complete,
        }


def run_reference(args: argparse.Namespace) -> dict[str, object] | None:
    """The reference's CPU path on the same configuration: rank 0 alone (others exit at once)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    workloads = _workloads(args.workload, args.shapes)
    baseline = CpuBaseline(workloads)
    for _ in range(args.warmup):
        baseline.run(args.cpu_step_s / 4)
    baseline.samples = [[] for _ in baseline.pieces]  # warm-up samples are not kept
    t0 = time.perf_counter()
    for _ in range(args.steps):
        baseline.run(args.cpu_step_s)
    wall = time.perf_counter() - t0
    summary = baseline.summary()
    value = summary["value"]
    return {
        "impl": "reference",
        "metric": _metric(args, len(workloads)),
        "value": value,
        "unit": "TFLOP/s",
        "n_gpus": int(os.environ.get("WORLD_SIZE", "1")),
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(wall / max(args.steps, 1) * 1e3, 1),
        "higher_is_better": True,
        "scaling": "strong" if args.workload == "colpar" else "weak",
        "vs_baseline": None,
        "dtype": "f16 in/out (CPU torch.matmul)",
        "data": "synthetic: seeded N(0,1)/sqrt(K) FP16 operands",
        "config": _config(args, workloads),
        "step_note": f"one step = {args.cpu_step_s:g} s of products over the workload's pieces, continuing round-robin",
        "cpu_baseline": summary,
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=20)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", choices=("ours", "reference"), default="ours")
    parser.add_argument(
        "--workload",
        choices=("grid", "sweep", "decode", "colpar", "rmsnorm"),
        default=None,
        help="default: colpar when started by torch.distributed.run, else grid",
    )
    parser.add_argument("--shapes", default=None, help="comma list of MxNxK overriding the workload")
    parser.add_argument("--budget", type=int, default=8, help="bandit probes per shape")
    parser.add_argument("--features", choices=("v2", "b200"), default="v2", help="the bandit's feature basis")
    parser.add_argument("--probe-ms", type=float, default=10.0)
    parser.add_argument(
        "--confirm", type=int, default=3, help="re-time the best N probed candidates per shape in scored-like passes (1 = off)"
    )
    parser.add_argument("--confirm-within", type=float, default=1.10, help="finalists: probe latency within this factor of the best")
    parser.add_argument("--seed", type=int, default=0)
    parser.add_argument("--e2e-steps", type=int, default=1)
    parser.add_argument("--cpu-budget-s", type=float, default=25.0, help="CPU baseline of our arm: seconds of products")
    parser.add_argument("--cpu-step-s", type=float, default=6.0, help="reference arm: seconds of products per step")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--detail", default=None, metavar="FILE", help="also write per-shape results and the tuning record to FILE")
    parser.add_argument("--choices", default=None, help="per-shape choices from an earlier --detail file")
    parser.add_argument("--skip-cublas", action="store_true", help="profiling runs: no cuBLAS passes")
    parser.add_argument("--force", default=None, help="profiling runs: one candidate key for every shape")
    parser.add_argument(
        "--exchange",
        choices=("fused", "nccl"),
        default="fused",
        help="colpar: all-gather fused into the GEMM epilogue, or NCCL all-gather + assembly",
    )
    parser.add_argument(
        "--peer-writes",
        choices=("stores", "bulk"),
        default=None,
        help=(
            "colpar fused exchange: epilogue 16-byte stores or TMA tensor stores into the peers' C "
            "(default: bulk at 2 GPUs, else stores)"
        ),
    )
    args = parser.parse_args()
    if args.workload is None:
        args.workload = "colpar" if _distributed_launch() and not args.shapes else "grid"
    if args.warmup < 3 and args.impl == "ours" and not args.shapes:
        print("note: fewer than 3 warm-up passes", file=sys.stderr)
    if args.impl == "reference":
        result = run_reference(args)
    elif args.workload == "colpar":
        result = run_colpar(args)
    elif args.workload == "rmsnorm":
        result = run_rmsnorm(args)
    else:
        result = run_ours(args)
    if result is not None:
        print(json.dumps(result), flush=True)


if __name__ == "__main__":
    main()
