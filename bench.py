"""Benchmark of the B200 FP16 matmul path on the 96-shape grid (and the other configurations).

Default workload ``grid`` (the configuration the headline metric is quoted on): 8 (K, N)
projection pairs of Llama-3-8B and Qwen2.5-7B x 12 values of M, FP16 operands N(0, 1)/sqrt(K)
from seeded generators. Flow, as the reference's protocol (bank 1 selects, bank 2 scores):

1. tuning (untimed): the Thompson-sampling bandit probes ``--budget`` candidates per shape
   with live timed launches (every probe's output is checked against an FP32 reference);
2. ``--warmup`` untimed passes, then ``--steps`` timed passes over the 96 shapes with each
   shape's recommended variant through the public API (``action_expansion.launch``: output and
   workspace allocated per call). Before every launch a 256 MiB write flushes L2; each launch is
   bracketed by CUDA events on the launching stream. The same passes with cuBLAS
   ``torch.matmul`` give the comparison;
3. an end-to-end pass: host->device copies of A and B from pinned memory, the launch, and the
   device->host copy of C, inside the events;
4. on rank 0 at N=1, the CPU baseline: the oracle's FP32 BLAS product on a bounded sample.

``value`` is the grid's aggregate TFLOP/s (total FLOPs of one pass / sum of per-shape median
latencies), ``geomean_latency_vs_cublas`` the headline ratio. Under torchrun every rank runs the
whole grid (replicas): value = sum over ranks' FLOPs / max over ranks' time.

``--impl reference`` times the reference's CPU path (the oracle port) on the host cores.
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


def _metric(args, count: int) -> str:
    """BASELINE's metric name for the grid; the same form naming the shape set otherwise."""
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
    from heliostune_b200.kernel import get_hardware_profile
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
        tuning = thompson_probe(workloads, b200_candidates_for, measure, hardware, budget=args.budget, policy_seed=args.seed)
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

    def family_roofline(fam: str) -> dict[str, object]:
        seconds = fam_time[fam] / 1e3
        hbm_bound = fam in ("split_k", "stream")
        if hbm_bound:
            achieved = fam_bytes[fam] / seconds / 1e9
            peak = peaks["hbm_gbs"]
            unit = "GB/s"
        else:
            achieved = fam_flops[fam] / seconds / 1e12
            peak = peaks["bf16_tflops"]
            unit = "TFLOP/s"
        return {
            "bound": "hbm" if hbm_bound else "tensor",
            "achieved": round(achieved, 2),
            "peak": peak,
            "unit": unit,
            "frac": round(achieved / peak, 4),
            "peak_source": f"{peak_source} (burst)",
            "launches_per_pass": fam_launches[fam],
            "share_of_pass": round(fam_time[fam] / pass_ms, 4),
        }

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
        "config": {
            "workload": f"{args.workload}: {len(workloads)} shapes" if not args.shapes else f"shapes {args.shapes}",
            "parallelism": f"replicas x{world}" if world > 1 else "single GPU",
            "l2": "256 MiB write before every launch",
            "selection": (
                f"Thompson bandit, {args.budget} probes per shape on bank-1 tensors"
                + (
                    f"; the best {args.confirm} probes within {args.confirm_within:.2f}x re-timed side by side in"
                    f" 5 passes on bank-1 tensors ({confirmed} shapes changed)"
                    if args.confirm > 1 and not (args.force or args.choices)
                    else ""
                )
                + "; scored on bank-2 tensors"
            ),
            "timing": "per-launch CUDA events on the launching stream; per-shape median over steps",
        },
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
            "note": "one pass: per shape H2D of A and B from pinned memory (copy-in stream), launch, D2H of C (copy-out stream); shapes pipelined, timed first copy to last D2H",
        },
        "gpu_launches": launches,
        "clocks": clocks,
        "wall_s_timed_region": round(ours_wall, 3),
        "tuning_s": round(tuning_s, 1),
        "status_bits": _native.status(local_rank),
    }
    if args.detail:
        detail = ROOT / "gpurun_out" / f"bench_detail_{args.tag or args.workload}.json"
        detail.parent.mkdir(exist_ok=True)
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
        result["cpu_baseline"] = cpu_baseline(workloads, args.cpu_rows, args.cpu_budget_s)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return result if rank == 0 else None


def run_colpar(args: argparse.Namespace) -> dict[str, object] | None:
    """Config 5: C[M, N] = A[M, K] B[K, N] with B split N-wise over the ranks, each rank's
    slice computed by the B200 GEMM, NCCL all-gather of the slices, column assembly."""
    import torch
    import torch.distributed as dist

    from heliostune_b200 import _native
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
    (w,) = _workloads("colpar", args.shapes)
    shard = ColumnShard(w.n, world, rank)
    g = torch.Generator(device=device).manual_seed(5)
    a = (torch.randn((w.m, w.k), generator=g, device=device) / math.sqrt(w.k)).to(torch.float16)
    g = torch.Generator(device=device).manual_seed(1000 + rank)
    b_shard = (torch.randn((w.k, shard.cols), generator=g, device=device) / math.sqrt(w.k)).to(torch.float16)

    if args.exchange == "fused" and world > 1:
        from heliostune_b200.column_parallel import FusedColumnParallel

        fused = FusedColumnParallel(w.m, w.n, device=device)

        def step(events):
            return fused(a, b_shard, phase_events=events)
    else:
        fused = None

        def step(events):
            return column_parallel_matmul(a, b_shard, phase_events=events)

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
    for s_ in range(args.steps):
        out = step(events[s_])
        del out
    torch.cuda.synchronize()
    epoch1 = time.time()
    sampler.__exit__(None, None, None)
    if world > 1:
        dist.barrier()
    gemm_ms = statistics.median(e[0].elapsed_time(e[1]) for e in events)
    gather_ms = statistics.median(e[1].elapsed_time(e[2]) for e in events)
    step_ms = statistics.median(e[0].elapsed_time(e[2]) for e in events)
    times = torch.tensor([step_ms, gemm_ms, gather_ms], device=device, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(times, op=dist.ReduceOp.MAX)
    step_ms, gemm_ms, gather_ms = (float(t) for t in times.tolist())
    peaks, source = _peaks()
    flops = 2.0 * w.m * w.n * w.k
    gemm_tflops = flops / world / (gemm_ms / 1e3) / 1e12
    gather_bytes = 2.0 * w.m * w.n * (world - 1) / world
    # Roofline of the whole step: the slower of the per-GPU GEMM at the tensor peak and the
    # all-gather bytes every GPU receives at the measured 770 GB/s peer bandwidth.
    t_roof = max(flops / world / (peaks["bf16_tflops_sustained"] * 1e12), gather_bytes / 770e9)
    result: dict[str, object] = {
        "metric": "column-parallel FP16 GEMM M=8192 K=8192 N=57344: TFLOP/s (whole job)",
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
        "config": {
            "workload": f"colpar M={w.m} N={w.n} K={w.k}",
            "parallelism": f"column-parallel x{world}",
            "gemm": column_parallel_candidate(w.m, shard.cols).key,
            "l2": "operands larger than L2",
        },
        "gemm_ms": round(gemm_ms, 4),
        "gather_ms": round(gather_ms, 4),
        "roofline": {
            "bound": "tensor",
            "achieved": round(gemm_tflops, 2),
            "peak": peaks["bf16_tflops_sustained"],
            "unit": "TFLOP/s",
            "frac": round(gemm_tflops / peaks["bf16_tflops_sustained"], 4),
            "peak_source": f"{source} (sustained)",
            "kernel": f"pair_gemm_kernel<{column_parallel_candidate(w.m, shard.cols).config.block_n},64> (GEMM phase, per GPU)",
            "traffic": None,
        },
        "step_roofline_frac": round(t_roof / (step_ms / 1e3), 4),
        "gather_gbs": round(gather_bytes / (gather_ms / 1e3) / 1e9, 1) if world > 1 else None,
        "gpu_launches": (1 if fused is not None or world == 1 else 2) * args.steps,
        "clocks": sampler.summary(epoch0, epoch1),
        "status_bits": _native.status(local_rank),
    }
    if fused is not None:
        result["config"]["exchange"] = "fused: GEMM epilogue stores every tile to all ranks over NVLink"
        result["gemm_ms_note"] = "fused mode: gemm_ms = barrier + GEMM with overlapped peer stores"
        fused.close()
    else:
        result["config"]["exchange"] = "NCCL all-gather + column assembly"
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return result if rank == 0 else None


def run_rmsnorm(args: argparse.Namespace) -> dict[str, object] | None:
    """Config 4: standalone RMSNorm over M in {1, 4096, 65536} x hidden in {4096, 8192}, and the
    RMSNorm feeding the (4096 -> 6144) QKV GEMM at M in {1, 128, 4096}. FP16, eps 1e-6,
    x ~ N(0, 1), gamma ~ 1 + 0.1 N(0, 1). Compared with the same math in eager torch."""
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
    }


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

    Each shape's A and B go host to device from pinned memory on a copy-in stream, the GEMM runs
    on the current stream once they have landed, and C goes back to pinned memory on a copy-out
    stream, so the next shape's inputs cross PCIe while this one's result returns. The pass is
    timed from the first copy to the last device-to-host copy; returns ``[pass_ms]``, h2d, d2h.
    """
    import torch

    from heliostune_b200.action_expansion import launch

    hosts = {}
    for w in workloads:
        a, b = operands[w.key]
        hosts[w.key] = (
            a.cpu().pin_memory(),
            b.cpu().pin_memory(),
            torch.empty((w.m, w.n), dtype=torch.float16).pin_memory(),
        )
    main = torch.cuda.current_stream(device)
    copy_in = torch.cuda.Stream(device)
    copy_out = torch.cuda.Stream(device)
    total = 0.0
    for step in range(steps + 1):  # the first pass warms up
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(main)
        copy_in.wait_event(start)
        for w in workloads:
            a_h, b_h, c_h = hosts[w.key]
            with torch.cuda.stream(copy_in):
                a = a_h.to(device, non_blocking=True)
                b = b_h.to(device, non_blocking=True)
            main.wait_stream(copy_in)
            a.record_stream(main)
            b.record_stream(main)
            c = launch(a, b, chosen[w.key])
            copy_out.wait_stream(main)
            with torch.cuda.stream(copy_out):
                c_h.copy_(c, non_blocking=True)
            c.record_stream(copy_out)
        main.wait_stream(copy_out)
        end.record(main)
        torch.cuda.synchronize()
        if step > 0:
            total += start.elapsed_time(end) / steps
    h2d = sum(2 * (w.m * w.k + w.k * w.n) for w in workloads)
    d2h = sum(2 * w.m * w.n for w in workloads)
    return [total], h2d, d2h


# ----------------------------------------------------------------------------------------------
# CPU baseline / reference arm
# ----------------------------------------------------------------------------------------------


def cpu_baseline(workloads, max_rows: int, budget_s: float) -> dict[str, object]:
    """The oracle's FP32 BLAS product on the host cores, on a bounded sample of each shape.

    Sample: the first ``min(M, max_rows)`` rows of A against the full B, inputs upcast from FP16
    inside the timing; shapes are visited in grid order until ``budget_s`` of CPU time is spent.
    """
    from oracle import oracle

    cores = os.cpu_count() or 1
    rng = np.random.default_rng(0)
    flops = 0.0
    seconds = 0.0
    sampled = 0
    b_cache: dict[tuple[int, int], np.ndarray] = {}
    for w in workloads:
        rows = min(w.m, max_rows)
        if (w.k, w.n) not in b_cache:
            b_cache.clear()
            b_cache[(w.k, w.n)] = (rng.standard_normal((w.k, w.n), dtype=np.float32) / math.sqrt(w.k)).astype(np.float16)
        b = b_cache[(w.k, w.n)]
        a = (rng.standard_normal((rows, w.k), dtype=np.float32) / math.sqrt(w.k)).astype(np.float16)
        t0 = time.perf_counter()
        oracle.gemm_fp32_blas(a, b)
        seconds += time.perf_counter() - t0
        flops += 2.0 * rows * w.n * w.k
        sampled += 1
        if seconds > budget_s:
            break
    return {
        "value": round(flops / seconds / 1e12, 4),
        "unit": "TFLOP/s",
        "cores": cores,
        "kind": "port",
        "sample": f"{sampled} shapes, first min(M, {max_rows}) rows each, FP16 upcast + FP32 BLAS (numpy) on {cores} host threads",
    }


def run_reference(args: argparse.Namespace) -> dict[str, object] | None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return None
    workloads = _workloads(args.workload, args.shapes)
    samples = []
    for _ in range(args.warmup):
        cpu_baseline(workloads, args.cpu_rows, args.cpu_budget_s / 4)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        samples.append(cpu_baseline(workloads, args.cpu_rows, args.cpu_budget_s))
    wall = time.perf_counter() - t0
    value = statistics.median(s["value"] for s in samples)
    base = samples[0]
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
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f16 inputs, fp32 accumulate (CPU)",
        "data": "synthetic: seeded N(0,1)/sqrt(K) FP16 operands",
        "config": {"workload": f"{args.workload}: {len(workloads)} shapes", "parallelism": "host CPU"},
        "cpu_baseline": {**base, "value": value},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=20)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", choices=("ours", "reference"), default="ours")
    parser.add_argument("--workload", choices=("grid", "sweep", "decode", "colpar", "rmsnorm"), default="grid")
    parser.add_argument("--shapes", default=None, help="comma list of MxNxK overriding the workload")
    parser.add_argument("--budget", type=int, default=8, help="bandit probes per shape")
    parser.add_argument("--probe-ms", type=float, default=10.0)
    parser.add_argument(
        "--confirm", type=int, default=3, help="re-time the best N probed candidates per shape in scored-like passes (1 = off)"
    )
    parser.add_argument("--confirm-within", type=float, default=1.10, help="finalists: probe latency within this factor of the best")
    parser.add_argument("--seed", type=int, default=0)
    parser.add_argument("--e2e-steps", type=int, default=1)
    parser.add_argument("--cpu-rows", type=int, default=64)
    parser.add_argument("--cpu-budget-s", type=float, default=20.0)
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--detail", action="store_true", help="also write per-shape results to bench_detail_<tag>.json")
    parser.add_argument("--choices", default=None, help="per-shape choices from an earlier --detail file")
    parser.add_argument("--skip-cublas", action="store_true", help="profiling runs: no cuBLAS passes")
    parser.add_argument("--force", default=None, help="profiling runs: one candidate key for every shape")
    parser.add_argument("--tag", default=None, help="name of the --detail file")
    parser.add_argument(
        "--exchange",
        choices=("fused", "nccl"),
        default="fused",
        help="colpar: all-gather fused into the GEMM epilogue, or NCCL all-gather + assembly",
    )
    args = parser.parse_args()
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
