"""Host-side helpers of bench.py: finalist selection for the confirmation passes, the metric
name, and the kernel-family labels the roofline is grouped by (no GPU needed)."""

from __future__ import annotations

import argparse

import pytest

import bench
from heliostune_b200.action_configs import (
    PAIR_DEEP_K,
    PAIR_NARROW,
    PAIR_WIDE,
    PAIR_WIDE_STREAM_K,
    ActionCandidate,
    StreamConfig,
)
from heliostune_b200.tuner import Probe


def test_finalists_keep_the_fastest_within_the_window_in_order() -> None:
    stream = ActionCandidate(StreamConfig(16, 128, 64, 4, 4, 0))
    probes = [
        Probe(PAIR_DEEP_K, 1.05),
        Probe(PAIR_WIDE, 1.00),
        Probe(PAIR_NARROW, 1.20),  # outside 1.10x
        Probe(stream, None, "ValueError: parity failure"),  # failed probes never qualify
        Probe(PAIR_WIDE_STREAM_K, 1.09),
    ]
    keys = [c.key for c in bench._finalists(probes, 3, 1.10)]
    assert keys == [PAIR_WIDE.key, PAIR_DEEP_K.key, PAIR_WIDE_STREAM_K.key]
    assert [c.key for c in bench._finalists(probes, 2, 1.10)] == [PAIR_WIDE.key, PAIR_DEEP_K.key]
    assert [c.key for c in bench._finalists(probes, 3, 1.0)] == [PAIR_WIDE.key]


def test_finalists_need_a_valid_probe() -> None:
    with pytest.raises(RuntimeError):
        bench._finalists([Probe(PAIR_WIDE, None, "KernelError: timeout")], 3, 1.10)


def test_metric_name_is_baselines_for_the_grid_only() -> None:
    grid = argparse.Namespace(workload="grid", shapes=None)
    assert bench._metric(grid, 96) == bench.METRIC
    sweep = argparse.Namespace(workload="sweep", shapes=None)
    assert "28-shape FP16 sweep" in bench._metric(sweep, 28)
    custom = argparse.Namespace(workload="grid", shapes="512x4608x3584")
    assert "1-shape FP16 custom shapes" in bench._metric(custom, 1)
    colpar = argparse.Namespace(workload="colpar", shapes=None)
    assert bench._metric(colpar, 1) == bench.COLPAR_METRIC  # both arms print this name


def test_kernel_families() -> None:
    assert bench._kernel_family(PAIR_WIDE) == "pair_wide"
    assert bench._kernel_family(PAIR_WIDE_STREAM_K) == "pair_wide"
    assert bench._kernel_family(PAIR_DEEP_K) == "pair_deep_k"
    assert bench._kernel_family(PAIR_NARROW) == "pair"
    assert bench._kernel_family(ActionCandidate(StreamConfig(16, 128, 64, 4, 4, 0))) == "stream"


def test_launch_counts() -> None:
    from heliostune_b200.action_configs import SplitKConfig
    from heliostune_b200.configs import Workload

    w = Workload(4, 6144, 4096, "x", "y", "z")
    assert bench._launch_count(ActionCandidate(SplitKConfig(16, 128, 64, 4, 3, 4)), w, 148) == 2  # + reduce
    assert bench._launch_count(ActionCandidate(StreamConfig(16, 128, 64, 4, 4, 0)), w, 148) == 1
    assert bench._launch_count(PAIR_WIDE, Workload(8192, 4096, 4096, "x", "y", "z"), 148) == 1


def _args(**overrides: object) -> argparse.Namespace:
    base = dict(
        workload="grid", shapes=None, budget=8, force=None, choices=None, confirm=3, confirm_within=1.10,
        exchange="fused", steps=2, warmup=1, cpu_step_s=0.05, cpu_budget_s=0.05,
    )
    base.update(overrides)
    return argparse.Namespace(**base)


def test_torchrun_launch_is_detected(monkeypatch: pytest.MonkeyPatch) -> None:
    for name in ("TORCHELASTIC_RUN_ID", "LOCAL_WORLD_SIZE"):
        monkeypatch.delenv(name, raising=False)
    assert not bench._distributed_launch()
    monkeypatch.setenv("LOCAL_WORLD_SIZE", "1")
    assert bench._distributed_launch()


def test_column_parallel_config_names_the_exchange(monkeypatch: pytest.MonkeyPatch) -> None:
    args = _args(workload="colpar")
    workloads = bench._workloads("colpar", None)
    monkeypatch.setenv("WORLD_SIZE", "8")
    config = bench._config(args, workloads)
    assert config["workload"] == "colpar M=8192 N=57344 K=8192"
    assert config["parallelism"] == "column-parallel x8" and config["exchange"].startswith("fused")
    monkeypatch.setenv("WORLD_SIZE", "1")
    assert bench._config(args, workloads)["exchange"].startswith("none")


def test_reference_arm_prints_our_config_and_a_cpu_baseline(monkeypatch: pytest.MonkeyPatch) -> None:
    monkeypatch.delenv("RANK", raising=False)
    monkeypatch.delenv("WORLD_SIZE", raising=False)
    args = _args(shapes="3x40x24,5000x16x8")  # the tall shape is cut into 2048-row blocks
    line = bench.run_reference(args)
    assert line is not None and line["impl"] == "reference"
    assert line["config"] == bench._config(args, bench._workloads("grid", args.shapes))
    cpu = line["cpu_baseline"]
    assert cpu["kind"] == "port" and cpu["cores"] >= 1 and cpu["cpu_model"]
    assert cpu["full_workload"] and cpu["value"] == line["value"] > 0
    assert line["e2e"] == {"value": line["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    monkeypatch.setenv("RANK", "1")
    assert bench.run_reference(args) is None  # only rank 0 runs the CPU arm


def test_cpu_baseline_walks_the_pieces_round_robin() -> None:
    from heliostune_b200.configs import Workload

    workloads = (Workload(3, 40, 24, "x", "y", "z"), Workload(4100, 8, 16, "x", "y", "z"))
    baseline = bench.CpuBaseline(workloads)
    assert [(r0, r1) for _, r0, r1 in baseline.pieces] == [(0, 3), (0, 2048), (2048, 4096), (4096, 4100)]
    baseline.run(0.0)  # at least one piece per call
    assert [len(t) for t in baseline.samples] == [1, 0, 0, 0]
    baseline.run(0.0)
    assert [len(t) for t in baseline.samples] == [1, 1, 0, 0]
    summary = baseline.summary()
    assert not summary["full_workload"] and "2 of 4 pieces" in summary["sample"]
