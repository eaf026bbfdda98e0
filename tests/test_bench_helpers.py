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
