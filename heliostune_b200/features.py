"""The 25-column v2 feature basis of the bandit.

``v2_joint_features`` restates ``_v2_values`` at ``src/heliostune/features.py:66-116`` column
for column. The reference only defines it for tile configurations; here every family is mapped
onto the same six launch fields by :func:`launch_fields`:

* tile / persistent -- the fields as given;
* split-K -- ``group_m`` carries ``split_k`` (the reference has no raster group for split-K);
* stream -- ``group_m`` carries the split the launcher will actually use for the shape;
* pair -- the fields as given (``block_m`` = 256 rows per two SMs).
"""

from __future__ import annotations

import math
from typing import NamedTuple

import numpy as np
from numpy.typing import NDArray

from heliostune_b200.action_configs import PairConfig, SplitKConfig, StreamConfig, stream_splits
from heliostune_b200.configs import HopperGemmConfig, KernelConfig, Workload
from heliostune_b200.schema import HardwareProfile

V2_FEATURE_NAMES: tuple[str, ...] = (
    "bias",
    "log_m",
    "log_n",
    "log_k",
    "log_m_over_n",
    "log_k_over_n",
    "log_flops",
    "block_m",
    "block_n",
    "block_k",
    "warps",
    "stages",
    "group_m",
    "m_tile_coverage",
    "m_divisible",
    "n_divisible",
    "k_divisible",
    "multiprocessors",
    "memory_gb",
    "compute_capability",
    "m_x_block_m",
    "n_x_block_n",
    "k_x_block_k",
    "sm_x_warps",
    "memory_x_tile_area",
)


class LaunchFields(NamedTuple):
    block_m: int
    block_n: int
    block_k: int
    num_warps: int
    num_stages: int
    group_m: int


def launch_fields(
    workload: Workload,
    config: KernelConfig | HopperGemmConfig | SplitKConfig | StreamConfig | PairConfig,
    hardware: HardwareProfile,
) -> LaunchFields:
    """Map any candidate configuration onto the six fields the v2 basis reads."""
    if isinstance(config, KernelConfig | HopperGemmConfig | PairConfig):
        group = config.group_m
    elif isinstance(config, SplitKConfig):
        group = config.split_k
    elif isinstance(config, StreamConfig):
        group = stream_splits(
            workload.m, workload.n, workload.k, config, hardware.multiprocessor_count
        )
    else:
        raise TypeError("unknown configuration type")
    return LaunchFields(
        config.block_m, config.block_n, config.block_k, config.num_warps, config.num_stages, group
    )


def _v2_values(workload: Workload, fields: LaunchFields, hardware: HardwareProfile) -> tuple[float, ...]:
    lm = math.log2(workload.m) / 14.0
    ln = math.log2(workload.n) / 14.0
    lk = math.log2(workload.k) / 14.0
    bm = math.log2(fields.block_m) / 7.0
    bn = math.log2(fields.block_n) / 7.0
    bk = math.log2(fields.block_k) / 7.0
    sms = hardware.multiprocessor_count / 128.0
    memory = hardware.total_memory_gb / 48.0
    major, minor = hardware.compute_capability
    capability = (major + minor / 10) / 10
    area = (fields.block_m * fields.block_n) / (128.0 * 128.0)
    warps = math.log2(fields.num_warps) / 3.0
    return (
        1.0,
        lm,
        ln,
        lk,
        (math.log2(workload.m) - math.log2(workload.n)) / 14.0,
        (math.log2(workload.k) - math.log2(workload.n)) / 14.0,
        math.log2(workload.flops) / 42.0,
        bm,
        bn,
        bk,
        warps,
        fields.num_stages / 5.0,
        fields.group_m / 8.0,
        min(workload.m, fields.block_m) / fields.block_m,
        float(workload.m % fields.block_m == 0),
        float(workload.n % fields.block_n == 0),
        float(workload.k % fields.block_k == 0),
        sms,
        memory,
        capability,
        lm * bm,
        ln * bn,
        lk * bk,
        sms * math.log2(fields.num_warps) / 3.0,  # same association as the reference
        memory * area,
    )


def v2_joint_features(
    workload: Workload,
    config: KernelConfig | HopperGemmConfig | SplitKConfig | StreamConfig,
    hardware: HardwareProfile,
) -> NDArray[np.float64]:
    """The 25-column feature vector of one (workload, configuration, hardware) triple."""
    fields = launch_fields(workload, config, hardware)
    return np.asarray(_v2_values(workload, fields, hardware), dtype=np.float64)
