"""The bandit's feature bases: the reference's 25-column v2 basis and a B200 extension.

``v2_joint_features`` restates ``_v2_values`` at ``src/heliostune/features.py:66-116`` column
for column. The reference only defines it for tile configurations; here every family is mapped
onto the same six launch fields by :func:`launch_fields`:

* tile / persistent -- the fields as given;
* split-K -- ``group_m`` carries ``split_k`` (the reference has no raster group for split-K);
* stream -- ``group_m`` carries the split the launcher will actually use for the shape;
* pair -- the fields as given (``block_m`` = 256 rows per two SMs).

The v2 fields cannot tell the B200 families apart: a 256 x 256 pair tile, its split and stream-K
forms and the 128-deep form differ in no field or in ``block_k`` alone, and a stream launch's
split hides in ``group_m``. :func:`b200_joint_features` appends two columns measured to help the
cold-start bandit on B200 timing tables (``heliostune_b200.replay``):

* ``log_roofline_tflops`` -- log2 of the throughput the shape's roofline allows on the B200
  (the slower of 2MNK at the dense FP16 tensor peak and the FP16 operand bytes at the HBM
  bandwidth, both as measured on this pool's B200s): the shape's baseline, the same for every
  candidate, which a linear reward model otherwise has to assemble from the log M, N, K columns;
* ``wave_fill`` -- the share of the B200's resident slots (SMs, CTA pairs or clusters of the
  launch's size) the candidate's grid keeps busy over its waves; stream-K counts as full.

Columns naming the family, cluster size, split count, K per split and stream-K were measured as
well and made the replay worse (more parameters for the same probes), so they are not part of
the basis; :func:`launch_shape` still describes each launch that way.
"""

from __future__ import annotations

import math
from typing import NamedTuple

import numpy as np
from numpy.typing import NDArray

from heliostune_b200.action_configs import (
    PAIR_STREAM_K,
    PairConfig,
    SplitKConfig,
    StreamConfig,
    resident_clusters,
    split_plan,
    stream_splits,
    wave_fill,
)
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


#: The v2 columns followed by the B200 columns of :func:`b200_joint_features`.
B200_FEATURE_NAMES: tuple[str, ...] = (*V2_FEATURE_NAMES, "log_roofline_tflops", "wave_fill")

#: Dense FP16 tensor peak (TFLOP/s per 148 SMs) and HBM bandwidth (GB/s) measured on this pool's
#: B200s (a cuBLAS GEMM and a device copy); they only set the scale of ``log_roofline_tflops``.
B200_TENSOR_TFLOPS_PER_148_SMS = 1620.0
B200_HBM_GBS = 6539.5


class LaunchShape(NamedTuple):
    family: str
    cluster: int  # CTAs per cluster (a CTA pair is 2)
    splits: int  # K intervals one output tile is summed from
    k_block: int
    stream_k: bool
    busy: float  # share of the resident slots busy over the launch's waves


def launch_shape(workload: Workload, config: object, sms: int) -> LaunchShape:
    """How a candidate occupies the B200 for ``workload``: family, cluster, splits, busy share."""
    m, n, k = workload.m, workload.n, workload.k
    if isinstance(config, PairConfig):
        tiles = -(-m // 256) * -(-n // config.block_n)
        splits = config.split_k if config.split_k > 1 else 1
        cluster = 2 * splits
        slots = resident_clusters(min(cluster, 8), sms)
        busy = 1.0 if config.split_k == PAIR_STREAM_K else wave_fill(tiles, slots)
        return LaunchShape("pair", cluster, splits, config.block_k, config.split_k == PAIR_STREAM_K, busy)
    if isinstance(config, StreamConfig):
        splits = stream_splits(m, n, k, config, sms)
        ctas = -(-n // config.block_n)
        return LaunchShape("stream", splits, splits, config.block_k, False, wave_fill(ctas, resident_clusters(splits, sms)))
    if isinstance(config, SplitKConfig):
        bk = 64 if config.block_k <= 64 else 128
        splits = split_plan(k, bk, config.split_k)[1]
        return LaunchShape("split_k", 1, splits, bk, False, wave_fill(-(-n // config.block_n) * splits, sms))
    if not isinstance(config, KernelConfig | HopperGemmConfig):
        raise TypeError("unknown configuration type")
    tiles = -(-m // config.block_m) * -(-n // config.block_n)
    family = "persistent" if isinstance(config, HopperGemmConfig) else "tile"
    return LaunchShape(family, 1, 1, config.block_k, False, wave_fill(tiles, sms))


def log_roofline_tflops(workload: Workload, sms: int) -> float:
    """log2 of the roofline throughput (TFLOP/s) of ``workload`` on a B200 with ``sms`` SMs."""
    flops = 2.0 * workload.m * workload.n * workload.k
    nbytes = 2.0 * (workload.m * workload.k + workload.k * workload.n + workload.m * workload.n)
    seconds = max(flops / (B200_TENSOR_TFLOPS_PER_148_SMS * sms / 148 * 1e12), nbytes / (B200_HBM_GBS * 1e9))
    return math.log2(flops / seconds / 1e12)


def b200_joint_features(
    workload: Workload,
    config: KernelConfig | HopperGemmConfig | SplitKConfig | StreamConfig | PairConfig,
    hardware: HardwareProfile,
) -> NDArray[np.float64]:
    """The v2 vector of the same triple followed by the B200 columns (:data:`B200_FEATURE_NAMES`)."""
    fields = launch_fields(workload, config, hardware)
    sms = hardware.multiprocessor_count
    extra = (log_roofline_tflops(workload, sms) / 11.0, launch_shape(workload, config, sms).busy)
    return np.asarray((*_v2_values(workload, fields, hardware), *extra), dtype=np.float64)


#: Feature bases by name: their column names and the function computing them.
FEATURE_BASES = {"v2": (V2_FEATURE_NAMES, v2_joint_features), "b200": (B200_FEATURE_NAMES, b200_joint_features)}
