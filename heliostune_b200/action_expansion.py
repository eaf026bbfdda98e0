"""Drop-in for ``heliostune.action_expansion``: split-K, the dispatcher and the measurement unit.

``_split_k_matmul`` and ``launch`` keep the reference's signatures, checks, error types and
allocation (``src/heliostune/action_expansion.py:124-185``): every call allocates its FP16 output
and its FP32 ``[split, M, N]`` workspace with ``torch.empty`` (so allocation is inside any timing
of the call), launches the partials kernel and the fixed-order reduction on the current stream,
and never falls back to another implementation. ``_stream_matmul`` adds the B200
weight-streaming family. ``measure_unit`` restates the per-unit protocol (``:188-273``).
"""

from __future__ import annotations

import math
import time
from collections.abc import Callable
from functools import partial
from typing import Any

import torch

from heliostune_b200 import _native
from heliostune_b200.action_collection import ATOL, REP_MS, RTOL, WARMUP_MS, tensor_seed, timing_order
from heliostune_b200.action_configs import (
    SPLIT_K_M_LIMIT,
    PairConfig,
    STREAM_M_LIMIT,
    ActionCandidate,
    SplitKConfig,
    StreamConfig,
    candidates_for,
)
from heliostune_b200.configs import DEFAULT_CONFIGS, HopperGemmConfig, KernelConfig, Workload
from heliostune_b200.hopper_kernel import hopper_matmul
from heliostune_b200.kernel import _device_guard, _stream, _validate, _within_tolerance, _workspace, matmul
from heliostune_b200.timing import do_bench


def _split_k_matmul(a: torch.Tensor, b: torch.Tensor, config: SplitKConfig) -> torch.Tensor:
    m, n, k = _validate(a, b)
    if not 1 <= m <= SPLIT_K_M_LIMIT or n < 1 or k < 1:
        raise ValueError("split-K requires 1 <= M <= 31 and positive N and K")
    output = torch.empty((m, n), device=a.device, dtype=torch.float16)
    native = _native.GemmConfig(
        _native.FAMILY_SPLIT_K,
        config.block_m,
        config.block_n,
        config.block_k,
        config.num_warps,
        config.num_stages,
        8,
        config.split_k,
    )
    workspace, ws_ptr, ws_bytes = _workspace(native, a, b, m, n, k)
    with _device_guard(a.device):
        _native.check(
            _native.library().hst_matmul_split_k(
                config.block_m,
                config.block_n,
                config.block_k,
                config.num_warps,
                config.num_stages,
                config.split_k,
                a.data_ptr(),
                a.stride(0),
                a.stride(1),
                b.data_ptr(),
                b.stride(0),
                b.stride(1),
                output.data_ptr(),
                n,
                m,
                n,
                k,
                ws_ptr,
                ws_bytes,
                _stream(a.device),
            )
        )
    del workspace
    return output


def _stream_matmul(a: torch.Tensor, b: torch.Tensor, config: StreamConfig) -> torch.Tensor:
    m, n, k = _validate(a, b)
    if not 1 <= m <= STREAM_M_LIMIT or n < 1 or k < 1:
        raise ValueError(f"the stream family requires 1 <= M <= {STREAM_M_LIMIT} and positive N and K")
    if config.block_m < m:
        raise ValueError(f"stream block_m {config.block_m} does not cover M={m}")
    output = torch.empty((m, n), device=a.device, dtype=torch.float16)
    native = _native.GemmConfig(
        _native.FAMILY_STREAM,
        config.block_m,
        config.block_n,
        config.block_k,
        config.num_warps,
        config.num_stages,
        8,
        config.split_k,
    )
    workspace, ws_ptr, ws_bytes = _workspace(native, a, b, m, n, k)
    with _device_guard(a.device):
        _native.check(
            _native.library().hst_matmul_stream(
                config.block_m,
                config.block_n,
                config.block_k,
                config.num_stages,
                config.split_k,
                a.data_ptr(),
                a.stride(0),
                a.stride(1),
                b.data_ptr(),
                b.stride(0),
                b.stride(1),
                output.data_ptr(),
                n,
                m,
                n,
                k,
                ws_ptr,
                ws_bytes,
                _stream(a.device),
            )
        )
    del workspace
    return output


def _pair_matmul(a: torch.Tensor, b: torch.Tensor, config: PairConfig) -> torch.Tensor:
    m, n, k = _validate(a, b)
    output = torch.empty((m, n), device=a.device, dtype=torch.float16)
    native = _native.GemmConfig(
        _native.FAMILY_PAIR,
        config.block_m,
        config.block_n,
        config.block_k,
        config.num_warps,
        config.num_stages,
        config.group_m,
        config.split_k,
    )
    workspace, ws_ptr, ws_bytes = _workspace(native, a, b, m, n, k)
    with _device_guard(a.device):
        _native.check(
            _native.library().hst_matmul_pair(
                config.block_n,
                config.block_k,
                config.num_stages,
                config.group_m,
                config.split_k,
                a.data_ptr(),
                a.stride(0),
                a.stride(1),
                b.data_ptr(),
                b.stride(0),
                b.stride(1),
                output.data_ptr(),
                n,
                m,
                n,
                k,
                ws_ptr,
                ws_bytes,
                _stream(a.device),
            )
        )
    del workspace
    return output


def launch(a: torch.Tensor, b: torch.Tensor, candidate: ActionCandidate) -> torch.Tensor:
    """Allocate and launch exactly the requested action, propagating every failure."""
    config = candidate.config
    if isinstance(config, KernelConfig):
        return matmul(a, b, config)
    if isinstance(config, HopperGemmConfig):
        return hopper_matmul(a, b, config)
    if isinstance(config, SplitKConfig):
        return _split_k_matmul(a, b, config)
    if isinstance(config, StreamConfig):
        return _stream_matmul(a, b, config)
    if isinstance(config, PairConfig):
        return _pair_matmul(a, b, config)
    raise TypeError("unknown action configuration")


def fp32_reference(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """The reference's check value: an FP32 product of the FP16 operands, TF32 disabled."""
    previous = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        return torch.mm(a.float(), b.float())
    finally:
        torch.backends.cuda.matmul.allow_tf32 = previous


def measure_unit(
    bank: int,
    index: int,
    workload: Workload,
    finalists: frozenset[str] | None,
    *,
    device: torch.device,
    warmup_ms: float = WARMUP_MS,
    rep_ms: float = REP_MS,
) -> list[dict[str, Any]]:
    """Check and time one bank/workload unit; every failure stays a row with its stage.

    Seeded uniform(-1, 1) FP16 operands, an FP32 reference with TF32 off, torch first, then the
    seeded shuffle of the 36 old configurations and the frozen candidates.
    """
    torch.manual_seed(tensor_seed(bank, index))
    a = torch.empty((workload.m, workload.k), device=device, dtype=torch.float16)
    b = torch.empty((workload.k, workload.n), device=device, dtype=torch.float16)
    a.uniform_(-1.0, 1.0)
    b.uniform_(-1.0, 1.0)
    expected = fp32_reference(a, b)
    difference = torch.empty_like(expected)
    actions: dict[str, tuple[str, Any, Callable[[], torch.Tensor]]] = {
        c.key: ("old", c.to_dict(), partial(matmul, a, b, c)) for c in DEFAULT_CONFIGS
    }
    for candidate in candidates_for(workload):
        actions[candidate.key] = (candidate.family, candidate.to_dict(), partial(launch, a, b, candidate))
    actions["torch"] = ("torch", None, partial(torch.matmul, a, b))
    rows: list[dict[str, Any]] = []
    for key in timing_order(bank, index, workload, finalists):
        family, config, function = actions[key]
        row: dict[str, Any] = {
            "workload_key": workload.key,
            "workload": workload.to_dict(),
            "bank": bank,
            "family": family,
            "config_key": key,
            "config": config,
            "correct": False,
            "error": None,
            "p20_ms": None,
            "median_ms": None,
            "p80_ms": None,
            "max_abs_error": None,
            "compile_seconds": None,
            "timing_seconds": None,
        }
        stage = "compile"
        try:
            torch.cuda.synchronize()
            started = time.monotonic()
            output = function()
            torch.cuda.synchronize()
            row["compile_seconds"] = time.monotonic() - started
            stage = "correctness"
            if not bool(torch.isfinite(output).all().item()):
                raise ValueError("non-finite output")
            torch.sub(output, expected, out=difference)
            difference.abs_()
            row["max_abs_error"] = float(difference.max().item())
            if not _within_tolerance(difference, expected, atol=ATOL, rtol=RTOL):
                raise ValueError("outside unchanged atol=rtol=1e-2 tolerance")
            row["correct"] = True
            del output
            stage = "timing"
            started = time.monotonic()
            p20, p50, p80 = do_bench(function, warmup_ms=warmup_ms, rep_ms=rep_ms)
            if not all(math.isfinite(v) and v > 0 for v in (p20, p50, p80)):
                raise ValueError("non-positive or non-finite timing")
            row.update(p20_ms=p20, median_ms=p50, p80_ms=p80, timing_seconds=time.monotonic() - started)
        except Exception as exc:  # noqa: BLE001 -- a failure is a row, as in the reference
            row["error"] = f"{stage}: {type(exc).__name__}: {exc}"
        rows.append(row)
    return rows
