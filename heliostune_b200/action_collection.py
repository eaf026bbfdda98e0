"""CPU-side protocol of a measurement collection: seeds, timing order, finalist selection.

Restates ``src/heliostune/action_collection.py:30-189``: the frozen protocol constants, the
seeded per-bank workload shuffle, the tensor seed ``bank * 10000 + index``, the per-unit timing
order (torch first, then a seeded shuffle of the configuration keys) and the bank-1 finalist
rule (minimum correct median, ties broken by key). Nothing here imports torch.
"""

from __future__ import annotations

import random
from collections.abc import Mapping, Sequence
from typing import Any

from heliostune_b200.action_configs import candidates_for
from heliostune_b200.configs import DEFAULT_CONFIGS, Workload

BANKS = (1, 2)
WARMUP_MS = 25
REP_MS = 100
QUANTILES = (0.2, 0.5, 0.8)
ATOL = 1e-2
RTOL = 1e-2


def protocol() -> dict[str, Any]:
    return {
        "warmup_ms": WARMUP_MS,
        "rep_ms": REP_MS,
        "quantiles": list(QUANTILES),
        "atol": ATOL,
        "rtol": RTOL,
        "selection_bank": 1,
        "scoring_bank": 2,
        "selection": "minimum correct bank-1 median, then config-key tie-break",
        "reference": "FP16 operands; FP32 matmul reference, TF32 disabled",
        "timed_calls": "allocating CUDA FP16 calls; split-K workspace/reduction included",
        "tensor_seed": "bank * 10000 + index in that bank's shuffled workload order",
        "workload_order_seed": "bank",
        "config_order_seed": "bank * 10000 + workload index + 70000",
    }


def bank_order(workloads: Sequence[Workload], bank: int) -> list[Workload]:
    order = list(workloads)
    random.Random(bank).shuffle(order)
    return order


def tensor_seed(bank: int, index: int) -> int:
    return bank * 10000 + index


def timing_order(
    bank: int, index: int, workload: Workload, finalists: frozenset[str] | None
) -> list[str]:
    """Configuration keys in timing order: torch first, then the seeded candidate shuffle."""
    keys = [c.key for c in DEFAULT_CONFIGS] + [c.key for c in candidates_for(workload)]
    if finalists is not None:
        keys = [key for key in keys if key in finalists]
    random.Random(bank * 10000 + index + 70000).shuffle(keys)
    return ["torch", *keys]


def select_finalists(rows: Sequence[Mapping[str, Any]]) -> dict[str, str | None]:
    """The minimum valid bank-1 median, separately for the old and the new actions."""
    selection: dict[str, str | None] = {}
    for group in ("old", "new"):
        valid = [
            r
            for r in rows
            if r["family"] != "torch"
            and (r["family"] == "old") == (group == "old")
            and r["correct"]
            and r["error"] is None
            and r["median_ms"] is not None
        ]
        selection[group] = (
            min(valid, key=lambda r: (r["median_ms"], r["config_key"]))["config_key"]
            if valid
            else None
        )
    return selection
