"""A deterministic pilot collection built by ``heliostune_b200.collection`` without a GPU.

``fake_measure`` stands in for ``action_expansion.measure_unit``: it returns rows with the unit
protocol's keys, order and identities (torch first, then the seeded shuffle), latencies drawn
from a hash of (bank, workload, configuration), and one configuration per unit that fails its
correctness check, so the artifact also carries failure rows. ``build`` runs the pilot plan
through ``Collection`` with a fixed session and clock. ``make_golden.py`` hands the result to
the reference's own analysis (scripts/analyze_action_expansion.py) and records what it returned;
the tests rebuild it and compare.
"""

from __future__ import annotations

import hashlib
from pathlib import Path
from typing import Any

from heliostune_b200.action_collection import timing_order
from heliostune_b200.action_configs import action_set_manifest
from heliostune_b200.collection import Collection, RunSpec
from heliostune_b200.configs import Workload
from heliostune_b200.schema import B200_PROFILE

SPEC = RunSpec(
    run_id="b200-fixture",
    runner="local",
    gpu="B200",
    pilot=True,
    source_commit="1" * 40,
    plan_commit="2" * 40,
    collector_sha256="3" * 64,
    source_sha256="4" * 64,
)


def _identities() -> dict[str, dict[str, Any]]:
    manifest = action_set_manifest()
    out = {r["config_key"]: r for arm in ("old", "new") for r in manifest[arm]}
    out["torch"] = {"family": "torch", "config_key": "torch", "config": None}
    return out


def _unit_hash(*parts: object) -> float:
    digest = hashlib.sha256("|".join(map(str, parts)).encode()).digest()
    return int.from_bytes(digest[:8], "big") / 2.0**64


def fake_measure(bank: int, index: int, workload: Workload, finalists: frozenset[str] | None) -> list[dict[str, Any]]:
    identities = _identities()
    keys = timing_order(bank, index, workload, finalists)
    failing = keys[1 + int(_unit_hash("fail", workload.key) * (len(keys) - 1))] if bank == 1 else None
    rows = []
    for key in keys:
        identity = identities[key]
        base = 0.01 + workload.flops / 400e12 * 1e3  # about 400 TFLOP/s, in milliseconds
        median = base * (0.7 + 0.8 * _unit_hash(bank, workload.key, key))
        row: dict[str, Any] = {
            "workload_key": workload.key,
            "workload": workload.to_dict(),
            "bank": bank,
            "family": identity["family"],
            "config_key": key,
            "config": identity["config"],
            "correct": key != failing,
            "error": None if key != failing else "correctness: ValueError: outside unchanged atol=rtol=1e-2 tolerance",
            "p20_ms": None if key == failing else median * 0.98,
            "median_ms": None if key == failing else median,
            "p80_ms": None if key == failing else median * 1.03,
            "max_abs_error": 0.0078125 if key != failing else 0.5,
            "compile_seconds": 0.001,
            "timing_seconds": None if key == failing else 0.125,
        }
        rows.append(row)
    return rows


def build(directory: Path) -> dict[str, Any]:
    """The pilot artifact, checkpointed under ``directory``."""
    ticks = iter(range(10**6))
    collection = Collection.fresh(
        SPEC,
        directory / "checkpoint.json",
        B200_PROFILE.to_dict(),
        {"torch": "fixture", "numpy": "fixture"},
        {"allow_tf32": False, "allow_fp16_reduced_precision_reduction": True, "float32_matmul_precision": "highest"},
    )
    session = {"id": "fixture-session", "runner": "local", "source_commit": SPEC.source_commit, "hardware": B200_PROFILE.to_dict()}
    return collection.run(fake_measure, session=session, clock=lambda: float(next(ticks)), log=lambda _m: None)
