"""Collection of raw measurement rows on the B200, in the reference's artifact format.

The reference's collector (``collect_on_device``, ``src/heliostune/action_expansion.py:276-324``,
over the run plumbing of ``src/heliostune/action_collection.py:60-262``) measures every
bank/workload unit with the unit protocol, checkpoints after each unit, resumes an interrupted
run, and writes one JSON artifact that its analysis script
(``scripts/analyze_action_expansion.py:159-382``) scores. This module produces the same artifact
from this library's kernels:

* top level: ``schema_version``, ``run``, ``plan_commit``, ``source_commit``, ``pilot``,
  ``hardware``, ``software``, ``precision``, ``protocol``, ``action_set``, ``rows``,
  ``selected``, ``duration_seconds``, ``sessions``;
* ``rows``: one row per timed action (``action_expansion.measure_unit``); bank 1 times torch,
  the 36 stock tile configurations and the frozen candidates of the workload, bank 2 times
  torch and the two bank-1 finalists (old and new);
* the checkpoint ``{"data": artifact, "completed_units": [[bank, workload_key], ...]}`` after
  every unit, written atomically; a resume must match every identity field.

``Collection`` keeps the state of one run; ``collect_on_device`` wires it to the GPU. The B200
is the only GPU this library's kernels run on, so it is the only label accepted without
``allow_unlisted_gpu``.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import re
import time
import uuid
from collections.abc import Callable, Mapping, Sequence
from dataclasses import dataclass, field
from pathlib import Path
from typing import Any

from heliostune_b200.action_collection import BANKS, bank_order, protocol, select_finalists
from heliostune_b200.action_configs import action_set_manifest
from heliostune_b200.configs import DEFAULT_WORKLOADS, Workload
from heliostune_b200.errors import ArtifactError, ProtocolError

RUN_ID_PATTERN = re.compile(r"[a-z0-9][a-z0-9._-]{0,63}")
RUNNERS = ("modal", "local")
#: The pilot's M values: one workload (the largest K, then N) at each (action_collection.py:31).
PILOT_M = (1, 7, 31, 1024)
#: GPU labels with a hardware check (``kernel.require_b200``).
LISTED_GPUS = ("B200",)
#: Fields a resumed checkpoint must match exactly (action_collection.py:42-51).
IDENTITY_FIELDS = ("run", "pilot", "plan_commit", "hardware", "software", "precision", "protocol", "action_set")

_HEX40 = re.compile(r"[0-9a-f]{40}")
_HEX64 = re.compile(r"[0-9a-f]{64}")

Measure = Callable[[int, int, Workload, "frozenset[str] | None"], list[dict[str, Any]]]


@dataclass(frozen=True, slots=True)
class RunSpec:
    """The identity of one collection, fixed before any GPU work."""

    run_id: str
    runner: str
    gpu: str
    pilot: bool
    source_commit: str
    plan_commit: str
    collector_sha256: str
    source_sha256: str
    allow_unlisted_gpu: bool = False

    def __post_init__(self) -> None:
        if not isinstance(self.run_id, str) or RUN_ID_PATTERN.fullmatch(self.run_id) is None:
            raise ProtocolError(
                "run ID must be 1-64 characters of lowercase letters, digits, '.', '_' or '-', "
                f"starting with a letter or digit; got {self.run_id!r}"
            )
        if self.runner not in RUNNERS:
            raise ProtocolError(f"runner must be one of {RUNNERS}, got {self.runner!r}")
        if not isinstance(self.gpu, str) or not self.gpu.strip():
            raise ProtocolError("GPU label must be a nonblank string")
        if type(self.pilot) is not bool or type(self.allow_unlisted_gpu) is not bool:
            raise ProtocolError("pilot and allow_unlisted_gpu must be booleans")
        if self.gpu not in LISTED_GPUS and not self.allow_unlisted_gpu:
            raise ProtocolError(
                f"GPU {self.gpu!r} has no hardware check ({', '.join(LISTED_GPUS)}); pass "
                "allow_unlisted_gpu to bind the run to its observed profile instead"
            )
        for name, pattern, what in (
            ("source_commit", _HEX40, "a full 40-character commit hash"),
            ("plan_commit", _HEX40, "a full 40-character commit hash"),
            ("collector_sha256", _HEX64, "a 64-character SHA-256 digest"),
            ("source_sha256", _HEX64, "a 64-character SHA-256 digest"),
        ):
            if not isinstance(getattr(self, name), str) or pattern.fullmatch(getattr(self, name)) is None:
                raise ProtocolError(f"{name} must be {what}")

    @property
    def validates_hardware(self) -> bool:
        return self.gpu in LISTED_GPUS

    def record(self) -> dict[str, str]:
        return {
            "run_id": self.run_id,
            "runner": self.runner,
            "gpu": self.gpu,
            "hardware_validation": "registry expectation" if self.validates_hardware else "unlisted GPU label",
        }


def collection_workloads(pilot: bool) -> tuple[Workload, ...]:
    """The 96 named workloads, or for the pilot the largest-K (then N) workload at each pilot M."""
    if not pilot:
        return DEFAULT_WORKLOADS
    return tuple(max((w for w in DEFAULT_WORKLOADS if w.m == m), key=lambda w: (w.k, w.n)) for m in PILOT_M)


def dumps_strict(value: object, *, compact: bool = False) -> str:
    """JSON without NaN or infinity: compact for checkpoints, indented and key-sorted for
    artifacts (the reference's serialisation, tooling/artifacts.py:93-99)."""
    try:
        if compact:
            return json.dumps(value, allow_nan=False, separators=(",", ":"))
        return json.dumps(value, allow_nan=False, indent=2, sort_keys=True) + "\n"
    except (TypeError, ValueError) as exc:
        raise ArtifactError(f"value is not strict JSON: {exc}") from exc


def _reject_constant(name: str) -> object:
    raise ArtifactError(f"non-finite JSON constant {name}")


def loads_strict(text: str, source: Path) -> object:
    try:
        return json.loads(text, parse_constant=_reject_constant)
    except json.JSONDecodeError as exc:
        raise ArtifactError(f"{source}: invalid JSON at line {exc.lineno}: {exc.msg}") from exc


def write_atomic(path: Path, payload: str) -> None:
    """Write through a temporary file in the same directory, then rename over ``path``."""
    path.parent.mkdir(parents=True, exist_ok=True)
    temporary = path.with_name(f".{path.name}.{os.getpid()}.tmp")
    try:
        with open(temporary, "w", encoding="utf-8") as stream:
            stream.write(payload)
            stream.flush()
            os.fsync(stream.fileno())
        os.replace(temporary, path)
    except OSError as exc:
        temporary.unlink(missing_ok=True)
        raise ArtifactError(f"cannot write {path}: {exc}") from exc


@dataclass
class Collection:
    """One run's artifact, the units already measured and where its checkpoint lives."""

    data: dict[str, Any]
    workloads: tuple[Workload, ...]
    checkpoint: Path
    completed: set[tuple[int, str]] = field(default_factory=set)

    @classmethod
    def fresh(
        cls,
        spec: RunSpec,
        checkpoint: Path,
        hardware: Mapping[str, Any],
        versions: Mapping[str, str],
        precision: Mapping[str, Any],
    ) -> Collection:
        data: dict[str, Any] = {
            "schema_version": 1,
            "run": spec.record(),
            "plan_commit": spec.plan_commit,
            "source_commit": spec.source_commit,
            "pilot": spec.pilot,
            "hardware": dict(hardware),
            "software": {**versions, "source_sha256": spec.source_sha256, "collector_sha256": spec.collector_sha256},
            "precision": dict(precision),
            "protocol": protocol(),
            "action_set": action_set_manifest(),
            "rows": [],
            "selected": {},
            "duration_seconds": 0.0,
            "sessions": [],
        }
        return cls(data, collection_workloads(spec.pilot), checkpoint)

    def resume(self) -> Collection:
        """Continue from the checkpoint when one exists; every identity field must match."""
        if not self.checkpoint.exists():
            return self
        saved = loads_strict(self.checkpoint.read_text(encoding="utf-8"), self.checkpoint)
        if not isinstance(saved, dict) or set(saved) != {"data", "completed_units"}:
            raise ProtocolError(f"{self.checkpoint} is not a collection checkpoint")
        data = saved["data"]
        if not isinstance(data, dict):
            raise ProtocolError(f"{self.checkpoint} has no checkpoint data")
        for name in IDENTITY_FIELDS:
            if data.get(name) != self.data[name]:
                raise ProtocolError(
                    f"checkpoint {self.checkpoint} differs in {name}; use a new run ID instead of mixing experiments"
                )
        planned = self.planned_units()
        completed = {(int(bank), str(key)) for bank, key in saved["completed_units"]}
        if not completed <= planned:
            raise ProtocolError(f"checkpoint {self.checkpoint} records units outside this run's plan")
        if {(int(r["bank"]), str(r["workload_key"])) for r in data["rows"]} != completed:
            raise ProtocolError(f"checkpoint {self.checkpoint} rows do not match its completed units")
        return Collection(data, self.workloads, self.checkpoint, completed)

    def planned_units(self) -> set[tuple[int, str]]:
        return {(bank, w.key) for bank in BANKS for w in self.workloads}

    @property
    def complete(self) -> bool:
        return self.planned_units() <= self.completed

    def save(self) -> None:
        units = sorted([bank, key] for bank, key in self.completed)
        write_atomic(self.checkpoint, dumps_strict({"data": self.data, "completed_units": units}, compact=True))

    def run(
        self,
        measure: Measure,
        *,
        session: Mapping[str, Any],
        clock: Callable[[], float] = time.monotonic,
        log: Callable[[str], None] = print,
        after_save: Callable[[], None] = lambda: None,
    ) -> dict[str, Any]:
        """Measure every unit not yet completed, bank 1 before bank 2, checkpointing after each.

        Bank 1 times every applicable action and records the old/new finalists; bank 2 times
        torch and those finalists only. The session records its units and duration."""
        started = clock()
        record = {**session, "units": [], "duration_seconds": 0.0}
        self.data["sessions"].append(record)
        before = float(self.data["duration_seconds"])
        for bank in BANKS:
            order = bank_order(self.workloads, bank)
            for index, workload in enumerate(order):
                if (bank, workload.key) in self.completed:
                    continue
                finalists = None
                if bank != 1:
                    finalists = frozenset(k for k in self.data["selected"][workload.key].values() if k)
                rows = measure(bank, index, workload, finalists)
                self.data["rows"].extend(rows)
                if bank == 1:
                    self.data["selected"][workload.key] = select_finalists(rows)
                record["units"].append([bank, workload.key])
                record["duration_seconds"] = clock() - started
                self.data["duration_seconds"] = before + record["duration_seconds"]
                self.completed.add((bank, workload.key))
                self.save()
                after_save()
                log(f"bank={bank} completed={index + 1}/{len(order)} workload={workload.key}")
        return self.data


def collect_on_device(
    spec: RunSpec,
    checkpoint: Path,
    *,
    warmup_ms: float | None = None,
    rep_ms: float | None = None,
    log: Callable[[str], None] = print,
) -> dict[str, Any]:
    """Run or resume one collection on the current CUDA device with ``measure_unit``."""
    import importlib.metadata

    import torch

    from heliostune_b200 import _native
    from heliostune_b200.action_collection import REP_MS, WARMUP_MS
    from heliostune_b200.action_expansion import measure_unit
    from heliostune_b200.kernel import get_hardware_profile, require_b200

    device = torch.device("cuda", torch.cuda.current_device())
    _native.library()
    hardware = get_hardware_profile(spec.gpu, device)
    if spec.validates_hardware:
        require_b200(hardware)
    versions = {name: importlib.metadata.version(name) for name in ("torch", "numpy")}
    versions["libheliostune_b200"] = hashlib.sha256(_native.LIBRARY_PATH.read_bytes()).hexdigest()
    precision = {
        "allow_tf32": torch.backends.cuda.matmul.allow_tf32,
        "allow_fp16_reduced_precision_reduction": torch.backends.cuda.matmul.allow_fp16_reduced_precision_reduction,
        "float32_matmul_precision": torch.get_float32_matmul_precision(),
    }
    collection = Collection.fresh(spec, checkpoint, hardware.to_dict(), versions, precision).resume()
    if collection.complete:
        return collection.data
    session = {"id": str(uuid.uuid4()), "runner": spec.runner, "source_commit": spec.source_commit, "hardware": hardware.to_dict()}

    def measure(bank: int, index: int, workload: Workload, finalists: frozenset[str] | None) -> list[dict[str, Any]]:
        return measure_unit(
            bank,
            index,
            workload,
            finalists,
            device=device,
            warmup_ms=WARMUP_MS if warmup_ms is None else warmup_ms,
            rep_ms=REP_MS if rep_ms is None else rep_ms,
        )

    return collection.run(measure, session=session, log=log)


def source_sha256(package: Path) -> str:
    """Digest of the package's files (path and content of each, in sorted order)."""
    digest = hashlib.sha256()
    for path in sorted(p for p in package.rglob("*") if p.is_file() and "__pycache__" not in p.parts and p.suffix != ".so"):
        digest.update(f"heliostune_b200/{path.relative_to(package).as_posix()}".encode())
        digest.update(b"\0")
        digest.update(hashlib.sha256(path.read_bytes()).digest())
    return digest.hexdigest()


def main(argv: Sequence[str] | None = None) -> None:
    """``python -m heliostune_b200.collection --run-id ID --out FILE [--pilot]`` on a GPU."""
    import subprocess

    parser = argparse.ArgumentParser(description="Collect raw rows in the reference's artifact format")
    parser.add_argument("--run-id", required=True)
    parser.add_argument("--out", required=True, type=Path)
    parser.add_argument("--checkpoint-dir", type=Path, default=None)
    parser.add_argument("--pilot", action="store_true")
    parser.add_argument("--runner", default="local", choices=RUNNERS)
    parser.add_argument("--warmup-ms", type=float, default=None)
    parser.add_argument("--rep-ms", type=float, default=None)
    args = parser.parse_args(argv)
    package = Path(__file__).resolve().parent
    try:
        head = subprocess.run(["git", "rev-parse", "HEAD"], cwd=package, capture_output=True, text=True, check=True).stdout.strip()
    except (OSError, subprocess.CalledProcessError):
        head = "0" * 40  # a checkout without git history
    spec = RunSpec(
        run_id=args.run_id,
        runner=args.runner,
        gpu="B200",
        pilot=args.pilot,
        source_commit=head,
        plan_commit=head,
        collector_sha256=hashlib.sha256(Path(__file__).read_bytes()).hexdigest(),
        source_sha256=source_sha256(package),
    )
    root = args.checkpoint_dir or args.out.parent / "checkpoints"
    checkpoint = root / spec.run_id / ("pilot" if spec.pilot else "full") / "checkpoint.json"
    data = collect_on_device(spec, checkpoint, warmup_ms=args.warmup_ms, rep_ms=args.rep_ms)
    write_atomic(args.out, dumps_strict(data))


if __name__ == "__main__":
    main()
