"""The raw-row collector (``heliostune_b200.collection``) without a GPU: its artifact is the one
the reference's analysis script accepted (tests/golden/collection_analysis.json, recorded by
make_golden.py), checkpoints resume to the same rows, and run identities are enforced."""

from __future__ import annotations

import hashlib
import json
from pathlib import Path

import pytest

from heliostune_b200.collection import Collection, RunSpec, collection_workloads, dumps_strict
from heliostune_b200.errors import ProtocolError
from heliostune_b200.schema import B200_PROFILE
from tests.conftest import load_golden
from tests.golden.collection_fixture import SPEC, build, fake_measure


def test_artifact_is_the_one_the_reference_analysis_scored(tmp_path: Path) -> None:
    data = build(tmp_path)
    golden = load_golden("collection_analysis.json")
    assert hashlib.sha256(dumps_strict(data).encode()).hexdigest() == golden["artifact_sha256"]
    # the analysis's per-workload selection is the collector's bank-1 finalist record
    for key, arms in golden["selected"].items():
        assert arms["old"]["config_key"] == data["selected"][key]["old"]
        assert arms["new"]["config_key"] == data["selected"][key]["new"]
    assert golden["failure_row_count"] == sum(not r["correct"] for r in data["rows"])


def test_bank_two_times_torch_and_the_finalists_only(tmp_path: Path) -> None:
    data = build(tmp_path)
    for workload in collection_workloads(True):
        bank2 = {r["config_key"] for r in data["rows"] if r["bank"] == 2 and r["workload_key"] == workload.key}
        finalists = {k for k in data["selected"][workload.key].values() if k}
        assert bank2 == {"torch", *finalists}
    checkpoint = json.loads((tmp_path / "checkpoint.json").read_text())
    assert set(checkpoint) == {"data", "completed_units"}
    assert len(checkpoint["completed_units"]) == 2 * len(collection_workloads(True))


def _fresh(directory: Path, spec: RunSpec = SPEC, hardware: dict | None = None) -> Collection:
    return Collection.fresh(
        spec,
        directory / "checkpoint.json",
        hardware or B200_PROFILE.to_dict(),
        {"torch": "fixture", "numpy": "fixture"},
        {"allow_tf32": False, "allow_fp16_reduced_precision_reduction": True, "float32_matmul_precision": "highest"},
    )


def test_an_interrupted_run_resumes_to_the_same_rows(tmp_path: Path) -> None:
    whole = build(tmp_path / "whole")
    calls = {"n": 0}

    def dies_after_three(*args):  # type: ignore[no-untyped-def]
        if calls["n"] == 3:
            raise RuntimeError("session lost")
        calls["n"] += 1
        return fake_measure(*args)

    session = {"id": "first", "runner": "local", "source_commit": SPEC.source_commit, "hardware": B200_PROFILE.to_dict()}
    with pytest.raises(RuntimeError, match="session lost"):
        _fresh(tmp_path / "split").run(dies_after_three, session=session, log=lambda _m: None)
    resumed = _fresh(tmp_path / "split").resume()
    assert len(resumed.completed) == 3 and not resumed.complete
    data = resumed.run(fake_measure, session={**session, "id": "second"}, log=lambda _m: None)
    assert data["rows"] == whole["rows"] and data["selected"] == whole["selected"]
    assert [s["id"] for s in data["sessions"]] == ["first", "second"]
    assert [len(s["units"]) for s in data["sessions"]] == [3, 2 * len(collection_workloads(True)) - 3]
    assert _fresh(tmp_path / "split").resume().complete


def test_a_checkpoint_of_another_experiment_is_refused(tmp_path: Path) -> None:
    build(tmp_path)
    other_hardware = {**B200_PROFILE.to_dict(), "multiprocessor_count": 132}
    with pytest.raises(ProtocolError, match="differs in hardware"):
        _fresh(tmp_path, hardware=other_hardware).resume()
    (tmp_path / "checkpoint.json").write_text('{"data": {}}')
    with pytest.raises(ProtocolError, match="not a collection checkpoint"):
        _fresh(tmp_path).resume()


def test_run_identity_is_validated() -> None:
    base = {name: getattr(SPEC, name) for name in RunSpec.__dataclass_fields__}
    for change, message in (
        ({"run_id": "Bad ID"}, "run ID"),
        ({"runner": "slurm"}, "runner"),
        ({"gpu": "H100"}, "no hardware check"),
        ({"source_commit": "abc"}, "source_commit"),
        ({"collector_sha256": "0" * 63}, "collector_sha256"),
    ):
        with pytest.raises(ProtocolError, match=message):
            RunSpec(**{**base, **change})
    assert RunSpec(**{**base, "gpu": "H100", "allow_unlisted_gpu": True}).record()["hardware_validation"] == "unlisted GPU label"
    assert [w.m for w in collection_workloads(True)] == [1, 7, 31, 1024]
    assert len(collection_workloads(False)) == 96
