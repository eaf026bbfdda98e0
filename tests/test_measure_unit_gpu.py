"""The per-unit measurement protocol (``action_expansion.measure_unit``) on the GPU, against the
reference's row format and order (src/heliostune/action_expansion.py:188-273).

Two small units run with short timing windows: every row has exactly the reference's keys, the
rows come in the protocol's order (torch first, then the seeded shuffle of the 36 stock tile
configurations and the frozen candidates), every variant is correct within the unchanged
1e-2/1e-2 tolerance and timed, and a variant that fails stays a row with its stage and message
while the other rows are still measured."""

from __future__ import annotations

import pytest
import torch

from heliostune_b200 import _native, action_expansion
from heliostune_b200.action_collection import timing_order
from heliostune_b200.configs import Workload
from tests.gpu_helpers import require_cuda

pytestmark = pytest.mark.gpu

#: The keys of a raw row, in the reference's order (action_expansion.py:226-241).
ROW_KEYS = [
    "workload_key", "workload", "bank", "family", "config_key", "config", "correct", "error",
    "p20_ms", "median_ms", "p80_ms", "max_abs_error", "compile_seconds", "timing_seconds",
]

UNITS = (
    (1, 3, Workload(m=7, n=264, k=136, model="test", projection="splitk", regime="m7")),
    (2, 5, Workload(m=96, n=512, k=256, model="test", projection="tile", regime="m96")),
)


@pytest.fixture(autouse=True)
def _cuda() -> None:
    require_cuda()
    _native.library()


@pytest.mark.parametrize("bank, index, workload", UNITS, ids=lambda v: getattr(v, "regime", str(v)))
def test_unit_rows_follow_the_reference_protocol(bank: int, index: int, workload: Workload) -> None:
    device = torch.device("cuda", torch.cuda.current_device())
    rows = action_expansion.measure_unit(bank, index, workload, None, device=device, warmup_ms=1.0, rep_ms=3.0)
    assert [row["config_key"] for row in rows] == timing_order(bank, index, workload, None)
    assert rows[0]["config_key"] == "torch" and rows[0]["family"] == "torch" and rows[0]["config"] is None
    for row in rows:
        assert list(row) == ROW_KEYS
        assert row["workload_key"] == workload.key and row["workload"] == workload.to_dict() and row["bank"] == bank
        assert row["correct"] is True and row["error"] is None, (row["config_key"], row["error"])
        assert 0 < row["p20_ms"] <= row["median_ms"] <= row["p80_ms"]
        assert 0 <= row["max_abs_error"] < 1.0  # within 1e-2 + 1e-2|C| for |C| of a few tens
        assert row["compile_seconds"] >= 0 and row["timing_seconds"] > 0
    families = {row["family"] for row in rows}
    assert {"torch", "old"} <= families
    assert ("split_k" in families) == (workload.m <= 31)


def test_unit_keeps_a_failing_variant_as_a_row(monkeypatch: pytest.MonkeyPatch) -> None:
    bank, index, workload = UNITS[0]
    real_launch = action_expansion.launch

    def failing(a, b, candidate):  # type: ignore[no-untyped-def]
        if candidate.family == "split_k":
            raise RuntimeError("requested kernel failed")
        return real_launch(a, b, candidate)

    monkeypatch.setattr(action_expansion, "launch", failing)
    device = torch.device("cuda", torch.cuda.current_device())
    rows = action_expansion.measure_unit(bank, index, workload, None, device=device, warmup_ms=1.0, rep_ms=2.0)
    failed = [row for row in rows if row["family"] == "split_k"]
    assert failed and all(
        row["correct"] is False
        and row["error"] == "compile: RuntimeError: requested kernel failed"
        and row["median_ms"] is None
        for row in failed
    )
    assert all(row["correct"] for row in rows if row["family"] != "split_k")
    # finalists narrow the unit to the named keys, torch always first
    finalists = frozenset(row["config_key"] for row in rows[1:4])
    narrowed = action_expansion.measure_unit(bank, index, workload, finalists, device=device, warmup_ms=1.0, rep_ms=2.0)
    assert [row["config_key"] for row in narrowed] == timing_order(bank, index, workload, finalists)
    assert narrowed[0]["config_key"] == "torch" and len(narrowed) == 4
