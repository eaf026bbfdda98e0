"""The offline replay of the probe loop (``heliostune_b200.replay``): table validation, the
reference's evaluation rule (bank 1 picks, bank 2 scores), equivalence with exhaustive search once
the budget covers every candidate, and the B200 feature basis's columns."""

from __future__ import annotations

import hashlib
import math

import numpy as np
import pytest

from heliostune_b200.action_configs import PAIR_DEEP_K_STREAM_K, PAIR_SPLIT2, PAIR_WIDE, ActionCandidate, SplitKConfig, StreamConfig
from heliostune_b200.bandit import BayesianLinearBandit
from heliostune_b200.configs import GRID_WORKLOADS, Workload
from heliostune_b200.features import B200_FEATURE_NAMES, V2_FEATURE_NAMES, b200_joint_features, launch_shape, v2_joint_features
from heliostune_b200.replay import TimingTable, bandit_curve, compare_feature_bases, random_curve, replay_candidates_for
from heliostune_b200.schema import B200_PROFILE
from tests.conftest import load_golden


def _noise(*parts: object) -> float:
    return int.from_bytes(hashlib.sha256("|".join(map(str, parts)).encode()).digest()[:4], "big") / 2.0**32


def _synthetic_table(workloads=GRID_WORKLOADS, unusable: frozenset[str] = frozenset()) -> dict:
    latency = {}
    for w in workloads:
        cells = {}
        for c in replay_candidates_for(w):
            base = w.flops / 1e15 * 1e3 * (1.0 + 3.0 * _noise("speed", w.key, c.key)) + 0.005
            cells[c.key] = [None] * 3 if c.key in unusable else [base * (1 + 0.02 * _noise(b, w.key, c.key)) for b in range(3)]
        latency[w.key] = cells
    return {"hardware": B200_PROFILE.to_dict(), "workloads": [w.to_dict() for w in workloads], "latency_ms": latency}


def test_table_cells_must_be_the_replay_candidates() -> None:
    data = _synthetic_table(GRID_WORKLOADS[:3])
    TimingTable.from_dict(data)
    first = GRID_WORKLOADS[0].key
    data["latency_ms"][first].pop(next(iter(data["latency_ms"][first])))
    with pytest.raises(ValueError, match="differ from the replay candidates"):
        TimingTable.from_dict(data)


def test_candidate_universe_spans_the_families() -> None:
    sizes = {w.m: len(replay_candidates_for(w)) for w in GRID_WORKLOADS}
    assert min(sizes.values()) > 8  # more candidates than the eight probes at every M
    families = {c.family for w in GRID_WORKLOADS for c in replay_candidates_for(w)}
    assert families == {"tile", "persistent", "split_k", "stream", "pair"}
    small = replay_candidates_for(Workload(4, 4096, 4096, "x", "y", "z"))
    assert {c.family for c in small} == {"tile", "persistent", "split_k", "stream"}
    large = replay_candidates_for(Workload(8192, 4096, 4096, "x", "y", "z"))
    assert {c.family for c in large} == {"tile", "persistent", "pair"}


def test_full_budget_equals_exhaustive_search() -> None:
    table = TimingTable.from_dict(_synthetic_table(GRID_WORKLOADS[:12]))
    workloads = table.workloads
    budget = max(len(table.usable(w)) for w in workloads)
    orders = [workloads] * budget
    model = BayesianLinearBandit(dimension=len(B200_FEATURE_NAMES), noise_variance=0.05, prior_precision=1.0, seed=3)
    curve = bandit_curve(table, workloads, orders, model, b200_joint_features)
    exhaustive = math.exp(
        np.mean([math.log(table.heldout_fraction(w, min(table.usable(w), key=lambda c, w=w: (table.get(w, c, 0), c.key)))) for w in workloads])
    )
    assert curve[-1] == pytest.approx(exhaustive, rel=1e-12)
    assert random_curve(table, workloads, orders, 5)[-1] == pytest.approx(exhaustive, rel=1e-12)
    assert all(0 < v <= 1.0 + 0.05 for v in curve)


def test_unusable_cells_are_never_probed_or_recommended() -> None:
    broken = frozenset({PAIR_WIDE.key})
    table = TimingTable.from_dict(_synthetic_table(GRID_WORKLOADS[-12:], unusable=broken))
    for w in table.workloads:
        assert PAIR_WIDE.key not in {c.key for c in table.usable(w)}
    result = compare_feature_bases(table, budget=4, seeds=2)
    assert set(result["auc"]) == {"random", "cold_thompson_v2", "cold_thompson_b200"}
    assert len(result["methods"]["cold_thompson_b200"]) == 4
    assert result["families"] == sorted({w.model for w in table.workloads})


def test_b200_columns() -> None:
    w = Workload(512, 4096, 4096, "x", "y", "z")
    plain = ActionCandidate(PAIR_SPLIT2.config.__class__(256, 256, 64, 4, 6, 8))
    v2 = [v2_joint_features(w, c.config, B200_PROFILE) for c in (plain, PAIR_SPLIT2)]
    b2 = [dict(zip(B200_FEATURE_NAMES, b200_joint_features(w, c.config, B200_PROFILE), strict=True)) for c in (plain, PAIR_SPLIT2, PAIR_DEEP_K_STREAM_K)]
    assert np.array_equal(v2[0], v2[1])  # a split pair tile looks the same as the plain one to v2
    assert np.array_equal(b200_joint_features(w, plain.config, B200_PROFILE)[: len(V2_FEATURE_NAMES)], v2[0])
    # 2 x 16 tiles of 256 x 256: 32 of 74 pairs busy; split over two pairs each: 32 of 33 clusters of four
    assert b2[0]["wave_fill"] == pytest.approx(32 / 74) and b2[1]["wave_fill"] == pytest.approx(32 / 33)
    assert b2[2]["wave_fill"] == 1.0  # stream-K shares the part-filled wave out along K
    assert b2[0]["log_roofline_tflops"] == b2[1]["log_roofline_tflops"] == b2[2]["log_roofline_tflops"]
    small, large = Workload(1, 4096, 4096, "x", "y", "z"), Workload(8192, 4096, 4096, "x", "y", "z")
    roof = [dict(zip(B200_FEATURE_NAMES, b200_joint_features(v, plain.config, B200_PROFILE), strict=True))["log_roofline_tflops"] for v in (small, large)]
    assert roof[0] < roof[1]  # a weight-streaming shape is HBM-bound, far below the tensor peak
    assert launch_shape(small, StreamConfig(16, 128, 64, 4, 4, 0), 148).family == "stream"
    assert launch_shape(small, SplitKConfig(16, 128, 64, 4, 3, 16), 148).splits == 16
    with pytest.raises(TypeError):
        launch_shape(small, object(), 148)


def test_replay_on_the_b200_table() -> None:
    """Cold Thompson on the committed B200 timing table (tests/golden/b200_grid_timings.json, made
    by ``python -m heliostune_b200.replay collect`` on a B200): both bases find within 0.5% of the
    exhaustive pick in 8 probes among 9-21 candidates, far above random search, and the B200
    basis does at least as well as v2 over the probe budgets."""
    table = TimingTable.from_dict(load_golden("b200_grid_timings.json"))
    result = compare_feature_bases(table, seeds=10)
    assert result["candidates_per_workload"] == {"min": 9, "max": 21}
    assert result["methods"]["exhaustive"][0]["mean_fraction_oracle"] > 0.999
    at8, auc = result["at_budget"], result["auc"]
    assert at8["cold_thompson_b200"] >= 0.995 and at8["cold_thompson_v2"] >= 0.995
    assert at8["random"] < 0.98 and auc["random"] < 0.9
    assert auc["cold_thompson_b200"] >= auc["cold_thompson_v2"]
    assert result["queries_to_95_percent"]["cold_thompson_b200"] <= result["queries_to_95_percent"]["cold_thompson_v2"]
