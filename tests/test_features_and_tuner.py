"""Bandit features, reward, collection protocol and the probe loop, checked against values the
reference computed (tests/golden/{features,manifest,bandit_curve}.json)."""

from __future__ import annotations

import hashlib

import numpy as np
import pytest

from heliostune_b200.action_collection import bank_order, protocol, select_finalists, tensor_seed, timing_order
from heliostune_b200.action_configs import ActionCandidate, SplitKConfig, StreamConfig
from heliostune_b200.configs import DEFAULT_CONFIGS, DEFAULT_WORKLOADS, GRID_WORKLOADS, KernelConfig
from heliostune_b200.features import V2_FEATURE_NAMES, launch_fields, v2_joint_features
from heliostune_b200.errors import ProtocolError
from heliostune_b200.retrieval import log_tflops_reward
from heliostune_b200.schema import B200_PROFILE, HardwareProfile
from heliostune_b200.tuner import probe_orders, thompson_probe
from tests.conftest import GOLDEN, load_golden


def _profiles() -> list[HardwareProfile]:
    return [HardwareProfile.from_dict(p) for p in load_golden("features.json")["profiles"]]


def test_v2_features_equal_the_reference_bit_for_bit() -> None:
    golden = load_golden("features.json")
    assert list(V2_FEATURE_NAMES) == golden["names"]
    full = np.stack(
        [v2_joint_features(w, c, p) for p in _profiles() for w in DEFAULT_WORKLOADS for c in DEFAULT_CONFIGS]
    )
    assert list(full.shape) == golden["shape"]
    assert hashlib.sha256(full.astype("<f8").tobytes()).hexdigest() == golden["sha256"]
    sample = np.load(GOLDEN / "features.npz")
    np.testing.assert_array_equal(full[sample["rows"]], sample["values"])


def test_every_family_maps_onto_the_v2_fields() -> None:
    w = GRID_WORKLOADS[0]
    assert launch_fields(w, SplitKConfig(16, 64, 64, 4, 3, 16), B200_PROFILE).group_m == 16
    stream = launch_fields(w, StreamConfig(16, 128, 64, 4, 8, 0), B200_PROFILE)
    assert stream.group_m >= 1
    for config in (SplitKConfig(16, 64, 64, 4, 3, 16), StreamConfig(16, 128, 64, 4, 8, 0)):
        x = v2_joint_features(w, config, B200_PROFILE)
        assert x.shape == (25,) and np.all(np.isfinite(x))


def test_reward_matches_the_reference() -> None:
    by_key = {w.key: w for w in DEFAULT_WORKLOADS}
    for key, latency, expected in load_golden("manifest.json")["rewards"]:
        assert log_tflops_reward(by_key[key], latency) == expected
    with pytest.raises(ValueError):
        log_tflops_reward(DEFAULT_WORKLOADS[0], 0.0)


def test_collection_protocol_matches_the_reference() -> None:
    golden = load_golden("manifest.json")
    by_key = {w.key: w for w in DEFAULT_WORKLOADS}
    for bank, keys in golden["bank_orders"].items():
        assert [w.key for w in bank_order(DEFAULT_WORKLOADS, int(bank))] == keys
    for case in golden["timing_orders"]:
        finalists = frozenset(case["finalists"]) if "finalists" in case else None
        order = timing_order(case["bank"], case["index"], by_key[case["workload"]], finalists)
        assert order == case["order"]
        assert tensor_seed(case["bank"], case["index"]) == case["seed"]
    assert select_finalists(golden["finalist_rows"]) == golden["finalists"]
    assert protocol()["atol"] == golden["protocol"]["atol"] == 1e-2
    assert protocol()["tensor_seed"] == golden["protocol"]["tensor_seed"]


def test_probe_loop_reproduces_the_reference_replay() -> None:
    """Fed the reference's synthetic latency table, the live loop probes the same configurations
    in the same order as replay._bandit_curve did."""
    golden = load_golden("bandit_curve.json")
    by_key = {w.key: w for w in DEFAULT_WORKLOADS}
    workloads = tuple(by_key[k] for k in golden["workloads"])
    configs = {c.key: c for c in DEFAULT_CONFIGS}
    candidates = tuple(ActionCandidate(configs[k]) for k in golden["configs"])
    latency = golden["latency_bank0"]
    calls: list[list[str]] = []

    def measure(workload, candidate):  # type: ignore[no-untyped-def]
        calls.append([workload.key, candidate.config.key])
        return latency[f"{workload.key}|{candidate.config.key}"]

    hardware = _profiles()[1]
    result = thompson_probe(workloads, lambda _w: candidates, measure, hardware, budget=8, policy_seed=golden["policy_seed"])
    assert calls == golden["probes"]
    for w in workloads:
        probes = result.probes[w.key]
        best = min(probes, key=lambda p: (p.latency_ms, p.candidate.key))
        assert result.recommendations[w.key] == best.candidate


def test_probe_loop_contains_failures() -> None:
    workloads = GRID_WORKLOADS[:3]
    good = ActionCandidate(KernelConfig(128, 128, 64, 4, 5))
    bad = ActionCandidate(KernelConfig(64, 64, 64, 4, 2))

    def measure(workload, candidate):  # type: ignore[no-untyped-def]
        if candidate == bad:
            raise RuntimeError("launch failed")
        return 1.0

    result = thompson_probe(workloads, lambda _w: (good, bad), measure, B200_PROFILE, budget=4)
    for w in workloads:
        assert [p.candidate for p in result.probes[w.key]].count(bad) == 1
        assert result.recommendations[w.key] == good


def test_probe_orders_are_seeded_permutations() -> None:
    orders = probe_orders(GRID_WORKLOADS, 3, 7)
    assert len(orders) == 3
    for order in orders:
        assert sorted(w.key for w in order) == sorted(w.key for w in GRID_WORKLOADS)
    assert orders == probe_orders(GRID_WORKLOADS, 3, 7)


def test_b200_hardware_check() -> None:
    from dataclasses import replace

    from heliostune_b200.kernel import require_b200

    require_b200(B200_PROFILE)
    with pytest.raises(ProtocolError, match="compute capability"):
        require_b200(replace(B200_PROFILE, device_name="NVIDIA H200", compute_capability=(9, 0)))
    with pytest.raises(ProtocolError, match="not a B200"):
        require_b200(replace(B200_PROFILE, device_name="NVIDIA GB300"))
