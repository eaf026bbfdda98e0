"""Live Thompson-sampling probe loop over the B200 variants.

Restates the reference's cold-Thompson probing (``src/heliostune/replay.py:423-453``, same loop
as ``multisource_engine.py:335-364``) with one change: a probe is a real timed launch on this
GPU instead of a lookup in a stored bank-0 timing table.

* One posterior is shared by every workload of the run.
* Budget round ``b = 1..budget`` visits the workloads in a permutation drawn from
  ``numpy.random.default_rng(policy_seed + 50_000)`` (``replay.py:608-615``).
* For each workload the bandit chooses among the candidates not yet probed for it (earliest
  candidate wins a tie), the candidate is measured, and the posterior is updated with the
  reward ``ln TFLOP/s`` (``retrieval.py:98-112``).
* The recommendation for a workload is its best observed candidate: minimum probe latency,
  then key (``replay.py:283-297``).

Failure containment (not needed by the reference's table replay): a candidate whose launch
raises or whose output fails the parity check gets no reward, is recorded, and is never offered
again for that workload.
"""

from __future__ import annotations

from collections.abc import Callable, Sequence
from dataclasses import dataclass, field
from functools import partial
from typing import Any

import numpy as np

from heliostune_b200.action_configs import ActionCandidate
from heliostune_b200.bandit import BayesianLinearBandit
from heliostune_b200.configs import Workload
from heliostune_b200.features import FEATURE_BASES
from heliostune_b200.retrieval import log_tflops_reward
from heliostune_b200.schema import HardwareProfile

#: Hyperparameters of the reference's replay comparison (``replay.py:494-495``).
NOISE_VARIANCE = 0.05
PRIOR_PRECISION = 1.0
DEFAULT_BUDGET = 8
ORDER_SEED_OFFSET = 50_000


@dataclass
class Probe:
    candidate: ActionCandidate
    latency_ms: float | None
    error: str | None = None


@dataclass
class ProbeResult:
    probes: dict[str, list[Probe]] = field(default_factory=dict)
    recommendations: dict[str, ActionCandidate] = field(default_factory=dict)

    def to_dict(self) -> dict[str, Any]:
        return {
            key: {
                "recommendation": self.recommendations[key].key if key in self.recommendations else None,
                "probes": [
                    {"candidate": p.candidate.key, "latency_ms": p.latency_ms, "error": p.error}
                    for p in probes
                ],
            }
            for key, probes in self.probes.items()
        }


def probe_orders(workloads: Sequence[Workload], budget: int, policy_seed: int) -> list[tuple[Workload, ...]]:
    """One seeded permutation of the workloads per budget round."""
    rng = np.random.default_rng(policy_seed + ORDER_SEED_OFFSET)
    return [tuple(workloads[i] for i in rng.permutation(len(workloads))) for _ in range(budget)]


def best_observed(probes: Sequence[Probe]) -> ActionCandidate | None:
    valid = [p for p in probes if p.latency_ms is not None]
    if not valid:
        return None
    return min(valid, key=lambda p: (p.latency_ms, p.candidate.key)).candidate


def thompson_probe(
    workloads: Sequence[Workload],
    candidates_for: Callable[[Workload], Sequence[ActionCandidate]],
    measure: Callable[[Workload, ActionCandidate], float],
    hardware: HardwareProfile,
    *,
    budget: int = DEFAULT_BUDGET,
    policy_seed: int = 0,
    noise_variance: float = NOISE_VARIANCE,
    prior_precision: float = PRIOR_PRECISION,
    model: BayesianLinearBandit | None = None,
    basis: str = "v2",
) -> ProbeResult:
    """Probe ``budget`` candidates per workload with one shared Thompson-sampling posterior.

    ``measure`` returns the latency in milliseconds of one candidate on one workload and raises
    to report a failure. ``basis`` is the feature basis: the reference's ``"v2"`` or ``"b200"``
    (v2 plus the shape's roofline throughput and the launch's wave fill).
    """
    names, feature_fn = FEATURE_BASES[basis]
    if model is None:
        model = BayesianLinearBandit(
            dimension=len(names),
            noise_variance=noise_variance,
            prior_precision=prior_precision,
            seed=policy_seed,
        )
    result = ProbeResult(probes={w.key: [] for w in workloads})
    excluded: dict[str, set[str]] = {w.key: set() for w in workloads}
    for order in probe_orders(workloads, budget, policy_seed):
        for workload in order:
            tried = excluded[workload.key]
            available = tuple(c for c in candidates_for(workload) if c.key not in tried)
            if not available:
                continue
            features = partial(_features, feature_fn, workload, hardware)
            selected = model.choose(available, features)
            tried.add(selected.key)
            try:
                latency = float(measure(workload, selected))
            except Exception as exc:  # noqa: BLE001 -- contained per candidate
                result.probes[workload.key].append(Probe(selected, None, f"{type(exc).__name__}: {exc}"))
                continue
            result.probes[workload.key].append(Probe(selected, latency))
            model.update(features(selected), log_tflops_reward(workload, latency))
    for workload in workloads:
        best = best_observed(result.probes[workload.key])
        if best is not None:
            result.recommendations[workload.key] = best
    return result


def _features(feature_fn, workload: Workload, hardware: HardwareProfile, candidate: ActionCandidate) -> np.ndarray:  # type: ignore[no-untyped-def]
    return feature_fn(workload, candidate.config, hardware)
