"""Offline replay of the probe loop on B200 timing tables: which feature basis lets the bandit
find the exhaustive pick in fewer probes.

The reference scores its policies by replaying them on stored timing matrices
(``src/heliostune/replay.py:283-297`` best observed, ``:380-400`` random search, ``:425-453``
cold Thompson, ``:486-798`` the comparison): three timing banks per (workload, configuration)
-- bank 0 is all a policy may observe, bank 1 picks the exhaustive reference configuration,
bank 2 scores both -- and a recommendation's value is the bank-2 latency of the bank-1 winner
divided by its own bank-2 latency, a geometric mean over the workloads of a held-out model
family. This module restates that loop for B200 tables:

* :func:`replay_candidates_for` -- the configurations a replay chooses among: every frozen
  candidate of the workload, the weight-streaming variants up to M = 256 and the CTA-pair
  variants from M = 64 (plain, split, stream-K, 128-deep, 256 x 512, 256 x 128). From 9 to 21
  per shape, more than the 8 probes, unlike the tuner's pool which holds at most 8.
* :func:`collect_timing_table` (GPU) -- median latency of every such configuration on every
  workload in three banks of seeded operands, each launch after an L2 flush; a configuration
  whose output fails the parity check is stored as unusable.
* :func:`compare_feature_bases` -- cold Thompson sampling with the v2 basis and with the B200
  basis (``features.b200_joint_features``), random search and exhaustive search, per held-out
  model family over seeded policy runs, as the reference's comparison does.
"""

from __future__ import annotations

import argparse
import json
import math
from collections.abc import Callable, Mapping, Sequence
from dataclasses import dataclass
from functools import partial
from pathlib import Path
from typing import Any

import numpy as np

from heliostune_b200.action_configs import (
    PAIR_CANDIDATES,
    PAIR_DEEP_K,
    PAIR_DEEP_K_STREAM_K,
    PAIR_NARROW,
    PAIR_SPLIT_CANDIDATES,
    PAIR_STREAM_K_CANDIDATE,
    PAIR_WIDE,
    PAIR_WIDE_STREAM_K,
    STREAM_M_LIMIT,
    ActionCandidate,
    _sorted,
    candidates_for,
    stream_candidates_for,
)
from heliostune_b200.bandit import BayesianLinearBandit
from heliostune_b200.configs import GRID_WORKLOADS, Workload
from heliostune_b200.features import FEATURE_BASES
from heliostune_b200.retrieval import log_tflops_reward
from heliostune_b200.schema import HardwareProfile

OBSERVATION_BANK = 0
REFERENCE_BANK = 1
EVALUATION_BANK = 2
BANKS = (OBSERVATION_BANK, REFERENCE_BANK, EVALUATION_BANK)
#: Policy seeds of fold f are f * stride + seed (replay.py:32-39).
PAIRED_SEED_STRIDE = 100_000
#: Smallest M the replay offers CTA-pair tiles for (a 256-row tile is 3/4 empty at M = 64).
REPLAY_PAIR_M_MINIMUM = 64

FeatureFunction = Callable[[Workload, Any, HardwareProfile], np.ndarray]
#: The bases compared by :func:`compare_feature_bases`.
BASES: Mapping[str, tuple[tuple[str, ...], FeatureFunction]] = FEATURE_BASES


def replay_candidates_for(workload: Workload) -> tuple[ActionCandidate, ...]:
    """Every configuration a replay may recommend for ``workload`` (see the module notes)."""
    pairs: tuple[ActionCandidate, ...] = ()
    if workload.m >= REPLAY_PAIR_M_MINIMUM:
        pairs = (
            *PAIR_CANDIDATES,
            *PAIR_SPLIT_CANDIDATES,
            PAIR_STREAM_K_CANDIDATE,
            PAIR_DEEP_K,
            PAIR_DEEP_K_STREAM_K,
            PAIR_WIDE,
            PAIR_WIDE_STREAM_K,
            PAIR_NARROW,
        )
    streams = stream_candidates_for(workload) if workload.m <= STREAM_M_LIMIT else ()
    return _sorted((*candidates_for(workload), *streams, *pairs))


@dataclass(frozen=True)
class TimingTable:
    """Latency in milliseconds per (workload key, configuration key, bank); None = unusable."""

    hardware: HardwareProfile
    workloads: tuple[Workload, ...]
    latency: Mapping[str, Mapping[str, tuple[float | None, float | None, float | None]]]

    @classmethod
    def from_dict(cls, data: Mapping[str, Any]) -> TimingTable:
        workloads = tuple(Workload.from_dict(w) for w in data["workloads"])
        latency: dict[str, dict[str, tuple[float | None, float | None, float | None]]] = {}
        for w in workloads:
            cells = data["latency_ms"][w.key]
            expected = {c.key for c in replay_candidates_for(w)}
            if set(cells) != expected:
                raise ValueError(f"table cells of {w.key} differ from the replay candidates")
            latency[w.key] = {key: tuple(values) for key, values in cells.items()}  # type: ignore[misc]
        return cls(HardwareProfile.from_dict(data["hardware"]), workloads, latency)

    def get(self, workload: Workload, candidate: ActionCandidate, bank: int) -> float | None:
        return self.latency[workload.key][candidate.key][bank]

    def usable(self, workload: Workload) -> tuple[ActionCandidate, ...]:
        """Candidates with a latency in every bank."""
        return tuple(
            c for c in replay_candidates_for(workload) if all(v is not None for v in self.latency[workload.key][c.key])
        )

    def reference(self, workload: Workload) -> ActionCandidate:
        """The exhaustive pick, chosen on bank 1 only (replay.py:203-211)."""
        return min(self.usable(workload), key=lambda c: (self.get(workload, c, REFERENCE_BANK), c.key))

    def heldout_fraction(self, workload: Workload, recommendation: ActionCandidate) -> float:
        """Bank-2 latency of the exhaustive pick over the recommendation's (replay.py:213-223)."""
        return self.get(workload, self.reference(workload), EVALUATION_BANK) / self.get(  # type: ignore[operator]
            workload, recommendation, EVALUATION_BANK
        )


def _geomean(values: Sequence[float]) -> float:
    return math.exp(sum(math.log(v) for v in values) / len(values))


def _best_observed(table: TimingTable, workload: Workload, queried: Sequence[ActionCandidate]) -> ActionCandidate:
    return min(queried, key=lambda c: (table.get(workload, c, OBSERVATION_BANK), c.key))


def _evaluate(table: TimingTable, workloads: Sequence[Workload], queried: Mapping[str, list[ActionCandidate]]) -> float:
    return _geomean([table.heldout_fraction(w, _best_observed(table, w, queried[w.key])) for w in workloads])


def _orders(workloads: Sequence[Workload], budget: int, policy_seed: int) -> list[tuple[Workload, ...]]:
    rng = np.random.default_rng(policy_seed + 50_000)
    return [tuple(workloads[i] for i in rng.permutation(len(workloads))) for _ in range(budget)]


def bandit_curve(
    table: TimingTable,
    workloads: Sequence[Workload],
    orders: Sequence[Sequence[Workload]],
    model: BayesianLinearBandit,
    features: FeatureFunction,
) -> list[float]:
    """Cold or warm Thompson sampling, one shared posterior, the reward ln TFLOP/s of bank 0;
    the value after each budget round (replay.py:425-453)."""
    queried: dict[str, list[ActionCandidate]] = {w.key: [] for w in workloads}
    curve = []
    for order in orders:
        for workload in order:
            available = [c for c in table.usable(workload) if c not in queried[workload.key]]
            if not available:
                continue
            feature = partial(_candidate_features, features, workload, table.hardware)
            selected = model.choose(available, feature)
            queried[workload.key].append(selected)
            model.update(feature(selected), log_tflops_reward(workload, table.get(workload, selected, OBSERVATION_BANK)))
        curve.append(_evaluate(table, workloads, queried))
    return curve


def _candidate_features(features: FeatureFunction, workload: Workload, hardware: HardwareProfile, candidate: ActionCandidate) -> np.ndarray:
    return features(workload, candidate.config, hardware)


def random_curve(table: TimingTable, workloads: Sequence[Workload], orders: Sequence[Sequence[Workload]], seed: int) -> list[float]:
    """Uniform choice among the candidates not yet probed (replay.py:380-400)."""
    rng = np.random.default_rng(seed)
    queried: dict[str, list[ActionCandidate]] = {w.key: [] for w in workloads}
    curve = []
    for order in orders:
        for workload in order:
            available = [c for c in table.usable(workload) if c not in queried[workload.key]]
            if available:
                queried[workload.key].append(available[int(rng.integers(len(available)))])
        curve.append(_evaluate(table, workloads, queried))
    return curve


def _aggregate(runs: Sequence[Sequence[float]]) -> list[dict[str, float | int]]:
    values = np.asarray(runs, dtype=np.float64)
    points = []
    for index in range(values.shape[1]):
        column = values[:, index]
        half = 0.0 if len(column) == 1 else float(1.96 * np.std(column, ddof=1) / math.sqrt(len(column)))
        mean = float(np.mean(column))
        points.append({"budget": index + 1, "mean_fraction_oracle": mean, "ci95_low": mean - half, "ci95_high": mean + half})
    return points


def compare_feature_bases(
    table: TimingTable,
    *,
    budget: int = 8,
    seeds: int = 30,
    noise_variance: float = 0.05,
    prior_precision: float = 1.0,
) -> dict[str, Any]:
    """Cold Thompson with each basis of :data:`BASES`, random search and exhaustive search,
    each workload family held out in turn (replay.py:486-798 without the source GPU)."""
    families = sorted({w.model for w in table.workloads})
    runs: dict[str, list[list[float]]] = {"random": [], **{f"cold_thompson_{name}": [] for name in BASES}}
    exhaustive = []
    for fold, family in enumerate(families):
        workloads = tuple(w for w in table.workloads if w.model == family)
        exhaustive.append(
            _geomean(
                [
                    table.heldout_fraction(
                        w, min(table.usable(w), key=lambda c, w=w: (table.get(w, c, OBSERVATION_BANK), c.key))
                    )
                    for w in workloads
                ]
            )
        )
        for seed in range(seeds):
            policy_seed = fold * PAIRED_SEED_STRIDE + seed
            orders = _orders(workloads, budget, policy_seed)
            runs["random"].append(random_curve(table, workloads, orders, policy_seed))
            for name, (names, features) in BASES.items():
                model = BayesianLinearBandit(
                    dimension=len(names), noise_variance=noise_variance, prior_precision=prior_precision, seed=policy_seed
                )
                runs[f"cold_thompson_{name}"].append(bandit_curve(table, workloads, orders, model, features))
    methods = {name: _aggregate(method_runs) for name, method_runs in runs.items()}
    methods["exhaustive"] = _aggregate([[value] for value in exhaustive])
    auc = {name: float(np.mean([p["mean_fraction_oracle"] for p in points])) for name, points in methods.items() if name != "exhaustive"}
    return {
        "workloads": len(table.workloads),
        "families": families,
        "candidates_per_workload": {
            "min": min(len(table.usable(w)) for w in table.workloads),
            "max": max(len(table.usable(w)) for w in table.workloads),
        },
        "budget": budget,
        "seeds": seeds,
        "methods": methods,
        "auc": auc,
        "at_budget": {name: points[-1]["mean_fraction_oracle"] for name, points in methods.items() if name != "exhaustive"},
        "queries_to_95_percent": {
            name: next((p["budget"] for p in points if p["mean_fraction_oracle"] >= 0.95), None)
            for name, points in methods.items()
            if name != "exhaustive"
        },
    }


def collect_timing_table(
    workloads: Sequence[Workload] = GRID_WORKLOADS,
    *,
    reps: int = 5,
    log: Callable[[str], None] = print,
) -> dict[str, Any]:
    """Time every replay candidate on every workload in the three banks (GPU).

    Bank b's operands are seeded N(0, 1)/sqrt(K) FP16 tensors (seed ``b * 10000 + index``); each
    cell is the median of ``reps`` launches through ``action_expansion.launch`` (allocation
    included, as the reference times its calls), each after a 256 MiB L2 flush, following one
    untimed launch. Bank 0's first output of each candidate is checked against the FP32 product
    (1e-2 elementwise and normwise); a candidate that fails or raises is unusable (None)."""
    import statistics

    import torch

    from heliostune_b200.action_expansion import fp32_reference, launch
    from heliostune_b200.kernel import get_hardware_profile, require_b200
    from heliostune_b200.timing import flush_buffer

    device = torch.device("cuda", torch.cuda.current_device())
    hardware = get_hardware_profile("B200", device)
    require_b200(hardware)
    flush = flush_buffer(device)
    latency: dict[str, dict[str, list[float | None]]] = {}
    for index, workload in enumerate(workloads):
        cells: dict[str, list[float | None]] = {c.key: [None, None, None] for c in replay_candidates_for(workload)}
        broken: set[str] = set()
        for bank in BANKS:
            g = torch.Generator(device=device).manual_seed(bank * 10000 + index)
            a = (torch.randn((workload.m, workload.k), generator=g, device=device) / math.sqrt(workload.k)).half()
            b = (torch.randn((workload.k, workload.n), generator=g, device=device) / math.sqrt(workload.k)).half()
            expected = fp32_reference(a, b) if bank == OBSERVATION_BANK else None
            for candidate in replay_candidates_for(workload):
                if candidate.key in broken:
                    continue
                try:
                    out = launch(a, b, candidate)
                    if expected is not None:
                        diff = (out.float() - expected).abs()
                        scale = expected.abs().max().item()
                        if not (bool((diff <= 1e-2 + 1e-2 * expected.abs()).all().item()) and diff.max().item() <= 1e-2 * scale):
                            raise ValueError("parity failure")
                    del out
                    events = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
                    for start, end in events:
                        flush.zero_()
                        start.record()
                        launch(a, b, candidate)
                        end.record()
                    torch.cuda.synchronize(device)
                    cells[candidate.key][bank] = statistics.median(s.elapsed_time(e) for s, e in events)
                except (ValueError, RuntimeError) as exc:
                    broken.add(candidate.key)
                    cells[candidate.key] = [None, None, None]
                    log(f"{workload.key} {candidate.key}: {exc}")
            del a, b, expected
        latency[workload.key] = cells
        log(f"{index + 1}/{len(workloads)} {workload.key}")
    return {
        "hardware": hardware.to_dict(),
        "workloads": [w.to_dict() for w in workloads],
        "banks": {"0": "policy-visible observations", "1": "exhaustive-reference selection", "2": "held-out evaluation"},
        "timing": f"median of {reps} launches after a 256 MiB L2 flush each, CUDA events, allocation included",
        "latency_ms": latency,
    }


def main(argv: Sequence[str] | None = None) -> None:
    """``collect OUT`` (GPU) writes a timing table; ``compare TABLE`` prints the comparison."""
    parser = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    sub = parser.add_subparsers(dest="command", required=True)
    collect = sub.add_parser("collect")
    collect.add_argument("out", type=Path)
    collect.add_argument("--reps", type=int, default=5)
    compare = sub.add_parser("compare")
    compare.add_argument("table", type=Path)
    compare.add_argument("--seeds", type=int, default=30)
    args = parser.parse_args(argv)
    if args.command == "collect":
        table = collect_timing_table(reps=args.reps)
        args.out.parent.mkdir(parents=True, exist_ok=True)
        args.out.write_text(json.dumps(table, indent=None, separators=(",", ":"), sort_keys=True) + "\n")
    else:
        table = TimingTable.from_dict(json.loads(args.table.read_text()))
        print(json.dumps(compare_feature_bases(table, seeds=args.seeds), indent=1))


if __name__ == "__main__":
    main()
