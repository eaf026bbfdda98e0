"""Generate the golden fixtures of tests/golden/ from the reference implementation.

Run in a container where the reference (mottopanikeiku/heliostune) is mounted, e.g.
``python tests/golden/make_golden.py /path/to/heliostune``. It imports the reference's own
Python modules (bandit, features, configs, action_configs, action_collection, retrieval, replay,
local_executor) and records what they compute on seeded inputs. The reference needs two things
its environment would normally provide: installed package metadata (for ``__version__``) and the
``zstandard`` module (imported by a tooling module, never called here); both are stubbed in a
temporary directory. The GEMM fixtures hold seeded FP16 operands and their FP32 product computed
by torch on the CPU in FP64 (an implementation independent of the oracle).

Nothing at test time reads the reference: tests only read the files this script writes.
"""

from __future__ import annotations

import hashlib
import json
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _stub_environment(root: Path) -> Path:
    stub = Path(tempfile.mkdtemp(prefix="hst-golden-"))
    dist = stub / "heliostune-0.0.0.dist-info"
    dist.mkdir()
    (dist / "METADATA").write_text("Metadata-Version: 2.1\nName: heliostune\nVersion: 0.0.0\n")
    (stub / "zstandard.py").write_text("# stub: the golden script never touches .zst archives\n")
    sys.path[:0] = [str(root / "src"), str(stub)]
    return stub


def _dump(name: str, data: object) -> None:
    (HERE / name).write_text(json.dumps(data, indent=1, sort_keys=True) + "\n")
    print("wrote", name)


def bandit_fixtures() -> None:
    from heliostune.bandit import BayesianLinearBandit

    scenarios = []
    rng = np.random.default_rng(1234)
    for case, (dim, prior, noise, seed, updates) in enumerate(
        [(3, 2.0, 0.5, 3, 4), (5, 1.0, 0.05, 11, 12), (25, 1.0, 0.05, 7, 30)]
    ):
        model = BayesianLinearBandit(dimension=dim, prior_precision=prior, noise_variance=noise, seed=seed)
        steps = []
        for _ in range(updates):
            x = rng.standard_normal(dim).round(6).tolist()
            y = float(round(rng.standard_normal(), 6))
            model.update(x, y)
            actions = rng.standard_normal((6, dim)).round(6).tolist()
            chosen = model.choose(list(range(6)), lambda i, a=actions: a[i])
            steps.append(
                {
                    "x": x,
                    "y": y,
                    "actions": actions,
                    "chosen": int(chosen),
                    "mean": model.mean.tolist(),
                }
            )
        final_precision = model.precision.tolist()
        sample = model.sample().tolist()
        transferred = model.transferred(0.08, seed=seed + 1)
        scenarios.append(
            {
                "dimension": dim,
                "prior_precision": prior,
                "noise_variance": noise,
                "seed": seed,
                "steps": steps,
                "final_sample": sample,
                "final_precision": final_precision,
                "transferred_precision": transferred.precision.tolist(),
                "transferred_mean": transferred.mean.tolist(),
            }
        )
    _dump("bandit.json", {"scenarios": scenarios})


def _profiles():
    from heliostune.schema import HardwareProfile

    return [
        HardwareProfile("H100", "NVIDIA H100 80GB HBM3", (9, 0), 132, 79.1),
        HardwareProfile("B200", "NVIDIA B200", (10, 0), 148, 179.0615234375),
        HardwareProfile("L4", "NVIDIA L4", (8, 9), 58, 22.0343017578125),
    ]


def feature_fixtures() -> None:
    from heliostune.configs import DEFAULT_CONFIGS, DEFAULT_WORKLOADS
    from heliostune.features import V2_FEATURE_NAMES, v2_joint_features

    profiles = _profiles()
    full = np.stack(
        [
            v2_joint_features(w, c, p)
            for p in profiles
            for w in DEFAULT_WORKLOADS
            for c in DEFAULT_CONFIGS
        ]
    )
    sample_rows = list(range(0, full.shape[0], 97))
    np.savez_compressed(HERE / "features.npz", rows=np.asarray(sample_rows), values=full[sample_rows])
    _dump(
        "features.json",
        {
            "names": list(V2_FEATURE_NAMES),
            "shape": list(full.shape),
            "sha256": hashlib.sha256(full.astype("<f8").tobytes()).hexdigest(),
            "profiles": [p.to_dict() for p in profiles],
        },
    )


def manifest_fixtures() -> None:
    from heliostune.action_collection import bank_order, protocol, select_finalists, tensor_seed, timing_order
    from heliostune.action_configs import ALL_CANDIDATES, action_set_manifest, candidates_for
    from heliostune.configs import DEFAULT_CONFIGS, DEFAULT_WORKLOADS, HOPPER_GEMM_CONFIGS
    from heliostune.hopper_spec import EDGE_WORKLOADS
    from heliostune.retrieval import log_tflops_reward

    rewards = [
        [w.key, latency, log_tflops_reward(w, latency)]
        for w in DEFAULT_WORKLOADS[::11]
        for latency in (0.0123, 1.0, 37.5)
    ]
    orders = {
        str(bank): [w.key for w in bank_order(DEFAULT_WORKLOADS, bank)] for bank in (1, 2)
    }
    timing = [
        {
            "bank": bank,
            "index": index,
            "workload": DEFAULT_WORKLOADS[wi].key,
            "order": timing_order(bank, index, DEFAULT_WORKLOADS[wi], None),
            "seed": tensor_seed(bank, index),
        }
        for bank, index, wi in ((1, 0, 0), (1, 17, 40), (2, 5, 95), (2, 63, 3))
    ]
    finalists = frozenset([DEFAULT_CONFIGS[3].key, ALL_CANDIDATES[2].key])
    timing.append(
        {
            "bank": 2,
            "index": 9,
            "workload": DEFAULT_WORKLOADS[1].key,
            "order": timing_order(2, 9, DEFAULT_WORKLOADS[1], finalists),
            "finalists": sorted(finalists),
            "seed": tensor_seed(2, 9),
        }
    )
    rows = [
        {"family": "torch", "config_key": "torch", "correct": True, "error": None, "median_ms": 0.5},
        {"family": "old", "config_key": "b", "correct": True, "error": None, "median_ms": 1.0},
        {"family": "old", "config_key": "a", "correct": True, "error": None, "median_ms": 1.0},
        {"family": "tile", "config_key": "tile:x", "correct": False, "error": None, "median_ms": 0.1},
        {"family": "split_k", "config_key": "split_k:y", "correct": True, "error": None, "median_ms": 0.7},
        {"family": "persistent", "config_key": "persistent:z", "correct": True, "error": "boom", "median_ms": 0.2},
    ]
    _dump(
        "manifest.json",
        {
            "action_set": action_set_manifest(),
            "all_candidate_keys": [c.key for c in ALL_CANDIDATES],
            "candidates_by_workload": {w.key: [c.key for c in candidates_for(w)] for w in DEFAULT_WORKLOADS},
            "default_config_keys": [c.key for c in DEFAULT_CONFIGS],
            "hopper_config_keys": [c.key for c in HOPPER_GEMM_CONFIGS],
            "default_workloads": [[w.key, w.m, w.n, w.k, w.flops] for w in DEFAULT_WORKLOADS],
            "edge_workloads": [w.key for w in EDGE_WORKLOADS],
            "rewards": rewards,
            "bank_orders": orders,
            "timing_orders": timing,
            "finalist_rows": rows,
            "finalists": select_finalists(rows),
            "protocol": protocol(),
        },
    )


class _Row:
    def __init__(self, workload, latency_ms):
        self.workload = workload
        self.latency_ms = latency_ms
        self.usable = True


class _SyntheticTable:
    """A latency matrix with the BenchmarkTable methods the replay loop calls."""

    def __init__(self, workloads, configs, hardware):
        self.hw = hardware
        self.lat = {}
        rng = np.random.default_rng(99)
        for w in workloads:
            for c in configs:
                base = w.flops / 1e9 / (50 + 3 * np.log2(c.block_m * c.block_n) - abs(np.log2(w.m) - 6))
                self.lat[(w.key, c.key, 0)] = float(base * (1 + 0.2 * rng.random()))
                self.lat[(w.key, c.key, 2)] = float(base * (1 + 0.2 * rng.random()))
        self.calls = []

    def hardware(self, gpu):
        return self.hw

    def get(self, gpu, workload, config, bank):
        self.calls.append([workload.key, config.key])
        return _Row(workload, self.lat[(workload.key, config.key, bank)])

    def _latency(self, gpu, workload, config, bank):
        return self.lat[(workload.key, config.key, bank)]

    def heldout_fraction(self, gpu, workload, recommendation):
        best = min(v for (wk, ck, b), v in self.lat.items() if wk == workload.key and b == 2)
        return best / self.lat[(workload.key, recommendation.key, 2)]


def bandit_curve_fixtures() -> None:
    from heliostune.bandit import BayesianLinearBandit
    from heliostune.configs import DEFAULT_CONFIGS, DEFAULT_WORKLOADS
    from heliostune.features import V2_FEATURE_NAMES
    from heliostune.replay import _bandit_curve

    hardware = _profiles()[1]
    workloads = tuple(w for w in DEFAULT_WORKLOADS if w.model == "qwen2.5-7b")
    configs = tuple(sorted(DEFAULT_CONFIGS, key=lambda c: c.key))
    table = _SyntheticTable(workloads, configs, hardware)
    policy_seed = 3
    order_rng = np.random.default_rng(policy_seed + 50_000)
    orders = [tuple(workloads[i] for i in order_rng.permutation(len(workloads))) for _ in range(8)]
    model = BayesianLinearBandit(dimension=len(V2_FEATURE_NAMES), noise_variance=0.05, prior_precision=1.0, seed=policy_seed)
    curve = _bandit_curve(table, "B200", workloads, configs, orders, model)
    _dump(
        "bandit_curve.json",
        {
            "policy_seed": policy_seed,
            "workloads": [w.key for w in workloads],
            "configs": [c.key for c in configs],
            "latency_bank0": {f"{wk}|{ck}": v for (wk, ck, b), v in table.lat.items() if b == 0},
            "probes": table.calls,
            "curve": curve,
            "final_mean": model.mean.tolist(),
        },
    )


def gemm_fixtures() -> None:
    import torch

    from heliostune.kernel import _within_tolerance

    cases = {}
    specs = [
        ("edge_1x8x8", 1, 8, 8, 0),
        ("edge_7x136x264", 7, 136, 264, 1),
        ("edge_131x1032x520", 131, 1032, 520, 2),
        ("splitk_7x131x17", 7, 131, 17, 3),
        ("splitk_31x131x1543", 31, 131, 1543, 4),
    ]
    for name, m, n, k, seed in specs:
        g = torch.Generator().manual_seed(seed)
        a = (torch.randn((m, k), generator=g) / k**0.5).to(torch.float16)
        b = (torch.randn((k, n), generator=g) / k**0.5).to(torch.float16)
        c = (a.double() @ b.double()).float()
        cases[f"{name}_a"] = a.numpy()
        cases[f"{name}_b"] = b.numpy()
        # Large products keep every 8th row of C to stay small; tests compare those rows.
        cases[f"{name}_c"] = c.numpy() if m * n <= 8192 else c.numpy()[::8]
        cases[f"{name}_crows"] = np.arange(0, m, 1 if m * n <= 8192 else 8)
    # Strided operands of the reference split-K test (tests/test_action_expansion.py:59-69).
    g = torch.Generator().manual_seed(31)
    a_full = torch.rand((31, 514), generator=g).to(torch.float16)
    b_full = torch.rand((514, 134), generator=g).to(torch.float16)
    a, b = a_full[:, ::2], b_full[::2, ::2]
    cases["strided_a_full"] = a_full.numpy()
    cases["strided_b_full"] = b_full.numpy()
    cases["strided_c"] = (a.double() @ b.double()).float().numpy()
    np.savez_compressed(HERE / "gemm_cases.npz", **cases)
    # The reference's tolerance known-answer test (tests/test_kernel.py:66-75).
    out = torch.tensor([1.0, 1.125], dtype=torch.float16)
    exp = torch.tensor([1.0, 1.0], dtype=torch.float32)
    diff = torch.empty_like(exp)
    torch.sub(out, exp, out=diff)
    diff.abs_()
    _dump(
        "tolerance_kat.json",
        {
            "output": [1.0, 1.125],
            "expected": [1.0, 1.0],
            "cases": [
                {"atol": 0.0, "rtol": 0.125, "within": _within_tolerance(diff, exp, atol=0.0, rtol=0.125)},
                {"atol": 0.0, "rtol": 0.124, "within": _within_tolerance(diff, exp, atol=0.0, rtol=0.124)},
                {"atol": 0.01, "rtol": 0.01, "within": _within_tolerance(diff, exp, atol=0.01, rtol=0.01)},
                {"atol": 0.125, "rtol": 0.0, "within": _within_tolerance(diff, exp, atol=0.125, rtol=0.0)},
            ],
        },
    )


def rmsnorm_fixtures() -> None:
    import torch

    from heliostune.local_executor import _residual_rmsnorm

    g = torch.Generator().manual_seed(17)
    x = torch.randn((8, 4096), generator=g).to(torch.bfloat16)
    residual = torch.randn((8, 4096), generator=g).to(torch.bfloat16)
    gamma = (1.0 + 0.02 * torch.randn((4096,), generator=g)).to(torch.bfloat16)
    expected = _residual_rmsnorm(torch, x, residual, gamma, 1e-5)
    zero = torch.zeros_like(x)
    expected_nores = _residual_rmsnorm(torch, x, zero, gamma, 1e-5)
    np.savez_compressed(
        HERE / "rmsnorm_bf16.npz",
        x=x.view(torch.int16).numpy().view(np.uint16),
        residual=residual.view(torch.int16).numpy().view(np.uint16),
        gamma=gamma.view(torch.int16).numpy().view(np.uint16),
        expected=expected.view(torch.int16).numpy().view(np.uint16),
        expected_no_residual=expected_nores.view(torch.int16).numpy().view(np.uint16),
    )
    print("wrote rmsnorm_bf16.npz")


def collection_fixtures(root: Path) -> None:
    """The reference's analysis script (scripts/analyze_action_expansion.py) on the pilot artifact
    that heliostune_b200.collection writes for the synthetic measurements of
    tests/golden/collection_fixture.py: the artifact's SHA-256 and what the analysis returned."""
    import hashlib
    import importlib.util

    from heliostune.action_collection import collection_workloads

    repo = HERE.parents[1]
    if str(repo) not in sys.path:
        sys.path.insert(0, str(repo))
    from heliostune_b200.collection import dumps_strict
    from tests.golden.collection_fixture import build

    spec = importlib.util.spec_from_file_location("analyze_action_expansion", root / "scripts" / "analyze_action_expansion.py")
    analyzer = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(analyzer)
    data = build(Path(tempfile.mkdtemp(prefix="hst-collection-")))
    text = dumps_strict(data)
    summary = analyzer.analyze(json.loads(text), expected_workloads=collection_workloads(True))
    _dump(
        "collection_analysis.json",
        {
            "artifact_sha256": hashlib.sha256(text.encode()).hexdigest(),
            "overall": summary["overall"],
            "by_m": summary["by_m"],
            "failure_row_count": summary["failure_row_count"],
            "selected": {w["workload_key"]: w["selected"] for w in summary["workloads"]},
        },
    )


def validation_fixtures() -> None:
    """The reference's pre-timing gate sample (hopper_spec.py:26-55) over its 96 workloads."""
    from heliostune.hopper_spec import validation_workloads

    _dump("validation_workloads.json", {"keys": [w.key for w in validation_workloads()]})


def main() -> None:
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_golden.py <path of the reference checkout>")
    root = Path(sys.argv[1])
    _stub_environment(root)
    bandit_fixtures()
    feature_fixtures()
    manifest_fixtures()
    bandit_curve_fixtures()
    gemm_fixtures()
    rmsnorm_fixtures()
    collection_fixtures(root)
    validation_fixtures()


if __name__ == "__main__":
    main()
