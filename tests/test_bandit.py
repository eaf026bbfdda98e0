"""The bandit: the reference's own tests (tests/test_bandit.py) ported, and a bit-exact replay
of posterior states and choices the reference's BayesianLinearBandit produced."""

from __future__ import annotations

import numpy as np
import pytest
from hypothesis import given, settings
from hypothesis import strategies as st

from heliostune_b200.bandit import BayesianLinearBandit
from tests.conftest import load_golden


def test_golden_scenarios_replay_bit_exactly() -> None:
    for scenario in load_golden("bandit.json")["scenarios"]:
        model = BayesianLinearBandit(
            dimension=scenario["dimension"],
            prior_precision=scenario["prior_precision"],
            noise_variance=scenario["noise_variance"],
            seed=scenario["seed"],
        )
        for step in scenario["steps"]:
            model.update(step["x"], step["y"])
            actions = step["actions"]
            assert model.choose(list(range(len(actions))), lambda i, a=actions: a[i]) == step["chosen"]
            np.testing.assert_array_equal(model.mean, np.asarray(step["mean"]))
        np.testing.assert_array_equal(model.precision, np.asarray(scenario["final_precision"]))
        np.testing.assert_array_equal(model.sample(), np.asarray(scenario["final_sample"]))
        target = model.transferred(0.08, seed=scenario["seed"] + 1)
        np.testing.assert_array_equal(target.precision, np.asarray(scenario["transferred_precision"]))
        np.testing.assert_array_equal(target.mean, np.asarray(scenario["transferred_mean"]))


def test_power_prior_transfer_preserves_only_discounted_likelihood() -> None:
    source = BayesianLinearBandit(dimension=3, prior_precision=2.0, noise_variance=0.5, seed=3)
    source.update([1.0, 0.0, 0.5], 2.0)
    source.update([0.0, 1.0, -0.5], -1.0)
    zero = source.transferred(0.0, seed=4)
    np.testing.assert_allclose(zero.precision, np.eye(3) * 2.0)
    np.testing.assert_allclose(zero.mean, np.zeros(3))
    full = source.transferred(1.0, seed=4)
    np.testing.assert_allclose(full.precision, source.precision)
    np.testing.assert_allclose(full.mean, source.mean)
    assert full.observed_count == 0


def test_rejected_update_is_atomic_when_cholesky_fails(monkeypatch: pytest.MonkeyPatch) -> None:
    model = BayesianLinearBandit(dimension=2)
    model.update([1.0, 0.0], 1.0)
    _ = model.mean
    precision, mean = model.precision, model.mean
    cholesky = model._cholesky.copy()

    def fail(_matrix: np.ndarray) -> np.ndarray:
        raise np.linalg.LinAlgError("forced failure")

    monkeypatch.setattr(np.linalg, "cholesky", fail)
    with pytest.raises(ValueError, match=r"dimension 2.*after 2 observations"):
        model.update([0.0, 1.0], 2.0)
    np.testing.assert_array_equal(model.precision, precision)
    np.testing.assert_array_equal(model._mean, mean)
    np.testing.assert_array_equal(model._cholesky, cholesky)
    assert model.observed_count == 1


def test_update_validates_cumulative_finiteness_before_commit() -> None:
    model = BayesianLinearBandit(dimension=1)
    model._precision[0, 0] = np.finfo(np.float64).max
    precision = model.precision
    with pytest.raises(ValueError, match="non-finite posterior state"):
        model.update([np.sqrt(np.finfo(np.float64).max)], 1.0)
    np.testing.assert_array_equal(model.precision, precision)


def test_samples_follow_the_posterior_mean_and_covariance() -> None:
    model = BayesianLinearBandit(dimension=2, prior_precision=0.5, noise_variance=0.25, seed=11)
    model.update([1.0, 2.0], 1.5)
    model.update([-1.0, 0.5], -0.5)
    model.update([0.3, -1.0], 0.2)
    samples = np.stack([model.sample() for _ in range(40_000)])
    np.testing.assert_allclose(samples.mean(axis=0), model.mean, atol=0.01)
    np.testing.assert_allclose(np.cov(samples, rowvar=False), np.linalg.inv(model.precision), rtol=0.05, atol=1e-3)


def test_choose_breaks_ties_in_favor_of_the_earliest_action() -> None:
    model = BayesianLinearBandit(dimension=2, seed=5)
    features = {"first": [1.0, 1.0], "second": [1.0, 1.0], "third": [1.0, 1.0]}
    assert model.choose(("first", "second", "third"), features.__getitem__) == "first"


@pytest.mark.parametrize("dimension", [0, -1])
def test_constructor_rejects_nonpositive_dimensions(dimension: int) -> None:
    with pytest.raises(ValueError, match="dimension must be positive"):
        BayesianLinearBandit(dimension=dimension)


@pytest.mark.parametrize("dimension", [True, 2.0, "2"])
def test_constructor_rejects_noninteger_dimensions(dimension: object) -> None:
    with pytest.raises(TypeError, match="dimension must be an integer"):
        BayesianLinearBandit(dimension=dimension)  # type: ignore[arg-type]


@pytest.mark.parametrize("parameter", ["prior_precision", "noise_variance"])
@pytest.mark.parametrize("value", [0.0, -1.0, float("inf"), float("nan"), "x"])
def test_constructor_rejects_invalid_distribution_parameters(parameter: str, value: object) -> None:
    with pytest.raises(ValueError, match=f"{parameter} must be positive and finite"):
        BayesianLinearBandit(dimension=1, **{parameter: value})  # type: ignore[arg-type]


@pytest.mark.parametrize("observation", [float("nan"), float("inf"), "x", None, [1.0, 2.0], True])
def test_update_rejects_nonfinite_or_nonscalar_observations(observation: object) -> None:
    model = BayesianLinearBandit(dimension=1)
    with pytest.raises(ValueError, match="finite scalar"):
        model.update([1.0], observation)  # type: ignore[arg-type]
    assert model.observed_count == 0


@pytest.mark.parametrize(
    ("features", "message"),
    [
        ([1.0], r"shape \(2,\), got \(1,\)"),
        ([[1.0, 2.0]], r"shape \(2,\), got \(1, 2\)"),
        ([1.0, float("nan")], "only finite values"),
        (["a", "b"], "finite one-dimensional numeric vector"),
    ],
)
def test_invalid_feature_vectors_are_rejected(features: object, message: str) -> None:
    model = BayesianLinearBandit(dimension=2)
    with pytest.raises(ValueError, match=message):
        model.update(features, 1.0)  # type: ignore[arg-type]
    with pytest.raises(ValueError, match=message):
        model.choose(["only"], lambda _a: features)  # type: ignore[arg-type,return-value]


def test_choose_rejects_empty_actions_and_overflowing_scores() -> None:
    with pytest.raises(ValueError, match="actions must not be empty"):
        BayesianLinearBandit(dimension=1).choose([], lambda a: [1.0])
    diffuse = BayesianLinearBandit(dimension=1, prior_precision=1e-300, seed=1)
    with pytest.raises(ValueError, match="action scores must be finite"):
        diffuse.choose(["huge"], lambda _a: [1e308])


@pytest.mark.parametrize("strength", [-0.1, 1.1, float("nan"), float("inf"), "x", None])
def test_transfer_strength_must_be_in_the_unit_interval(strength: object) -> None:
    with pytest.raises(ValueError, match="transfer_strength must be finite and between 0 and 1"):
        BayesianLinearBandit(dimension=1).transferred(strength)  # type: ignore[arg-type]


_floats = st.floats(min_value=-100.0, max_value=100.0, allow_nan=False, allow_infinity=False)


@settings(max_examples=60, deadline=None)
@given(
    dimension=st.integers(1, 5),
    data=st.data(),
    prior=st.floats(0.1, 10.0),
    noise=st.floats(0.1, 10.0),
)
def test_precision_is_the_ridge_prior_plus_scaled_gram_matrix(
    dimension: int, data: st.DataObject, prior: float, noise: float
) -> None:
    count = data.draw(st.integers(0, 12))
    rows = [data.draw(st.lists(_floats, min_size=dimension, max_size=dimension)) for _ in range(count)]
    ys = data.draw(st.lists(_floats, min_size=count, max_size=count))
    model = BayesianLinearBandit(dimension=dimension, prior_precision=prior, noise_variance=noise)
    for x, y in zip(rows, ys, strict=True):
        model.update(x, y)
    x = np.asarray(rows, dtype=np.float64).reshape(count, dimension)
    expected = np.eye(dimension) * prior + x.T @ x / noise
    np.testing.assert_allclose(model.precision, expected, rtol=1e-9, atol=1e-6)
    assert model.observed_count == count
