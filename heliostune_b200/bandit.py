"""Bayesian linear Thompson sampling over launch configurations.

Same model and numerics as ``BayesianLinearBandit`` at ``src/heliostune/bandit.py:17-259``:
observations ``y = x . w + e`` with ``e ~ N(0, noise_variance)`` and a zero-mean isotropic ridge
prior of precision ``prior_precision``. The posterior is held in information form
(precision ``P``, information vector ``h``); an update adds ``x x^T / s2`` and ``x y / s2``.
The mean solves ``L L^T mu = h`` with ``L = cholesky(P)``; a sample is
``mu + L^-T z`` with ``z`` standard normal from a seeded ``numpy`` generator, so a given seed
and update sequence reproduces the reference's choices exactly. Ties go to the earliest action.
"""

from __future__ import annotations

import math
from collections.abc import Callable, Sequence
from typing import TypeVar

import numpy as np
from numpy.typing import ArrayLike, NDArray

from heliostune_b200.features import V2_FEATURE_NAMES

ActionT = TypeVar("ActionT")


def _positive_finite(value: object, name: str) -> float:
    try:
        number = float(value)  # type: ignore[arg-type]
    except (TypeError, ValueError) as exc:
        raise ValueError(f"{name} must be positive and finite") from exc
    if not math.isfinite(number) or number <= 0.0:
        raise ValueError(f"{name} must be positive and finite")
    return number


class BayesianLinearBandit:
    """A Gaussian linear posterior with one Thompson sample per choice."""

    def __init__(
        self,
        dimension: int = len(V2_FEATURE_NAMES),
        *,
        prior_precision: float = 1.0,
        noise_variance: float = 1.0,
        seed: int = 0,
    ) -> None:
        if isinstance(dimension, bool) or not isinstance(dimension, int | np.integer):
            raise TypeError("dimension must be an integer")
        if dimension <= 0:
            raise ValueError("dimension must be positive")
        self._prior_precision = _positive_finite(prior_precision, "prior_precision")
        self._noise_variance = _positive_finite(noise_variance, "noise_variance")
        self._dimension = int(dimension)
        self._precision = np.eye(self._dimension, dtype=np.float64) * self._prior_precision
        self._information = np.zeros(self._dimension, dtype=np.float64)
        self._observed_count = 0
        self._cholesky: NDArray[np.float64] | None = None
        self._mean: NDArray[np.float64] | None = None
        self._rng = np.random.default_rng(seed)

    @property
    def dimension(self) -> int:
        return self._dimension

    @property
    def observed_count(self) -> int:
        """Observations added directly to this posterior (transferred evidence excluded)."""
        return self._observed_count

    @property
    def precision(self) -> NDArray[np.float64]:
        return self._precision.copy()

    @property
    def information(self) -> NDArray[np.float64]:
        return self._information.copy()

    @property
    def mean(self) -> NDArray[np.float64]:
        if self._mean is None:
            factor = self._factor()
            self._mean = np.linalg.solve(factor.T, np.linalg.solve(factor, self._information))
        return self._mean.copy()

    def update(self, features: ArrayLike, observation: float) -> None:
        """Condition on one (features, observation) pair; a rejected update changes nothing."""
        x = self._checked(features)
        if isinstance(observation, bool | np.bool_):
            raise ValueError("observation must be a finite scalar")
        try:
            y = float(observation)  # type: ignore[arg-type]
        except (TypeError, ValueError) as exc:
            raise ValueError("observation must be a finite scalar") from exc
        if not math.isfinite(y):
            raise ValueError("observation must be a finite scalar")
        scale = 1.0 / self._noise_variance
        with np.errstate(over="ignore", invalid="ignore"):
            precision = self._precision + scale * np.outer(x, x)
            information = self._information + scale * x * y
        if not (np.all(np.isfinite(precision)) and np.all(np.isfinite(information))):
            raise ValueError("observation would produce a non-finite posterior state")
        count = self._observed_count + 1
        try:
            factor = np.linalg.cholesky(precision)
        except np.linalg.LinAlgError as exc:
            raise ValueError(
                f"posterior precision Cholesky failed for dimension {self._dimension} "
                f"after {count} observations"
            ) from exc
        self._precision, self._information = precision, information
        self._observed_count = count
        self._cholesky, self._mean = factor, None

    def sample(self) -> NDArray[np.float64]:
        """One coefficient vector drawn from the posterior."""
        factor = self._factor()
        z = self._rng.standard_normal(self._dimension)
        return self.mean + np.linalg.solve(factor.T, z)

    def choose(self, actions: Sequence[ActionT], feature_fn: Callable[[ActionT], ArrayLike]) -> ActionT:
        """The action maximising the sampled linear reward; the earliest action wins ties."""
        if len(actions) == 0:
            raise ValueError("actions must not be empty")
        rows = np.stack([self._checked(feature_fn(action)) for action in actions])
        theta = self.sample()
        with np.errstate(over="ignore", invalid="ignore"):
            scores = rows @ theta
        if not np.all(np.isfinite(scores)):
            raise ValueError("action scores must be finite")
        return actions[int(np.argmax(scores))]

    def transferred(
        self,
        transfer_strength: float,
        *,
        prior_precision: float | None = None,
        noise_variance: float | None = None,
        seed: int = 0,
    ) -> BayesianLinearBandit:
        """A new posterior: target ridge prior plus this likelihood raised to ``strength``."""
        try:
            strength = float(transfer_strength)
        except (TypeError, ValueError) as exc:
            raise ValueError("transfer_strength must be finite and between 0 and 1") from exc
        if not math.isfinite(strength) or not 0.0 <= strength <= 1.0:
            raise ValueError("transfer_strength must be finite and between 0 and 1")
        target = type(self)(
            self._dimension,
            prior_precision=self._prior_precision if prior_precision is None else prior_precision,
            noise_variance=self._noise_variance if noise_variance is None else noise_variance,
            seed=seed,
        )
        if strength != 0.0:
            likelihood = self._precision.copy()
            likelihood[np.diag_indices(self._dimension)] -= self._prior_precision
            target._precision += strength * likelihood
            target._information = strength * self._information
        return target

    def _checked(self, features: ArrayLike) -> NDArray[np.float64]:
        try:
            x = np.asarray(features, dtype=np.float64)
        except (TypeError, ValueError) as exc:
            raise ValueError("features must be a finite one-dimensional numeric vector") from exc
        if x.shape != (self._dimension,):
            raise ValueError(f"features must have shape ({self._dimension},), got {x.shape}")
        if not np.all(np.isfinite(x)):
            raise ValueError("features must contain only finite values")
        return x.copy()

    def _factor(self) -> NDArray[np.float64]:
        if self._cholesky is None:
            try:
                self._cholesky = np.linalg.cholesky(self._precision)
            except np.linalg.LinAlgError as exc:
                raise ValueError(
                    f"posterior precision Cholesky failed for dimension {self._dimension} "
                    f"after {self._observed_count} observations"
                ) from exc
        return self._cholesky
