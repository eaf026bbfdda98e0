"""The bandit's reward: natural log of achieved TFLOP/s.

Restates ``log_tflops_reward`` at ``src/heliostune/retrieval.py:98-112``: a GEMM of
``workload.flops`` operations that takes ``latency_ms`` milliseconds achieves
``flops / (latency_ms * 1e9)`` TFLOP/s; the log is taken as a sum of logs.
"""

from __future__ import annotations

import math

from heliostune_b200.configs import Workload


def log_tflops_reward(workload: Workload, latency_ms: float) -> float:
    if not math.isfinite(latency_ms) or latency_ms <= 0.0:
        raise ValueError("latency_ms must be finite and positive")
    reward = math.log(workload.flops) - math.log(latency_ms) - math.log(1e9)
    if not math.isfinite(reward):
        raise ValueError("log-TFLOP/s reward must be finite")
    return reward
