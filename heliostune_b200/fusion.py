"""RMSNorm on the B200, and the closed registry that hands it out.

The reference exposes its residual RMSNorm as ``torch.library`` ops named
``heliostune_fusion_v2::residual_rmsnorm_w{4,8,16,32}`` behind a closed loader
(``src/heliostune/fusion_kernels.py:72-93``, ``src/heliostune/_fusion_gpu.py:76-188``). This
build measures the form without a residual: ``y = fp16((x * rsqrt(mean(x^2) + eps)) * gamma)``
with an FP32 row sum, for any ``[rows, hidden]`` FP16 input. ``rmsnorm`` launches
``hst_rmsnorm`` of the C-ABI library; ``load_rmsnorm`` is the registry.
"""

from __future__ import annotations

from collections.abc import Callable

import torch

from heliostune_b200 import _native
from heliostune_b200.kernel import _stream

DEFAULT_EPS = 1e-6


def rmsnorm(x: torch.Tensor, gamma: torch.Tensor, eps: float = DEFAULT_EPS) -> torch.Tensor:
    """Row RMSNorm of a CUDA FP16 ``[rows, hidden]`` matrix; inputs are never modified."""
    if x.ndim != 2 or gamma.ndim != 1 or gamma.shape[0] != x.shape[1]:
        raise ValueError("rmsnorm expects x [rows, hidden] and gamma [hidden]")
    if x.dtype != torch.float16 or gamma.dtype != torch.float16:
        raise ValueError("rmsnorm inputs must have dtype torch.float16")
    if x.device.type != "cuda" or gamma.device != x.device:
        raise ValueError("rmsnorm inputs must be on the same CUDA device")
    if x.stride(1) != 1 or not gamma.is_contiguous():
        raise ValueError("rmsnorm needs unit-stride rows and a contiguous gamma")
    rows, hidden = int(x.shape[0]), int(x.shape[1])
    y = torch.empty((rows, hidden), device=x.device, dtype=torch.float16)
    with torch.cuda.device(x.device):
        _native.check(
            _native.library().hst_rmsnorm(
                x.data_ptr(),
                x.stride(0) if rows > 1 else hidden,
                gamma.data_ptr(),
                y.data_ptr(),
                hidden,
                rows,
                hidden,
                float(eps),
                _stream(x.device),
            )
        )
    return y


RMSNORM_ENTRYPOINTS: tuple[str, ...] = ("heliostune_b200::rmsnorm",)


def load_rmsnorm(entrypoint: str) -> Callable[..., torch.Tensor]:
    """Closed registry: only declared entry points resolve, anything else is a ``KeyError``."""
    if entrypoint not in RMSNORM_ENTRYPOINTS:
        raise KeyError(f"unknown RMSNorm entry point {entrypoint!r}")
    return rmsnorm
