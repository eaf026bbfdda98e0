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
from heliostune_b200.action_configs import ActionCandidate
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


def rmsnorm_matmul(
    x: torch.Tensor,
    gamma: torch.Tensor,
    w: torch.Tensor,
    candidate: ActionCandidate,
    eps: float = DEFAULT_EPS,
) -> torch.Tensor:
    """``RMSNorm(x; gamma, eps) @ W`` -- the RMSNorm feeding the QKV projection.

    The normalised rows are produced exactly as the reference's formula rounds them,
    ``fp16((x * rsqrt(mean(x^2) + eps)) * gamma)``, into a per-call workspace by the RMSNorm
    kernel, and the GEMM candidate consumes that workspace on the same stream. Materialising the
    ``[M, K]`` FP16 rows costs ``4MK`` bytes of HBM traffic (write + read) next to the GEMM's
    ``2(MK + KN + MN)``; rescaling the A tiles inside the GEMM instead would put the same work
    on the shared-memory path the tensor-core main loop is limited by.
    """
    from heliostune_b200.action_expansion import launch

    if w.ndim != 2 or w.shape[0] != x.shape[1]:
        raise ValueError(f"incompatible shapes: x {tuple(x.shape)} and W {tuple(w.shape)}")
    normalised = rmsnorm(x, gamma, eps)
    return launch(normalised, w, candidate)


RMSNORM_ENTRYPOINTS: tuple[str, ...] = ("heliostune_b200::rmsnorm",)


def load_rmsnorm(entrypoint: str) -> Callable[..., torch.Tensor]:
    """Closed registry: only declared entry points resolve, anything else is a ``KeyError``."""
    if entrypoint not in RMSNORM_ENTRYPOINTS:
        raise KeyError(f"unknown RMSNorm entry point {entrypoint!r}")
    return rmsnorm
