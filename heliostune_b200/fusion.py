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
from heliostune_b200.kernel import _device_guard, _stream

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
    with _device_guard(x.device):
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
    *,
    fused: bool | None = None,
) -> torch.Tensor:
    """``RMSNorm(x; gamma, eps) @ W`` -- the RMSNorm feeding the QKV projection.

    Fused (weight-streaming candidates with ``block_m <= 128``; the default for
    ``block_m <= 32``, where it costs nothing over the GEMM alone): one launch of
    ``hst_rmsnorm_matmul_stream``, whose main loop rescales each x tile it loads by gamma and sums
    the squares of its rows, and whose epilogue multiplies the FP32 results by
    ``rsqrt(mean(x^2) + eps)`` -- no normalised copy of x, no second kernel. The products are
    rounded once, after the row factor, instead of the reference's intermediate FP16 rows. From
    64 rows on, rescaling the tiles in flight outlasts the stage it must hide behind, so the
    unfused form is the default there.

    Unfused (any other candidate, or ``fused=False``): the normalised rows are produced exactly as
    the reference's formula rounds them, ``fp16((x * rsqrt(mean(x^2) + eps)) * gamma)``, by the
    RMSNorm kernel into a per-call buffer that the GEMM candidate then consumes on the same stream.
    """
    from heliostune_b200.action_configs import StreamConfig
    from heliostune_b200.action_expansion import launch

    if w.ndim != 2 or w.shape[0] != x.shape[1]:
        raise ValueError(f"incompatible shapes: x {tuple(x.shape)} and W {tuple(w.shape)}")
    config = candidate.config
    can_fuse = (
        isinstance(config, StreamConfig)
        and config.block_m <= 128
        and x.shape[0] <= config.block_m
        and x.shape[1] % 8 == 0
        and x.stride(1) == 1
        and (x.shape[0] == 1 or x.stride(0) % 8 == 0)
        and x.data_ptr() % 16 == 0
        and w.is_contiguous()
        and w.shape[1] % 8 == 0
        and gamma.is_contiguous()
        and gamma.data_ptr() % 16 == 0
        and x.dtype == w.dtype == gamma.dtype == torch.float16
        and x.device == w.device == gamma.device
    )
    if fused is None:
        fused = can_fuse and config.block_m <= 32
    elif fused and not can_fuse:
        raise ValueError("the fused RMSNorm GEMM needs a stream candidate with block_m <= 128 and aligned row-major operands")
    if not fused:
        return launch(rmsnorm(x, gamma, eps), w, candidate)
    m, k = int(x.shape[0]), int(x.shape[1])
    n = int(w.shape[1])
    out = torch.empty((m, n), device=x.device, dtype=torch.float16)
    with _device_guard(x.device):
        _native.check(
            _native.library().hst_rmsnorm_matmul_stream(
                config.block_m,
                config.block_n,
                config.block_k,
                config.num_stages,
                config.split_k,
                x.data_ptr(),
                x.stride(0) if m > 1 else k,
                gamma.data_ptr(),
                float(eps),
                w.data_ptr(),
                n,
                out.data_ptr(),
                n,
                m,
                n,
                k,
                _stream(x.device),
            )
        )
    return out


RMSNORM_ENTRYPOINTS: tuple[str, ...] = ("heliostune_b200::rmsnorm",)


def load_rmsnorm(entrypoint: str) -> Callable[..., torch.Tensor]:
    """Closed registry: only declared entry points resolve, anything else is a ``KeyError``."""
    if entrypoint not in RMSNORM_ENTRYPOINTS:
        raise KeyError(f"unknown RMSNorm entry point {entrypoint!r}")
    return rmsnorm
