"""RMSNorm on the B200, and the closed registries that hand it out.

Two forms:

* the reference's own residual RMSNorm, ``y = bf16((z * rsqrt(mean(z^2) + 1e-5)) * gamma)`` with
  ``z = x + residual`` on BF16 ``(128, 4096)`` rows, registered as the ``torch.library`` op
  ``heliostune_fusion_v2::residual_rmsnorm`` and handed out by ``load_residual_rmsnorm`` under
  the reference's four entry-point names ``heliostune_fusion_v2::residual_rmsnorm_w{4,8,16,32}``
  (``src/heliostune/_fusion_gpu.py:49-208``, ``src/heliostune/fusion_kernels.py:28-82``); the op
  launches ``hst_residual_rmsnorm`` with 4, 8, 16 or 32 warps per row;
* the FP16 form without a residual that the QKV configuration measures,
  ``y = fp16((x * rsqrt(mean(x^2) + eps)) * gamma)``, for any ``[rows, hidden]`` input
  (``rmsnorm``, ``hst_rmsnorm``; registry ``load_rmsnorm``), also fused into the GEMM
  (``rmsnorm_matmul``).

Both sum the squares of a row in FP32.

And the gated-MLP projection of the reference's epilogue suite (``gated_mlp``,
``silu(x Wg^T) * (x Wu^T)`` in BF16, local_executor.py:1970-1979) as one weight-streaming launch
with the activation and product in its epilogue (``hst_gated_mlp_stream``), for M <= 64.
"""

from __future__ import annotations

from collections.abc import Callable
from types import MappingProxyType

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


# ----------------------------------------------------------------------------------------------
# The reference's residual RMSNorm
# ----------------------------------------------------------------------------------------------

#: Row shape and epsilon the reference's op is defined for (_fusion_gpu.py:76-109).
RESIDUAL_RMSNORM_SHAPE = (128, 4096)
RESIDUAL_RMSNORM_EPS = 1e-5


@torch.library.custom_op("heliostune_fusion_v2::residual_rmsnorm", mutates_args=())
def _residual_rmsnorm_op(x: torch.Tensor, residual: torch.Tensor, gamma: torch.Tensor, num_warps: int) -> torch.Tensor:
    """``bf16((z * rsqrt(mean(z^2) + 1e-5)) * gamma)``, ``z = x + residual``, one CTA of
    ``num_warps`` warps per row (``hst_residual_rmsnorm``)."""
    return residual_rmsnorm(x, residual, gamma, eps=RESIDUAL_RMSNORM_EPS, num_warps=num_warps)


@_residual_rmsnorm_op.register_fake
def _(x: torch.Tensor, residual: torch.Tensor, gamma: torch.Tensor, num_warps: int) -> torch.Tensor:
    return torch.empty_like(x)


def residual_rmsnorm(
    x: torch.Tensor,
    residual: torch.Tensor,
    gamma: torch.Tensor,
    *,
    eps: float = RESIDUAL_RMSNORM_EPS,
    num_warps: int = 8,
) -> torch.Tensor:
    """Residual RMSNorm of BF16 ``[rows, hidden]`` rows on the GPU, any row count and width:
    ``bf16((z * rsqrt(mean(z^2) + eps)) * gamma)`` with ``z = fp32(x) + fp32(residual)``. Inputs
    are never modified; the output is allocated per call."""
    if x.ndim != 2 or residual.shape != x.shape or gamma.ndim != 1 or gamma.shape[0] != x.shape[1]:
        raise ValueError("residual_rmsnorm expects x and residual [rows, hidden] and gamma [hidden]")
    if not x.dtype == residual.dtype == gamma.dtype == torch.bfloat16:
        raise ValueError("x, residual, and gamma must have dtype torch.bfloat16")
    if x.device.type != "cuda" or residual.device != x.device or gamma.device != x.device:
        raise ValueError("x, residual, and gamma must be on the same CUDA device")
    if x.stride(1) != 1 or residual.stride(1) != 1 or not gamma.is_contiguous():
        raise ValueError("residual_rmsnorm needs unit-stride rows and a contiguous gamma")
    rows, hidden = int(x.shape[0]), int(x.shape[1])
    y = torch.empty((rows, hidden), device=x.device, dtype=torch.bfloat16)
    with _device_guard(x.device):
        _native.check(
            _native.library().hst_residual_rmsnorm(
                x.data_ptr(),
                x.stride(0) if rows > 1 else hidden,
                residual.data_ptr(),
                residual.stride(0) if rows > 1 else hidden,
                gamma.data_ptr(),
                y.data_ptr(),
                hidden,
                rows,
                hidden,
                float(eps),
                int(num_warps),
                _stream(x.device),
            )
        )
    return y


def _validate_residual_rmsnorm_inputs(x: torch.Tensor, residual: torch.Tensor, gamma: torch.Tensor) -> None:
    """The reference op's input contract and messages (_fusion_gpu.py:96-116)."""
    if x.shape != RESIDUAL_RMSNORM_SHAPE or residual.shape != RESIDUAL_RMSNORM_SHAPE:
        raise ValueError("x and residual must have shape (128, 4096)")
    if gamma.shape != (RESIDUAL_RMSNORM_SHAPE[1],):
        raise ValueError("gamma must have shape (4096,)")
    if x.dtype != torch.bfloat16 or residual.dtype != torch.bfloat16 or gamma.dtype != torch.bfloat16:
        raise ValueError("x, residual, and gamma must have dtype torch.bfloat16")
    if not x.is_cuda or not residual.is_cuda or not gamma.is_cuda:
        raise ValueError("x, residual, and gamma must be CUDA tensors")
    if residual.device != x.device or gamma.device != x.device:
        raise ValueError("x, residual, and gamma must be on the same CUDA device")
    if not x.is_contiguous() or not residual.is_contiguous() or not gamma.is_contiguous():
        raise ValueError("x, residual, and gamma must be contiguous")


def _residual_rmsnorm_variant(num_warps: int) -> Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor]:
    def variant(x: torch.Tensor, residual: torch.Tensor, gamma: torch.Tensor) -> torch.Tensor:
        _validate_residual_rmsnorm_inputs(x, residual, gamma)
        return torch.ops.heliostune_fusion_v2.residual_rmsnorm(x, residual, gamma, num_warps)

    variant.__name__ = f"residual_rmsnorm_w{num_warps}"
    variant.__qualname__ = variant.__name__
    return variant


residual_rmsnorm_w4 = _residual_rmsnorm_variant(4)
residual_rmsnorm_w8 = _residual_rmsnorm_variant(8)
residual_rmsnorm_w16 = _residual_rmsnorm_variant(16)
residual_rmsnorm_w32 = _residual_rmsnorm_variant(32)

#: The reference's closed entry-point set (fusion_kernels.py:28-62), in its order.
RESIDUAL_RMSNORM_ENTRYPOINTS: MappingProxyType[str, Callable[..., torch.Tensor]] = MappingProxyType(
    {
        "heliostune_fusion_v2::residual_rmsnorm_w4": residual_rmsnorm_w4,
        "heliostune_fusion_v2::residual_rmsnorm_w8": residual_rmsnorm_w8,
        "heliostune_fusion_v2::residual_rmsnorm_w16": residual_rmsnorm_w16,
        "heliostune_fusion_v2::residual_rmsnorm_w32": residual_rmsnorm_w32,
    }
)


def load_residual_rmsnorm(entrypoint: str) -> Callable[..., torch.Tensor]:
    """Closed lookup of one of the reference's four entry points; anything else is a
    ``ValueError`` with the reference's message (fusion_kernels.py:65-82)."""
    try:
        return RESIDUAL_RMSNORM_ENTRYPOINTS[entrypoint]
    except (KeyError, TypeError) as exc:
        raise ValueError(f"unknown residual RMSNorm entrypoint: {entrypoint!r}") from exc


# ----------------------------------------------------------------------------------------------
# Gated-MLP projection with its epilogue
# ----------------------------------------------------------------------------------------------

#: Rows the fused gated-MLP kernel serves (the decode regime; UMMA N = M padded to 16..64).
GATED_MLP_M_LIMIT = 64


def gated_mlp(
    x: torch.Tensor,
    gate_weight: torch.Tensor,
    up_weight: torch.Tensor,
    *,
    block_m: int = 0,
    block_k: int = 64,
    num_stages: int = 0,
    split_k: int = 0,
) -> torch.Tensor:
    """``bf16(silu(x @ gate_weight.T) * (x @ up_weight.T))`` with FP32 accumulation, the gated-MLP
    epilogue suite's operation (local_executor.py:1970-1979; shapes ``x [batch, hidden]``,
    weights ``[intermediate, hidden]``, all BF16 row-major). One launch streams both weights
    once; the activation and the product happen on the FP32 sums before the only rounding.
    ``batch`` must be at most :data:`GATED_MLP_M_LIMIT`; ``hidden`` a multiple of 8."""
    if x.ndim != 2 or gate_weight.ndim != 2 or up_weight.shape != gate_weight.shape:
        raise ValueError("gated_mlp expects x [batch, hidden] and two weights [intermediate, hidden]")
    if gate_weight.shape[1] != x.shape[1]:
        raise ValueError(f"incompatible shapes: x {tuple(x.shape)} and weights {tuple(gate_weight.shape)}")
    if not x.dtype == gate_weight.dtype == up_weight.dtype == torch.bfloat16:
        raise ValueError("x and the weights must have dtype torch.bfloat16")
    if x.device.type != "cuda" or gate_weight.device != x.device or up_weight.device != x.device:
        raise ValueError("x and the weights must be on the same CUDA device")
    if not (x.is_contiguous() and gate_weight.is_contiguous() and up_weight.is_contiguous()):
        raise ValueError("x and the weights must be contiguous row-major tensors")
    m, k = int(x.shape[0]), int(x.shape[1])
    n = int(gate_weight.shape[0])
    if not 1 <= m <= GATED_MLP_M_LIMIT:
        raise ValueError(f"the fused gated MLP serves 1 <= batch <= {GATED_MLP_M_LIMIT}, got {m}")
    out = torch.empty((m, n), device=x.device, dtype=torch.bfloat16)
    with _device_guard(x.device):
        _native.check(
            _native.library().hst_gated_mlp_stream(
                block_m, block_k, num_stages, split_k,
                x.data_ptr(), k, gate_weight.data_ptr(), k, up_weight.data_ptr(), k,
                out.data_ptr(), n, m, n, k,
                _stream(x.device),
            )
        )
    return out


# ----------------------------------------------------------------------------------------------
# The FP16 form's registry
# ----------------------------------------------------------------------------------------------

RMSNORM_ENTRYPOINTS: tuple[str, ...] = ("heliostune_b200::rmsnorm",)


def load_rmsnorm(entrypoint: str) -> Callable[..., torch.Tensor]:
    """Closed registry: only declared entry points resolve, anything else is a ``KeyError``."""
    if entrypoint not in RMSNORM_ENTRYPOINTS:
        raise KeyError(f"unknown RMSNorm entry point {entrypoint!r}")
    return rmsnorm


def _main(argv: list[str] | None = None) -> None:
    """``python -m heliostune_b200.fusion {gated,residual} [--batch B] [--reps R]``: runs one op on
    seeded inputs of the reference's suite shapes (gated: x [B, 4096], weights [11008, 4096];
    residual: 128 x 4096) and prints the median event time of R launches, each after an L2
    flush. Meant for profiling a single kernel."""
    import argparse
    import json

    from heliostune_b200.timing import flush_buffer

    parser = argparse.ArgumentParser(description=_main.__doc__.split("\n")[0])
    parser.add_argument("op", choices=("gated", "residual"))
    parser.add_argument("--batch", type=int, default=8)
    parser.add_argument("--reps", type=int, default=3)
    args = parser.parse_args(argv)
    device = torch.device("cuda", torch.cuda.current_device())
    g = torch.Generator(device=device).manual_seed(17)
    if args.op == "gated":
        x = torch.randn((args.batch, 4096), generator=g, device=device).to(torch.bfloat16)
        gate = (torch.randn((11008, 4096), generator=g, device=device) / 64).to(torch.bfloat16)
        up = (torch.randn((11008, 4096), generator=g, device=device) / 64).to(torch.bfloat16)

        def run() -> torch.Tensor:
            return gated_mlp(x, gate, up)
    else:
        x = torch.randn(RESIDUAL_RMSNORM_SHAPE, generator=g, device=device).to(torch.bfloat16)
        r = torch.randn(RESIDUAL_RMSNORM_SHAPE, generator=g, device=device).to(torch.bfloat16)
        gamma = (1 + 0.02 * torch.randn((RESIDUAL_RMSNORM_SHAPE[1],), generator=g, device=device)).to(torch.bfloat16)

        def run() -> torch.Tensor:
            return residual_rmsnorm_w8(x, r, gamma)
    flush = flush_buffer(device)
    times = []
    for _ in range(args.reps):
        flush.zero_()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        run()
        end.record()
        torch.cuda.synchronize(device)
        times.append(start.elapsed_time(end) * 1e3)
    print(json.dumps({"op": args.op, "batch": args.batch, "us": sorted(times)[len(times) // 2]}))


if __name__ == "__main__":
    _main()
