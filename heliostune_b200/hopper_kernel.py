"""Drop-in for ``heliostune.hopper_kernel``: the persistent tile-scheduler GEMM and the
pre-timing correctness gate.

``hopper_matmul`` has the signature, validation and error messages of
``src/heliostune/hopper_kernel.py:236-290``: row-major contiguous inputs with K and N multiples of
8 (the 16-byte row alignment a TMA tensor map needs). On a B200 the launch runs the persistent
tcgen05 kernel through ``hst_matmul_persistent``: one CTA per SM walks the output tiles in
``group_m`` raster order, with a double-buffered TMEM accumulator so each tile's epilogue
overlaps the next main loop.

``validate_candidate_kernels`` / ``assert_candidate_kernels_correct`` restate the reference's
gate (``hopper_kernel.py:413-623``): every candidate runs on a small sample of workloads against
an FP32 reference before anything is timed; a failure or an exception is one journal entry,
never retried. Here the candidates are ``ActionCandidate`` values of every family of this
library (the skinny atomic GEMV the reference also gates is not built).
"""

from __future__ import annotations

from collections.abc import Callable, Sequence
from dataclasses import dataclass

import torch

from heliostune_b200 import _native
from heliostune_b200.configs import TENSOR_DESCRIPTOR_ALIGNMENT, HopperGemmConfig, Workload
from heliostune_b200.kernel import _device_guard, _stream, _validate


def hopper_matmul(a: torch.Tensor, b: torch.Tensor, config: HopperGemmConfig) -> torch.Tensor:
    """Multiply two CUDA FP16 matrices with the persistent candidate kernel."""
    m, n, k = _validate(a, b)
    if not a.is_contiguous() or not b.is_contiguous():
        raise ValueError("tensor descriptors require row-major contiguous inputs")
    if k % TENSOR_DESCRIPTOR_ALIGNMENT or n % TENSOR_DESCRIPTOR_ALIGNMENT:
        raise ValueError(
            "tensor descriptors require 16-byte aligned leading strides: "
            f"K={k} and N={n} must both be multiples of {TENSOR_DESCRIPTOR_ALIGNMENT}"
        )
    output = torch.empty((m, n), device=a.device, dtype=torch.float16)
    with _device_guard(a.device):
        _native.check(
            _native.library().hst_matmul_persistent(
                config.block_m,
                config.block_n,
                config.block_k,
                config.num_warps,
                config.num_stages,
                config.group_m,
                a.data_ptr(),
                b.data_ptr(),
                output.data_ptr(),
                m,
                n,
                k,
                _stream(a.device),
            )
        )
    return output


@dataclass(frozen=True, slots=True)
class KernelValidation:
    """One candidate/workload correctness outcome (``hopper_kernel.py:413-433``)."""

    kernel: str
    config_key: str
    workload_key: str
    correct: bool
    max_abs_error: float | None = None
    error: str | None = None

    def to_dict(self) -> dict[str, object]:
        return {
            "kernel": self.kernel,
            "config_key": self.config_key,
            "workload_key": self.workload_key,
            "correct": self.correct,
            "max_abs_error": self.max_abs_error,
            "error": self.error,
        }


@torch.inference_mode()
def validate_candidate_kernels(
    gpu: str | None = None,
    *,
    candidates_for: Callable[[Workload], Sequence[object]] | None = None,
    workloads: Sequence[Workload] | None = None,
    atol: float = 1e-2,
    rtol: float = 1e-2,
    tensor_seed: int = 0,
) -> list[KernelValidation]:
    """Check every candidate ``candidates_for(workload)`` offers (default: the B200 tuner's pool)
    on every workload of ``workloads`` (default: :func:`configs.validation_workloads`) against the
    FP32 product of seeded uniform(-1, 1) FP16 operands, elementwise within ``atol + rtol |ref|``.
    The GPU is checked (a B200 when ``gpu`` names one) before any tensor is allocated."""
    from heliostune_b200.action_configs import b200_candidates_for
    from heliostune_b200.action_expansion import fp32_reference, launch
    from heliostune_b200.configs import validation_workloads
    from heliostune_b200.errors import ProtocolError
    from heliostune_b200.kernel import _within_tolerance, get_hardware_profile, require_b200

    if not (atol >= 0 and rtol >= 0):
        raise ProtocolError("atol and rtol must be non-negative")
    if type(tensor_seed) is not int or tensor_seed < 0:
        raise ProtocolError("tensor_seed must be a non-negative integer")
    device = torch.device("cuda", torch.cuda.current_device())
    profile = get_hardware_profile(gpu, device)
    if gpu is not None:
        require_b200(profile)
    offered = candidates_for or b200_candidates_for
    sample = validation_workloads() if workloads is None else tuple(workloads)
    if not sample:
        raise ProtocolError("validation workload manifest must not be empty")
    results: list[KernelValidation] = []
    for index, workload in enumerate(sample):
        torch.manual_seed(tensor_seed + index)
        a = torch.empty((workload.m, workload.k), device=device, dtype=torch.float16).uniform_(-1.0, 1.0)
        b = torch.empty((workload.k, workload.n), device=device, dtype=torch.float16).uniform_(-1.0, 1.0)
        expected = fp32_reference(a, b)
        for candidate in offered(workload):
            kernel, key = candidate.family, candidate.key  # type: ignore[attr-defined]
            try:
                output = launch(a, b, candidate)  # type: ignore[arg-type]
                torch.cuda.synchronize(device)
            except Exception as exc:  # noqa: BLE001 -- journaled, never retried
                results.append(KernelValidation(kernel, key, workload.key, False, error=f"{type(exc).__name__}: {exc}"))
                continue
            if not bool(torch.isfinite(output).all().item()):
                results.append(
                    KernelValidation(kernel, key, workload.key, False, error="correctness check failed: non-finite output")
                )
                continue
            difference = (output.float() - expected).abs()
            max_abs = float(difference.max().item()) if difference.numel() else 0.0
            if not _within_tolerance(difference, expected, atol=atol, rtol=rtol):
                results.append(
                    KernelValidation(
                        kernel, key, workload.key, False, max_abs_error=max_abs,
                        error=f"correctness check failed (atol={atol}, rtol={rtol})",
                    )
                )
                continue
            results.append(KernelValidation(kernel, key, workload.key, True, max_abs_error=max_abs))
            del output, difference
        del expected, a, b
    return results


def assert_candidate_kernels_correct(
    gpu: str | None = None,
    *,
    candidates_for: Callable[[Workload], Sequence[object]] | None = None,
    workloads: Sequence[Workload] | None = None,
    atol: float = 1e-2,
    rtol: float = 1e-2,
    tensor_seed: int = 0,
) -> list[KernelValidation]:
    """:func:`validate_candidate_kernels`, raising ``ProtocolError`` naming the first failures:
    the call a benchmark makes before it starts timing (``hopper_kernel.py:590-623``)."""
    from heliostune_b200.errors import ProtocolError

    results = validate_candidate_kernels(
        gpu, candidates_for=candidates_for, workloads=workloads, atol=atol, rtol=rtol, tensor_seed=tensor_seed
    )
    failures = [r for r in results if not r.correct]
    if failures:
        detail = "; ".join(f"{f.kernel}[{f.config_key}]@{f.workload_key}: {f.error}" for f in failures[:8])
        raise ProtocolError(f"{len(failures)} of {len(results)} candidate kernel checks failed: {detail}")
    return results
