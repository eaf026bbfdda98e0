"""Shared checks of the GPU parity tests."""

from __future__ import annotations

import pytest
import torch

from heliostune_b200.action_expansion import fp32_reference

#: The reference's elementwise tolerance (action_collection.py:37-38, tests/test_action_expansion.py:40).
ATOL = 1e-2
RTOL = 1e-2
#: Normwise bound of the build: max|C - C_ref| / max|C_ref|.
NORMWISE = 1e-2


def require_cuda() -> None:
    if not torch.cuda.is_available():
        pytest.skip("CUDA is unavailable")


def normwise(out: torch.Tensor, expected: torch.Tensor) -> float:
    scale = expected.abs().max().item()
    diff = (out.float() - expected).abs().max().item()
    return diff / scale if scale > 0 else diff


def assert_gemm_parity(out: torch.Tensor, a: torch.Tensor, b: torch.Tensor) -> float:
    """The reference's check (tests/test_action_expansion.py:29-40) plus the normwise bound."""
    expected = fp32_reference(a, b)
    assert out.shape == (a.shape[0], b.shape[1])
    assert out.dtype == torch.float16
    assert out.device == a.device
    assert bool(torch.isfinite(out).all().item())
    torch.testing.assert_close(out.float(), expected, atol=ATOL, rtol=RTOL)
    error = normwise(out, expected)
    assert error <= NORMWISE
    return error


def scaled_normal(shape: tuple[int, int], k: int, generator: torch.Generator) -> torch.Tensor:
    """N(0, 1) / sqrt(K) in FP16: the operand distribution of the measured grid."""
    return (torch.randn(shape, generator=generator, device="cuda") / k**0.5).to(torch.float16)
