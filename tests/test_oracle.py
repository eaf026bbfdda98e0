"""The CPU oracle pinned against the reference's known-answer tests and golden vectors."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import oracle
from tests.conftest import GOLDEN, load_golden

CASES = ("edge_1x8x8", "edge_7x136x264", "edge_131x1032x520", "splitk_7x131x17", "splitk_31x131x1543")


@pytest.fixture(scope="module")
def gemm_cases() -> dict[str, np.ndarray]:
    return dict(np.load(GOLDEN / "gemm_cases.npz"))


@pytest.mark.parametrize("name", CASES)
def test_gemm_oracle_matches_golden_products(gemm_cases: dict[str, np.ndarray], name: str) -> None:
    a, b = gemm_cases[f"{name}_a"], gemm_cases[f"{name}_b"]
    rows = gemm_cases[f"{name}_crows"]
    expected = gemm_cases[f"{name}_c"]
    np.testing.assert_array_equal(oracle.gemm_fp32_reference(a, b)[rows], expected)
    if a.shape[0] * b.shape[1] <= 8192:
        np.testing.assert_array_equal(oracle.gemm_fp32_reference_c(a, b), expected)
    # The FP32 BLAS baseline differs from the FP64 sum only by FP32 rounding of partial sums.
    np.testing.assert_allclose(oracle.gemm_fp32_blas(a, b)[rows], expected, rtol=1e-5, atol=1e-6)


def test_gemm_oracle_handles_strided_operands(gemm_cases: dict[str, np.ndarray]) -> None:
    a = gemm_cases["strided_a_full"][:, ::2]
    b = gemm_cases["strided_b_full"][::2, ::2]
    expected = gemm_cases["strided_c"]
    np.testing.assert_array_equal(oracle.gemm_fp32_reference(a, b), expected)
    np.testing.assert_array_equal(oracle.gemm_fp32_reference_c(a, b), expected)


@pytest.mark.parametrize("name", CASES)
@pytest.mark.parametrize("splits", (4, 16))
def test_split_k_restatement_is_within_the_reference_tolerance(
    gemm_cases: dict[str, np.ndarray], name: str, splits: int
) -> None:
    a, b = gemm_cases[f"{name}_a"], gemm_cases[f"{name}_b"]
    rows = gemm_cases[f"{name}_crows"]
    out = oracle.gemm_split_k(a, b, 64, splits)[rows]
    assert oracle.within_tolerance(out, gemm_cases[f"{name}_c"], atol=1e-2, rtol=1e-2)
    assert oracle.normwise_error(out, gemm_cases[f"{name}_c"]) < 2e-3


def test_tolerance_known_answers() -> None:
    kat = load_golden("tolerance_kat.json")
    out = np.asarray(kat["output"], dtype=np.float16)
    exp = np.asarray(kat["expected"], dtype=np.float32)
    for case in kat["cases"]:
        assert oracle.within_tolerance(out, exp, atol=case["atol"], rtol=case["rtol"]) == case["within"]


def test_fp16_rounding_matches_ieee() -> None:
    rng = np.random.default_rng(5)
    values = np.concatenate(
        [
            rng.standard_normal(20000).astype(np.float32) * np.float32(3000),
            rng.standard_normal(5000).astype(np.float32) * np.float32(1e-5),  # subnormals
            np.asarray([65504, 65519.9, 65520, -65536, 2.0**-25, 2.0**-24, 0.0, -0.0], np.float32),
        ]
    )
    np.testing.assert_array_equal(oracle.f32_to_f16(values).view(np.uint16), values.astype(np.float16).view(np.uint16))


def test_rmsnorm_oracle_matches_the_reference_formula() -> None:
    """Without the residual the oracle is the reference's eager formula
    (local_executor.py:1982-1985); the golden output is what that function returned."""
    data = np.load(GOLDEN / "rmsnorm_bf16.npz")
    x, gamma = data["x"], data["gamma"]
    out = oracle.rmsnorm_reference(x, gamma, 1e-5, bf16=True)
    expected = data["expected_no_residual"]
    to_f32 = lambda v: (v.astype(np.uint32) << 16).view(np.float32)  # noqa: E731
    diff = np.abs(to_f32(out) - to_f32(expected))
    ulp = np.abs(to_f32(expected)) * 2.0**-7
    assert np.all(diff <= ulp + 1e-30)
    assert np.mean(out == expected) > 0.995


def test_residual_rmsnorm_oracle_matches_the_reference_output() -> None:
    """With the residual (z = x + r, eps 1e-5, BF16) the oracle returns the bits the reference's
    own function returned on the same inputs (local_executor.py:1982-1985)."""
    data = np.load(GOLDEN / "rmsnorm_bf16.npz")
    out = oracle.rmsnorm_reference(data["x"], data["gamma"], 1e-5, bf16=True, residual=data["residual"])
    assert np.mean(out == data["expected"]) > 0.999
    to_f32 = lambda v: (v.astype(np.uint32) << 16).view(np.float32)  # noqa: E731
    assert np.all(np.abs(to_f32(out) - to_f32(data["expected"])) <= np.abs(to_f32(data["expected"])) * 2.0**-7 + 1e-30)


def test_rmsnorm_fp16_oracle_is_the_fp64_formula() -> None:
    rng = np.random.default_rng(3)
    x = rng.standard_normal((4, 4096)).astype(np.float16)
    gamma = (1 + 0.1 * rng.standard_normal(4096)).astype(np.float16)
    xf = x.astype(np.float64)
    inv = 1.0 / np.sqrt(np.mean(xf * xf, axis=1, keepdims=True) + 1e-6)
    expected = (xf * inv * gamma.astype(np.float64)).astype(np.float16)
    out = oracle.rmsnorm_reference(x, gamma, 1e-6)
    assert np.mean(out.view(np.uint16) == expected.view(np.uint16)) > 0.999
