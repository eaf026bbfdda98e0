"""Parity over the whole measured grid: every candidate the tuner's pool offers for each of the 96
shapes, at full size, against the FP32 product and against cuBLAS ``torch.matmul``.

For each shape (seeded N(0, 1)/sqrt(K) FP16 operands) every pool candidate runs on the full
problem; a block of rows (all rows up to M = 128, else one row per 128-row band at an offset that
moves from band to band, plus the last row) is compared with

* the reference's check value (FP32 product, TF32 off): elementwise ``1e-2 + 1e-2 |C|`` and
  normwise ``max|C - C_ref| / max|C_ref| <= 1e-2``;
* the exact product (FP64 on the same rows): the normwise error is no larger than cuBLAS
  ``torch.matmul``'s on the same inputs and rows. Both accumulate in FP32 and round once to
  FP16, so the largest error is an FP16 rounding of the same exact value in almost every case;
  on the B200 the two maxima are equal for 448 of the 540 (shape, candidate) pairs and ours is
  smaller for the rest.
"""

from __future__ import annotations

import math

import pytest
import torch

from heliostune_b200 import _native
from heliostune_b200.action_configs import b200_candidates_for
from heliostune_b200.action_expansion import fp32_reference, launch
from heliostune_b200.configs import GRID_WORKLOADS, Workload
from tests.gpu_helpers import ATOL, NORMWISE, RTOL, require_cuda

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _cuda() -> None:
    require_cuda()
    _native.library()


def sampled_rows(m: int) -> list[int]:
    if m <= 128:
        return list(range(m))
    bands = -(-m // 128)
    return sorted({min(m - 1, band * 128 + (band * 37) % 128) for band in range(bands)} | {m - 1})[:129]


def _normwise(out: torch.Tensor, exact: torch.Tensor) -> float:
    return (out.double() - exact).abs().max().item() / exact.abs().max().item()


@pytest.mark.parametrize("workload", GRID_WORKLOADS, ids=lambda w: w.key)
def test_every_pool_candidate_on_the_grid_shape(workload: Workload) -> None:
    g = torch.Generator(device="cuda").manual_seed(workload.m * 131 + workload.n + workload.k)
    a = (torch.randn((workload.m, workload.k), generator=g, device="cuda") / math.sqrt(workload.k)).half()
    b = (torch.randn((workload.k, workload.n), generator=g, device="cuda") / math.sqrt(workload.k)).half()
    index = torch.tensor(sampled_rows(workload.m), device="cuda")
    a_rows = a.index_select(0, index)
    expected = fp32_reference(a_rows, b)
    exact = a_rows.double() @ b.double()
    cublas_error = _normwise(torch.matmul(a, b).index_select(0, index), exact)
    candidates = b200_candidates_for(workload)
    assert candidates
    for candidate in candidates:
        out = launch(a, b, candidate)
        assert out.shape == (workload.m, workload.n) and out.dtype == torch.float16
        rows = out.index_select(0, index)
        assert bool(torch.isfinite(rows).all().item()), candidate.key
        torch.testing.assert_close(rows.float(), expected, atol=ATOL, rtol=RTOL, msg=candidate.key)
        scale = expected.abs().max().item()
        assert (rows.float() - expected).abs().max().item() <= NORMWISE * scale, candidate.key
        error = _normwise(rows, exact)
        assert error <= cublas_error, (candidate.key, error, cublas_error)
