"""Failure detection on the GPU without a fault: a bounded wait that runs out reports through
the status word, and the context stays usable."""

from __future__ import annotations

import pytest
import torch

from heliostune_b200 import _native
from heliostune_b200.action_configs import NON_SPLIT_CANDIDATES
from heliostune_b200.action_expansion import launch
from tests.gpu_helpers import assert_gemm_parity, require_cuda

pytestmark = pytest.mark.gpu


def test_bounded_wait_reports_and_the_context_survives() -> None:
    require_cuda()
    lib = _native.library()
    device = torch.cuda.current_device()
    _native.status(device, clear=True)
    _native.check(lib.hst_probe_wait_timeout(20_000_000, torch.cuda.current_stream().cuda_stream))
    bits = _native.status(device, clear=True)
    assert bits & 16, bits
    assert _native.status(device) == 0
    a = torch.rand((64, 256), device="cuda", dtype=torch.float16)
    b = torch.rand((256, 256), device="cuda", dtype=torch.float16)
    assert_gemm_parity(launch(a, b, NON_SPLIT_CANDIDATES[0]), a, b)
    assert _native.status(device) == 0


def test_invalid_arguments_become_value_errors() -> None:
    require_cuda()
    lib = _native.library()
    with pytest.raises(ValueError, match="probe limit"):
        _native.check(lib.hst_probe_wait_timeout(5_000_000_000, None))
    with pytest.raises(ValueError, match="ldc"):
        _native.check(lib.hst_matmul_tile(128, 128, 64, 4, 5, 8, 1, 8, 1, 1, 8, 1, 1, 4, 4, 8, 8, None, 0, None))
