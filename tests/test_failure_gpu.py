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


def test_peer_barrier_that_nobody_answers_times_out_and_reports() -> None:
    """hst_peer_barrier for rank 0 of two, the second "rank" a plain buffer on the same GPU that no
    kernel ever writes back from: the bounded wait runs out, sets status bit 64,
    and the store into the other rank's words has landed. One GPU, one kernel; nothing waits on
    another launch. The wait is bounded at 20 ms here."""
    import ctypes

    require_cuda()
    lib = _native.library()
    device = torch.cuda.current_device()
    _native.status(device, clear=True)
    mine = torch.zeros(4, dtype=torch.int64, device="cuda")
    other = torch.zeros(4, dtype=torch.int64, device="cuda")
    words = (ctypes.c_void_p * 2)(mine.data_ptr(), other.data_ptr())
    _native.check(lib.hst_peer_barrier(words, 2, 0, 1, 5, 20_000_000, torch.cuda.current_stream().cuda_stream))
    bits = _native.status(device, clear=True)
    assert bits & 64, bits
    assert other.tolist() == [0, 0, 5, 0]  # slot 1, entry of rank 0
    assert mine.tolist() == [0, 0, 0, 0]
    assert _native.status(device) == 0
