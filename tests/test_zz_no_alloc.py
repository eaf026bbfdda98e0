"""The allocation-free split-K entry point against the ordinary split-K entry point.

Callers that cannot allocate device memory at call time (a process that reserved the whole GPU
at start-up, or an FFI binding of the C ABI without a device allocator) use
``hst_matmul_split_k_noalloc``: the FP32 partials live in a fixed array inside the library. Both
entry points run the same split-K kernel and the same fixed-order reduction, so their outputs
must agree bit for bit; each is also checked against the FP32 reference with the parity
tolerance of the other GEMM tests. Calls come in a row on one device, so a later call finds the
partials an earlier one left in the shared array: a 16-split call followed by a 2-split call on
the same M x N would expose a reduction that read stale slots. The file sorts last so pytest
collects it after every other test.
"""

from __future__ import annotations

import ctypes

import pytest
import torch

from heliostune_b200 import _native

pytestmark = pytest.mark.gpu


def _operands(m: int, n: int, k: int, seed: int) -> tuple[torch.Tensor, torch.Tensor]:
    g = torch.Generator(device="cuda").manual_seed(seed)
    a = (torch.randn((m, k), generator=g, device="cuda") / k**0.5).to(torch.float16)
    b = (torch.randn((k, n), generator=g, device="cuda") / k**0.5).to(torch.float16)
    return a, b


def _with_workspace(a: torch.Tensor, b: torch.Tensor, split: int) -> torch.Tensor:
    lib = _native.library()
    m, k = a.shape
    n = b.shape[1]
    config = _native.GemmConfig(_native.FAMILY_SPLIT_K, 16, 128, 64, 4, 3, 8, split)
    size = ctypes.c_size_t()
    _native.check(
        lib.hst_gemm_workspace_size(
            ctypes.byref(config), a.data_ptr(), a.stride(0), a.stride(1), b.data_ptr(), b.stride(0),
            b.stride(1), m, n, k, torch.cuda.current_device(), ctypes.byref(size),
        )
    )
    workspace = torch.empty(max(size.value, 1), dtype=torch.uint8, device="cuda")
    c = torch.empty((m, n), dtype=torch.float16, device="cuda")
    _native.check(
        lib.hst_matmul_split_k(
            16, 128, 64, 4, 3, split, a.data_ptr(), a.stride(0), a.stride(1), b.data_ptr(),
            b.stride(0), b.stride(1), c.data_ptr(), n, m, n, k, workspace.data_ptr(), size.value,
            torch.cuda.current_stream().cuda_stream,
        )
    )
    torch.cuda.synchronize()
    return c


def _without_allocation(a: torch.Tensor, b: torch.Tensor, split: int) -> torch.Tensor:
    lib = _native.library()
    m, k = a.shape
    n = b.shape[1]
    c = torch.empty((m, n), dtype=torch.float16, device="cuda")
    _native.check(
        lib.hst_matmul_split_k_noalloc(
            16, 128, 64, 4, 3, split, a.data_ptr(), a.stride(0), a.stride(1), b.data_ptr(),
            b.stride(0), b.stride(1), c.data_ptr(), n, m, n, k,
            torch.cuda.current_stream().cuda_stream,
        )
    )
    torch.cuda.synchronize()
    return c


def test_allocation_free_split_k_matches_the_workspace_entry_point() -> None:
    if not torch.cuda.is_available():
        pytest.skip("CUDA is unavailable")
    from tests.gpu_helpers import assert_gemm_parity

    # Calls in a row: each finds the previous call's partials in the shared array. The third
    # repeats the second's M x N with fewer splits, so slots 2..15 still hold 16-split partials.
    cases = ((31, 4096, 4096, 16, 1), (7, 3584, 18944, 16, 2), (7, 3584, 18944, 2, 3), (1, 4096, 4096, 4, 4))
    for m, n, k, split, seed in cases:
        a, b = _operands(m, n, k, seed)
        expected = _with_workspace(a, b, split)
        got = _without_allocation(a, b, split)
        assert torch.equal(got.view(torch.int16), expected.view(torch.int16)), (m, n, k, split)
        assert_gemm_parity(got, a, b)
        assert_gemm_parity(expected, a, b)
    assert _native.status(torch.cuda.current_device()) == 0


def test_allocation_free_split_k_rejects_sizes_beyond_its_array() -> None:
    if not torch.cuda.is_available():
        pytest.skip("CUDA is unavailable")
    a, b = _operands(31, 37888, 3584, 3)  # 16 splits x 31 x 37888 partials > 4 Mi floats
    with pytest.raises(ValueError, match="scratch array holds"):
        _without_allocation(a, b, 16)
