"""Drop-in for ``heliostune.hopper_kernel.hopper_matmul``: the persistent tile-scheduler GEMM.

Same signature, validation and error messages as ``src/heliostune/hopper_kernel.py:236-290``:
row-major contiguous inputs with K and N multiples of 8 (the 16-byte row alignment a TMA tensor
map needs). On a B200 the launch runs the persistent tcgen05 kernel through
``hst_matmul_persistent``: one CTA per SM walks the output tiles in ``group_m`` raster order,
with a double-buffered TMEM accumulator so each tile's epilogue overlaps the next main loop.
"""

from __future__ import annotations

import torch

from heliostune_b200 import _native
from heliostune_b200.configs import TENSOR_DESCRIPTOR_ALIGNMENT, HopperGemmConfig
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
