"""The gated-MLP projection with its epilogue (``fusion.gated_mlp``, ``hst_gated_mlp_stream``)
against the reference's formula, ``bf16(silu(x Wg^T) * (x Wu^T))`` with FP32 matmuls
(local_executor.py:1970-1979), on the epilogue suite's case (batch 8, hidden 4096,
intermediate 11008, BF16, tolerance 0.02/0.02) and on ragged shapes for every tile and split."""

from __future__ import annotations

import pytest
import torch

from heliostune_b200 import fusion

gpu = pytest.mark.gpu


def test_inputs_are_checked_before_any_cuda_work() -> None:
    x = torch.zeros((8, 64), dtype=torch.bfloat16)
    w = torch.zeros((32, 64), dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="two weights"):
        fusion.gated_mlp(x, w, w[:16])
    with pytest.raises(ValueError, match="incompatible shapes"):
        fusion.gated_mlp(x[:, :32], w, w)
    with pytest.raises(ValueError, match="bfloat16"):
        fusion.gated_mlp(x.half(), w, w)
    with pytest.raises(ValueError, match="same CUDA device"):
        fusion.gated_mlp(x, w, w)


def _operands(m: int, k: int, n: int, seed: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn((m, k), generator=g, device="cuda").to(torch.bfloat16)
    gate = (torch.randn((n, k), generator=g, device="cuda") / k**0.5).to(torch.bfloat16)
    up = (torch.randn((n, k), generator=g, device="cuda") / k**0.5).to(torch.bfloat16)
    return x, gate, up


def _reference(x: torch.Tensor, gate: torch.Tensor, up: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """The reference's BF16 output (FP32 matmuls, TF32 off) and the exact value (FP64)."""
    previous = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        g = torch.mm(x.float(), gate.float().T)
        u = torch.mm(x.float(), up.float().T)
    finally:
        torch.backends.cuda.matmul.allow_tf32 = previous
    expected = (torch.nn.functional.silu(g) * u).to(torch.bfloat16)
    g64 = torch.mm(x.double(), gate.double().T)
    exact = g64 * torch.sigmoid(g64) * torch.mm(x.double(), up.double().T)
    return exact, expected


def _check(out: torch.Tensor, x: torch.Tensor, gate: torch.Tensor, up: torch.Tensor) -> None:
    exact, expected = _reference(x, gate, up)
    assert out.shape == expected.shape and out.dtype == torch.bfloat16
    torch.testing.assert_close(out, expected, atol=0.02, rtol=0.02)  # the suite's policy
    # One BF16 ulp of the exact value, plus 1e-4 absolute: where the gate or up dot product
    # cancels to ~1e-5 the FP32 accumulation over K (any order, cuBLAS's too) decides the bits.
    bound = exact.abs() * 2.0**-7 + 1e-4
    err = (out.double() - exact).abs()
    assert bool((err <= bound).all()), (err - bound).max().item()


@gpu
def test_epilogue_suite_case() -> None:
    from tests.gpu_helpers import require_cuda

    require_cuda()
    x, gate, up = _operands(8, 4096, 11008, seed=17)
    copies = (x.clone(), gate.clone(), up.clone())
    out = fusion.gated_mlp(x, gate, up)
    _check(out, x, gate, up)
    _, expected = _reference(x, gate, up)
    assert (out == expected).float().mean().item() > 0.99
    for before, after in zip(copies, (x, gate, up), strict=True):
        assert torch.equal(before.view(torch.int16), after.view(torch.int16))
    again = fusion.gated_mlp(x, gate, up)
    assert torch.equal(out.view(torch.int16), again.view(torch.int16))


@gpu
@pytest.mark.parametrize("m", (1, 5, 16, 17, 32, 33, 64))
@pytest.mark.parametrize("block_k", (64, 128))
@pytest.mark.parametrize("split_k", (0, 1, 2, 4))
def test_rows_tiles_and_splits_on_a_ragged_shape(m: int, block_k: int, split_k: int) -> None:
    from tests.gpu_helpers import require_cuda

    require_cuda()
    x, gate, up = _operands(m, 1000, 1000, seed=m * 7 + split_k)  # N past the last 128-column tile
    out = fusion.gated_mlp(x, gate, up, block_k=block_k, split_k=split_k)
    _check(out, x, gate, up)
    wider = fusion.gated_mlp(x, gate, up, block_m=64, block_k=block_k, split_k=split_k)
    _check(wider, x, gate, up)


@gpu
def test_bad_arguments_are_rejected() -> None:
    from heliostune_b200 import _native
    from tests.gpu_helpers import require_cuda

    require_cuda()
    x, gate, up = _operands(65, 256, 256, seed=1)
    with pytest.raises(ValueError, match="batch <= 64"):
        fusion.gated_mlp(x, gate, up)
    x = x[:16].contiguous()
    for kwargs, message in (
        ({"block_m": 8}, "block_m"),
        ({"block_k": 32}, "block_k"),
        ({"split_k": 3}, "split_k"),
        ({"num_stages": 99}, "num_stages"),
    ):
        with pytest.raises(ValueError, match=message):
            fusion.gated_mlp(x, gate, up, **kwargs)
    assert _native.status(torch.cuda.current_device()) == 0
