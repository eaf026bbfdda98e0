"""The reference's residual RMSNorm entry points: the closed registry, the ``torch.library`` op's
namespace and schema, and the input contract (no GPU needed); the kernel against the oracle's BF16
path and the reference's own tolerance on the GPU."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from heliostune_b200 import fusion
from tests.conftest import GOLDEN

ENTRYPOINTS = tuple(f"heliostune_fusion_v2::residual_rmsnorm_w{w}" for w in (4, 8, 16, 32))


def test_registry_is_exactly_the_reference_entrypoints() -> None:
    assert tuple(fusion.RESIDUAL_RMSNORM_ENTRYPOINTS) == ENTRYPOINTS
    for name in ENTRYPOINTS:
        assert fusion.load_residual_rmsnorm(name).__name__ == name.split("::")[1]
    for bad in ("heliostune_fusion_v2::residual_rmsnorm", "heliostune_fusion_v2::residual_rmsnorm_w2", "", 4):
        with pytest.raises(ValueError, match="unknown residual RMSNorm entrypoint"):
            fusion.load_residual_rmsnorm(bad)  # type: ignore[arg-type]
    with pytest.raises(TypeError):
        fusion.RESIDUAL_RMSNORM_ENTRYPOINTS["x"] = fusion.rmsnorm  # type: ignore[index]


def test_registered_op_has_the_reference_namespace_and_no_mutation() -> None:
    schema = torch.ops.heliostune_fusion_v2.residual_rmsnorm.default._schema
    assert schema.name == "heliostune_fusion_v2::residual_rmsnorm"
    assert [a.name for a in schema.arguments] == ["x", "residual", "gamma", "num_warps"]
    assert not any(a.alias_info is not None and a.alias_info.is_write for a in schema.arguments)


def test_inputs_are_checked_in_the_reference_order() -> None:
    variant = fusion.load_residual_rmsnorm(ENTRYPOINTS[0])
    x = torch.zeros((128, 4096), dtype=torch.bfloat16)
    gamma = torch.zeros(4096, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match=r"shape \(128, 4096\)"):
        variant(x[:64], x[:64], gamma)
    with pytest.raises(ValueError, match=r"gamma must have shape \(4096,\)"):
        variant(x, x, gamma[:8])
    with pytest.raises(ValueError, match="dtype torch.bfloat16"):
        variant(x.half(), x, gamma)
    with pytest.raises(ValueError, match="must be CUDA tensors"):
        variant(x, x, gamma)


gpu = pytest.mark.gpu


def _bf16_inputs(rows: int, hidden: int, seed: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn((rows, hidden), generator=g, device="cuda").to(torch.bfloat16)
    residual = torch.randn((rows, hidden), generator=g, device="cuda").to(torch.bfloat16)
    gamma = (1.0 + 0.02 * torch.randn((hidden,), generator=g, device="cuda")).to(torch.bfloat16)
    return x, residual, gamma


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def _f32(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


@gpu
@pytest.mark.parametrize("entrypoint", ENTRYPOINTS)
def test_reference_entrypoints_match_the_fp32_formula_and_the_oracle(entrypoint: str) -> None:
    """The reference's GPU test (tests/test_fusion_kernels.py:481-507) on this kernel, plus the
    oracle within one BF16 ulp and bit-equal for nearly every element."""
    from oracle import oracle
    from tests.gpu_helpers import require_cuda

    require_cuda()
    torch.manual_seed(17)
    x = torch.randn((128, 4096), device="cuda", dtype=torch.bfloat16)
    residual = torch.randn_like(x)
    gamma = (1.0 + 0.02 * torch.randn((4096,), device="cuda")).to(torch.bfloat16)
    x0, r0, g0 = x.clone(), residual.clone(), gamma.clone()
    z = x.float() + residual.float()
    mean_square = torch.mean(z * z, dim=-1, keepdim=True, dtype=torch.float32)
    expected = (z * torch.rsqrt(mean_square + 1e-5) * gamma.float()).to(torch.bfloat16)
    actual = fusion.load_residual_rmsnorm(entrypoint)(x, residual, gamma)
    assert actual.shape == (128, 4096) and actual.dtype == torch.bfloat16
    torch.testing.assert_close(actual, expected, atol=1e-5, rtol=0.0078125)
    ref = oracle.rmsnorm_reference(_bits(x), _bits(gamma), 1e-5, bf16=True, residual=_bits(residual))
    got = _bits(actual)
    assert np.all(np.abs(_f32(got) - _f32(ref)) <= np.abs(_f32(ref)) * 2.0**-7 + 1e-30)
    assert np.mean(got == ref) > 0.99
    for before, after in ((x0, x), (r0, residual), (g0, gamma)):
        assert torch.equal(before.view(torch.int16), after.view(torch.int16))
    again = fusion.load_residual_rmsnorm(entrypoint)(x, residual, gamma)
    assert torch.equal(actual.view(torch.int16), again.view(torch.int16))


@gpu
def test_golden_fixture_of_the_reference_function() -> None:
    """The bits the reference's own function returned (tests/golden/rmsnorm_bf16.npz)."""
    from tests.gpu_helpers import require_cuda

    require_cuda()
    data = np.load(GOLDEN / "rmsnorm_bf16.npz")
    as_bf16 = lambda a: torch.from_numpy(a.view(np.int16)).view(torch.bfloat16).cuda()  # noqa: E731
    for warps in (4, 8, 16, 32):
        out = fusion.residual_rmsnorm(as_bf16(data["x"]), as_bf16(data["residual"]), as_bf16(data["gamma"]), num_warps=warps)
        got, expected = _bits(out), data["expected"]
        assert np.all(np.abs(_f32(got) - _f32(expected)) <= np.abs(_f32(expected)) * 2.0**-7 + 1e-30)
        assert np.mean(got == expected) > 0.99


@gpu
@pytest.mark.parametrize("shape", ((1, 4096), (3, 1000), (5, 4104), (300, 8192), (2, 40000), (7, 24)))
@pytest.mark.parametrize("warps", (1, 4, 32))
def test_any_row_count_and_width_against_the_oracle(shape: tuple[int, int], warps: int) -> None:
    """Vector kernel (widths divisible by 8) and the scalar kernel (others, or too wide a row for
    the warps given) against the oracle."""
    from oracle import oracle
    from tests.gpu_helpers import require_cuda

    require_cuda()
    rows, hidden = shape
    x, residual, gamma = _bf16_inputs(rows, hidden, seed=rows * 31 + hidden)
    out = fusion.residual_rmsnorm(x, residual, gamma, num_warps=warps)
    ref = oracle.rmsnorm_reference(_bits(x), _bits(gamma), 1e-5, bf16=True, residual=_bits(residual))
    got = _bits(out)
    assert np.all(np.abs(_f32(got) - _f32(ref)) <= np.abs(_f32(ref)) * 2.0**-7 + 1e-30)
    assert np.mean(got == ref) > 0.99


@gpu
def test_strided_rows_and_bad_arguments() -> None:
    from heliostune_b200 import _native
    from tests.gpu_helpers import require_cuda

    require_cuda()
    x, residual, gamma = _bf16_inputs(64, 2 * 4096, seed=9)
    xs, rs = x[:, :4096], residual[:, 4096:]  # row stride 8192
    out = fusion.residual_rmsnorm(xs, rs, gamma[:4096].contiguous())
    dense = fusion.residual_rmsnorm(xs.contiguous(), rs.contiguous(), gamma[:4096].contiguous())
    assert torch.equal(out.view(torch.int16), dense.view(torch.int16))
    lib = _native.library()
    stream = torch.cuda.current_stream().cuda_stream
    args = (x.data_ptr(), 4096, residual.data_ptr(), 4096, gamma.data_ptr(), out.data_ptr(), 4096)
    assert lib.hst_residual_rmsnorm(*args, 64, 4096, 1e-5, 0, stream) == _native.HST_ERR_INVALID
    assert lib.hst_residual_rmsnorm(*args, 64, 4096, 1e-5, 33, stream) == _native.HST_ERR_INVALID
    assert lib.hst_residual_rmsnorm(*args, 64, 4096, -1.0, 8, stream) == _native.HST_ERR_INVALID
    assert lib.hst_residual_rmsnorm(*args, 0, 4096, 1e-5, 8, stream) == _native.HST_OK
