"""GPU parity of the RMSNorm kernel against the oracle (small) and the FP32 formula (full size)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from heliostune_b200 import _native
from heliostune_b200.fusion import load_rmsnorm, rmsnorm
from oracle import oracle
from tests.gpu_helpers import require_cuda

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _cuda() -> None:
    require_cuda()
    _native.library()


def _inputs(rows: int, hidden: int, seed: int) -> tuple[torch.Tensor, torch.Tensor]:
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn((rows, hidden), generator=g, device="cuda").to(torch.float16)
    gamma = (1.0 + 0.1 * torch.randn((hidden,), generator=g, device="cuda")).to(torch.float16)
    return x, gamma


@pytest.mark.parametrize("shape", ((4, 4096), (1, 8192), (3, 1000), (5, 4104), (2, 40000)))
def test_matches_the_oracle(shape: tuple[int, int]) -> None:
    x, gamma = _inputs(*shape, seed=shape[0])
    y = rmsnorm(x, gamma, 1e-6).cpu().numpy()
    expected = oracle.rmsnorm_reference(x.cpu().numpy(), gamma.cpu().numpy(), 1e-6)
    # within one FP16 ulp of the FP64 formula, and almost always the same bits
    ulp = np.abs(expected.astype(np.float32)) * 2.0**-10 + 2.0**-24
    assert np.all(np.abs(y.astype(np.float32) - expected.astype(np.float32)) <= ulp)
    assert np.mean(y.view(np.uint16) == expected.view(np.uint16)) > 0.99


@pytest.mark.parametrize("rows", (1, 4096, 65536))
@pytest.mark.parametrize("hidden", (4096, 8192))
def test_full_size_against_the_fp32_formula(rows: int, hidden: int) -> None:
    x, gamma = _inputs(rows, hidden, seed=rows + hidden)
    x0 = x.clone()
    y = rmsnorm(x, gamma, 1e-6)
    xf = x.float()
    expected = (xf * torch.rsqrt((xf * xf).mean(dim=-1, keepdim=True) + 1e-6) * gamma.float()).to(torch.float16)
    torch.testing.assert_close(y, expected, atol=1e-5, rtol=2.0**-9)
    assert torch.equal(rmsnorm(x, gamma, 1e-6).view(torch.int16), y.view(torch.int16))
    assert torch.equal(x.view(torch.int16), x0.view(torch.int16))


@pytest.mark.parametrize("rows", (1, 128, 4096))
def test_rmsnorm_feeding_the_qkv_gemm(rows: int) -> None:
    from heliostune_b200.action_configs import b200_candidates_for
    from heliostune_b200.action_expansion import fp32_reference
    from heliostune_b200.configs import Workload
    from heliostune_b200.fusion import rmsnorm_matmul
    from tests.gpu_helpers import assert_gemm_parity

    x, gamma = _inputs(rows, 4096, seed=rows)
    g = torch.Generator(device="cuda").manual_seed(7)
    w = (torch.randn((4096, 6144), generator=g, device="cuda") / 64).to(torch.float16)
    xf = x.float()
    normalised = (xf * torch.rsqrt((xf * xf).mean(dim=-1, keepdim=True) + 1e-6) * gamma.float()).to(torch.float16)
    workload = Workload(m=rows, n=6144, k=4096, model="llama-3-8b", projection="attention-qkv", regime="m")
    for candidate in b200_candidates_for(workload)[:4]:
        out = rmsnorm_matmul(x, gamma, w, candidate)
        assert_gemm_parity(out, normalised, w)
        # and against the FP32 product of the unrounded normalised rows
        exact = fp32_reference((xf * torch.rsqrt((xf * xf).mean(dim=-1, keepdim=True) + 1e-6) * gamma.float()), w.float())
        assert (out.float() - exact).abs().max().item() <= 1e-2 * exact.abs().max().item()


def test_registry_is_closed() -> None:
    assert load_rmsnorm("heliostune_b200::rmsnorm") is rmsnorm
    with pytest.raises(KeyError):
        load_rmsnorm("heliostune_fusion_v2::residual_rmsnorm_w4")


@pytest.mark.parametrize("rows", (1, 7, 16, 31, 64, 100, 128))
@pytest.mark.parametrize("split", (0, 1, 3, 4))
@pytest.mark.parametrize("nk", ((6144, 4096), (1000, 1000)), ids=lambda s: f"n{s[0]}k{s[1]}")
def test_rmsnorm_prologue_inside_the_stream_gemm(rows: int, split: int, nk: tuple[int, int]) -> None:
    """The fused kernel against the FP32 formula: the row factor applied after the GEMM."""
    from heliostune_b200.action_configs import ActionCandidate, StreamConfig, stream_block_m
    from heliostune_b200.action_expansion import fp32_reference
    from heliostune_b200.fusion import rmsnorm_matmul

    n, k = nk
    x, gamma = _inputs(rows, k, seed=rows * 7 + split)
    g = torch.Generator(device="cuda").manual_seed(11)
    w = (torch.randn((k, n), generator=g, device="cuda") / k**0.5).to(torch.float16)
    x0 = x.clone()
    xf = x.float()
    exact = fp32_reference(xf * torch.rsqrt((xf * xf).mean(dim=-1, keepdim=True) + 1e-6) * gamma.float(), w.float())
    bm = stream_block_m(rows)
    for block_n, block_k in ((128, 64), (128, 128), (256, 64)):
        if block_n == 256 and bm not in (64, 128):
            continue
        candidate = ActionCandidate(StreamConfig(bm, block_n, block_k, 4, 4, split))
        out = rmsnorm_matmul(x, gamma, w, candidate, 1e-6, fused=True)
        err = (out.float() - exact).abs()
        assert bool(torch.all(err <= 1e-2 + 1e-2 * exact.abs())), (block_n, block_k, err.max().item())
        assert err.max().item() <= 1e-2 * exact.abs().max().item()
        assert torch.equal(out.view(torch.int16), rmsnorm_matmul(x, gamma, w, candidate, 1e-6, fused=True).view(torch.int16))
        unfused = rmsnorm_matmul(x, gamma, w, candidate, 1e-6, fused=False)
        assert (out.float() - unfused.float()).abs().max().item() <= 1e-2 * exact.abs().max().item()
    assert torch.equal(x.view(torch.int16), x0.view(torch.int16))


def test_rmsnorm_prologue_rejects_what_it_cannot_fuse() -> None:
    from heliostune_b200.action_configs import ActionCandidate, StreamConfig
    from heliostune_b200.fusion import rmsnorm_matmul

    x, gamma = _inputs(200, 4096, seed=3)
    w = torch.zeros((4096, 1024), device="cuda", dtype=torch.float16)
    with pytest.raises(ValueError, match="fused RMSNorm"):
        rmsnorm_matmul(x, gamma, w, ActionCandidate(StreamConfig(256, 128, 64, 4, 4, 0)), fused=True)
    # the unfused path still serves it
    out = rmsnorm_matmul(x, gamma, w, ActionCandidate(StreamConfig(256, 128, 64, 4, 4, 0)))
    assert out.shape == (200, 1024) and bool((out == 0).all())
