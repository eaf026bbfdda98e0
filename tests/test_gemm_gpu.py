"""GPU parity of every GEMM family against the FP32 reference and the CPU oracle.

The first three tests are the reference's own GPU tests (tests/test_action_expansion.py:43-82)
on the B200 API; the rest add the edge shapes, the stock configurations, the B200 streaming
family, the golden fixtures through the C ABI, bitwise run-to-run reproducibility and no input
mutation. The full-size grid shapes, with the comparison against cuBLAS's error, are in
test_grid_parity_gpu.py."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from heliostune_b200 import _native
from heliostune_b200.action_configs import (
    ALL_CANDIDATES,
    PAIR_CANDIDATES,
    PAIR_DEEP_K,
    PAIR_NARROW,
    PAIR_STREAM_K,
    PairConfig,
    NON_SPLIT_CANDIDATES,
    SPLIT_K_CANDIDATES,
    ActionCandidate,
    StreamConfig,
    stream_block_m,
    stream_candidates_for,
)
from heliostune_b200.action_expansion import launch
from heliostune_b200.configs import DEFAULT_CONFIGS, EDGE_WORKLOADS, KernelConfig, Workload
from heliostune_b200.kernel import matmul
from oracle import oracle
from tests.conftest import GOLDEN
from tests.gpu_helpers import assert_gemm_parity, require_cuda, scaled_normal

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _cuda() -> None:
    require_cuda()
    _native.library()


@pytest.mark.parametrize("candidate", SPLIT_K_CANDIDATES, ids=lambda c: c.key)
@pytest.mark.parametrize("m", (1, 7, 31))
@pytest.mark.parametrize("k", (17, 1543))
def test_split_k_masks_edges_and_empty_splits(candidate: ActionCandidate, m: int, k: int) -> None:
    torch.manual_seed(17)
    a = torch.rand((m, k), device="cuda", dtype=torch.float16)
    b = torch.rand((k, 131), device="cuda", dtype=torch.float16)
    assert_gemm_parity(launch(a, b, candidate), a, b)


@pytest.mark.parametrize("candidate", SPLIT_K_CANDIDATES, ids=lambda c: c.key)
def test_split_k_supports_strided_inputs(candidate: ActionCandidate) -> None:
    torch.manual_seed(31)
    a = torch.rand((31, 514), device="cuda", dtype=torch.float16)[:, ::2]
    b = torch.rand((514, 134), device="cuda", dtype=torch.float16)[::2, ::2]
    assert not a.is_contiguous() and not b.is_contiguous()
    assert_gemm_parity(launch(a, b, candidate), a, b)


@pytest.mark.parametrize("candidate", NON_SPLIT_CANDIDATES, ids=lambda c: c.key)
@pytest.mark.parametrize("m", (1, 7, 31, 257))
def test_frozen_tile_and_persistent_candidates_match_reference(candidate: ActionCandidate, m: int) -> None:
    torch.manual_seed(257)
    a = torch.rand((m, 256), device="cuda", dtype=torch.float16)
    b = torch.rand((256, 256), device="cuda", dtype=torch.float16)
    assert_gemm_parity(launch(a, b, candidate), a, b)


@pytest.mark.parametrize("workload", EDGE_WORKLOADS, ids=lambda w: w.projection)
@pytest.mark.parametrize("candidate", ALL_CANDIDATES, ids=lambda c: c.key)
def test_edge_workloads(workload: Workload, candidate: ActionCandidate) -> None:
    if candidate.family == "split_k" and workload.m > 31:
        pytest.skip("split-K is defined for M <= 31")
    g = torch.Generator(device="cuda").manual_seed(workload.m * 7 + workload.n)
    a = scaled_normal((workload.m, workload.k), workload.k, g)
    b = scaled_normal((workload.k, workload.n), workload.k, g)
    assert_gemm_parity(launch(a, b, candidate), a, b)


@pytest.mark.parametrize("config", DEFAULT_CONFIGS, ids=lambda c: c.key)
@pytest.mark.parametrize("shape", ((100, 264, 136), (37, 131, 77)), ids=("aligned", "odd"))
def test_stock_tile_configurations(config: KernelConfig, shape: tuple[int, int, int]) -> None:
    m, n, k = shape
    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    a = scaled_normal((m, k), k, g)
    b = scaled_normal((k, n), k, g)
    assert_gemm_parity(matmul(a, b, config), a, b)


@pytest.mark.parametrize("m", (1, 2, 16, 17, 31, 32, 64, 100, 128, 200, 256))
def test_stream_family(m: int) -> None:
    k, n = 4096, 4096
    workload = Workload(m=m, n=n, k=k, model="t", projection="t", regime="t")
    g = torch.Generator(device="cuda").manual_seed(m)
    a = scaled_normal((m, k), k, g)
    b = scaled_normal((k, n), k, g)
    candidates = stream_candidates_for(workload)
    assert candidates
    for candidate in candidates:
        assert_gemm_parity(launch(a, b, candidate), a, b)
    for split in (1, 2, 3, 4, 5, 6, 7, 8):
        fixed = ActionCandidate(StreamConfig(stream_block_m(m), 128, 64, 4, 4, split))
        assert_gemm_parity(launch(a, b, fixed), a, b)


@pytest.mark.parametrize("split", (3, 5, 6, 7))
@pytest.mark.parametrize("block_n", (128, 256))
@pytest.mark.parametrize("shape", ((64, 4608, 3584), (100, 1000, 1000), (128, 6144, 4096)), ids=lambda s: "x".join(map(str, s)))
def test_stream_odd_cluster_sizes(split: int, block_n: int, shape: tuple[int, int, int]) -> None:
    """Clusters of 3, 5, 6 and 7 CTAs: the last owner holds fewer columns than the others."""
    m, n, k = shape
    g = torch.Generator(device="cuda").manual_seed(m + split)
    a = scaled_normal((m, k), k, g)
    b = scaled_normal((k, n), k, g)
    bm = stream_block_m(m) if block_n == 128 else (64 if m <= 64 else 128)
    candidate = ActionCandidate(StreamConfig(bm, block_n, 64, 4, 4, split))
    first = launch(a, b, candidate)
    assert_gemm_parity(first, a, b)
    assert torch.equal(first.view(torch.int16), launch(a, b, candidate).view(torch.int16))


@pytest.mark.parametrize("candidate", (*PAIR_CANDIDATES, PAIR_DEEP_K, PAIR_NARROW), ids=lambda c: c.key)
@pytest.mark.parametrize(
    "shape",
    ((512, 4096, 4096), (257, 264, 136), (1000, 1032, 520), (131, 8, 8), (2048, 3584, 18944)),
    ids=lambda s: "x".join(map(str, s)),
)
def test_pair_family(candidate: ActionCandidate, shape: tuple[int, int, int]) -> None:
    m, n, k = shape
    g = torch.Generator(device="cuda").manual_seed(m + k)
    a = scaled_normal((m, k), k, g)
    b = scaled_normal((k, n), k, g)
    assert_gemm_parity(launch(a, b, candidate), a, b)


@pytest.mark.parametrize("split", (2, 4))
@pytest.mark.parametrize("block_n", (128, 256))
@pytest.mark.parametrize(
    "shape", ((512, 4096, 4096), (300, 1032, 520), (129, 264, 2000), (512, 4608, 3584)),
    ids=lambda s: "x".join(map(str, s)),
)
def test_pair_split_k(split: int, block_n: int, shape: tuple[int, int, int]) -> None:
    m, n, k = shape
    g = torch.Generator(device="cuda").manual_seed(m * split + block_n)
    a = scaled_normal((m, k), k, g)
    b = scaled_normal((k, n), k, g)
    candidate = ActionCandidate(PairConfig(256, block_n, 64, 4, 6, 8, split))
    first = launch(a, b, candidate)
    assert_gemm_parity(first, a, b)
    assert torch.equal(first.view(torch.int16), launch(a, b, candidate).view(torch.int16))


@pytest.mark.parametrize("block_n, block_k", ((128, 64), (256, 64), (256, 128)))
@pytest.mark.parametrize(
    "shape",
    (
        (512, 4096, 4096),  # under one wave: every tile shared along K
        (2048, 3584, 3584),  # one full wave and a part-filled one
        (8192, 3584, 640),  # four tiles past six waves: one full wave joins them
        (512, 1024, 8192),  # few deep tiles: about ten pieces per tile
        (600, 1000, 4000),  # ragged rows and columns
        (300, 1032, 520),  # too little K to share: whole tiles only
    ),
    ids=lambda s: "x".join(map(str, s)),
)
def test_pair_stream_k(block_n: int, block_k: int, shape: tuple[int, int, int]) -> None:
    m, n, k = shape
    g = torch.Generator(device="cuda").manual_seed(m + n + block_n)
    a = scaled_normal((m, k), k, g)
    b = scaled_normal((k, n), k, g)
    stages = 6 if block_k == 64 else 3
    candidate = ActionCandidate(PairConfig(256, block_n, block_k, 4, stages, 8, PAIR_STREAM_K))
    first = launch(a, b, candidate)
    assert_gemm_parity(first, a, b)
    for _ in range(2):  # later launches see the earlier ones' publication words: never matched
        assert torch.equal(first.view(torch.int16), launch(a, b, candidate).view(torch.int16))


@pytest.mark.parametrize(
    "config",
    (PairConfig(256, 512, 64, 4, 4, 16), PairConfig(256, 512, 64, 4, 4, 8, PAIR_STREAM_K)),
    ids=lambda c: ActionCandidate(c).key,
)
@pytest.mark.parametrize(
    "shape",
    (
        (256, 512, 64),  # one tile, one K block
        (300, 1000, 520),  # ragged: the second UMMA of the last column tile is half outside
        (1000, 2056, 777),  # 8 columns past the last full tile
        (2048, 3584, 3584),  # 56 tiles: under one wave of pairs
        (512, 28672, 1024),  # 112 tiles: a wave and a half
        (8192, 4096, 512),  # 256 tiles, shallow K: the accumulator halves turn over fast
    ),
    ids=lambda s: "x".join(map(str, s)),
)
def test_pair_wide_tile(config: PairConfig, shape: tuple[int, int, int]) -> None:
    m, n, k = shape
    g = torch.Generator(device="cuda").manual_seed(m * 3 + n)
    a = scaled_normal((m, k), k, g)
    b = scaled_normal((k, n), k, g)
    candidate = ActionCandidate(config)
    first = launch(a, b, candidate)
    assert_gemm_parity(first, a, b)
    assert torch.equal(first.view(torch.int16), launch(a, b, candidate).view(torch.int16))


def test_pair_stream_k_ignores_stale_workspace_contents() -> None:
    lib = _native.library()
    m, n, k = 512, 4096, 2048
    g = torch.Generator(device="cuda").manual_seed(77)
    a = scaled_normal((m, k), k, g)
    b = scaled_normal((k, n), k, g)
    config = _native.GemmConfig(_native.FAMILY_PAIR, 256, 256, 64, 4, 6, 8, PAIR_STREAM_K)
    size = ctypes.c_size_t()
    _native.check(
        lib.hst_gemm_workspace_size(
            ctypes.byref(config), a.data_ptr(), k, 1, b.data_ptr(), n, 1, m, n, k,
            torch.cuda.current_device(), ctypes.byref(size),
        )
    )
    assert size.value >= 74 * 256 * 256 * 4  # one partial tile per pair
    outputs = []
    for fill in (0xFF, 0x00, None):
        ws = torch.empty(size.value, dtype=torch.uint8, device="cuda")
        if fill is None:
            ws.random_(0, 256, generator=g)
        else:
            ws.fill_(fill)
        for _ in range(2):  # the second call meets the first one's partials and words
            c = torch.empty((m, n), dtype=torch.float16, device="cuda")
            _native.check(
                lib.hst_gemm(
                    ctypes.byref(config), a.data_ptr(), k, 1, b.data_ptr(), n, 1, c.data_ptr(), n,
                    m, n, k, ws.data_ptr(), size.value, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream),
                )
            )
            outputs.append(c)
    assert_gemm_parity(outputs[0], a, b)
    for c in outputs[1:]:
        assert torch.equal(outputs[0].view(torch.int16), c.view(torch.int16))


def test_pair_family_with_strided_operands_and_deep_k() -> None:
    g = torch.Generator(device="cuda").manual_seed(9)
    a = scaled_normal((300, 2 * 1540), 1540, g)[:, ::2]
    b = scaled_normal((1540, 2 * 520), 1540, g)[:, ::2]
    for config in (PairConfig(256, 256, 128, 4, 3, 8), PairConfig(256, 128, 128, 4, 4, 4)):
        assert_gemm_parity(launch(a, b, ActionCandidate(config)), a, b)


def test_cached_workspace_sizes_follow_operand_alignment() -> None:
    # The host caches the planner's workspace size per config, shape, strides and 16-byte
    # alignment: an unaligned A (a one-element offset into a larger buffer) needs the packing
    # workspace, the aligned one does not, and alternating them must keep both exact.
    from heliostune_b200.kernel import _WORKSPACE_SIZES

    g = torch.Generator(device="cuda").manual_seed(11)
    m, n, k = 512, 1024, 1024
    base = scaled_normal((m * k + 8,), k, g)
    aligned = base[: m * k].view(m, k)
    unaligned = base[1 : m * k + 1].view(m, k)
    b = scaled_normal((k, n), k, g)
    candidate = ActionCandidate(PairConfig(256, 256, 128, 4, 3, 8))
    _WORKSPACE_SIZES.clear()
    for a in (aligned, unaligned, aligned, unaligned):
        assert_gemm_parity(launch(a, b, candidate), a, b)
    sizes = {key[8]: size for key, size in _WORKSPACE_SIZES.items()}  # key[8]: A's address mod 16
    assert sizes[0] == 0 and sizes[2] > 0


def _abi_gemm(config: _native.GemmConfig, a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """Call hst_gemm of the C ABI directly with device buffers."""
    lib = _native.library()
    m, k = a.shape
    n = b.shape[1]
    size = ctypes.c_size_t()
    _native.check(
        lib.hst_gemm_workspace_size(
            ctypes.byref(config), a.data_ptr(), a.stride(0), a.stride(1), b.data_ptr(), b.stride(0),
            b.stride(1), m, n, k, torch.cuda.current_device(), ctypes.byref(size),
        )
    )
    ws = torch.empty(max(size.value, 1), dtype=torch.uint8, device="cuda")
    c = torch.empty((m, n), dtype=torch.float16, device="cuda")
    _native.check(
        lib.hst_gemm(
            ctypes.byref(config), a.data_ptr(), a.stride(0), a.stride(1), b.data_ptr(), b.stride(0),
            b.stride(1), c.data_ptr(), n, m, n, k, ws.data_ptr(), size.value,
            torch.cuda.current_stream().cuda_stream,
        )
    )
    torch.cuda.synchronize()
    return c


GOLDEN_CASES = ("edge_1x8x8", "edge_7x136x264", "edge_131x1032x520", "splitk_7x131x17", "splitk_31x131x1543")
ABI_CONFIGS = {
    "tile": _native.GemmConfig(_native.FAMILY_TILE, 128, 128, 64, 4, 5, 8, 0),
    "tile256": _native.GemmConfig(_native.FAMILY_TILE, 256, 128, 64, 8, 4, 8, 0),
    "persistent": _native.GemmConfig(_native.FAMILY_PERSISTENT, 128, 256, 64, 8, 3, 8, 0),
    "split_k": _native.GemmConfig(_native.FAMILY_SPLIT_K, 16, 128, 64, 4, 3, 8, 16),
    "stream": _native.GemmConfig(_native.FAMILY_STREAM, 256, 128, 64, 4, 4, 8, 0),
    "stream2": _native.GemmConfig(_native.FAMILY_STREAM, 128, 256, 64, 4, 3, 8, 4),
    "pair": _native.GemmConfig(_native.FAMILY_PAIR, 256, 256, 64, 4, 6, 8, 0),
}


@pytest.mark.parametrize("name", GOLDEN_CASES)
@pytest.mark.parametrize("family", list(ABI_CONFIGS))
def test_golden_fixtures_through_the_c_abi(name: str, family: str) -> None:
    cases = np.load(GOLDEN / "gemm_cases.npz")
    a_np, b_np = cases[f"{name}_a"], cases[f"{name}_b"]
    m = a_np.shape[0]
    if family == "split_k" and m > 31 or family.startswith("stream") and m > (128 if family == "stream2" else 256):
        pytest.skip("outside the family's M range")
    a = torch.from_numpy(a_np).cuda()
    b = torch.from_numpy(b_np).cuda()
    out = _abi_gemm(ABI_CONFIGS[family], a, b).cpu().numpy()
    rows = cases[f"{name}_crows"]
    expected = cases[f"{name}_c"]
    assert oracle.within_tolerance(out[rows], expected, atol=1e-2, rtol=1e-2)
    assert oracle.normwise_error(out[rows], expected) <= 1e-2
    # and against the oracle on every row
    full = oracle.gemm_fp32_reference(a_np, b_np)
    assert oracle.normwise_error(out, full) <= 1e-2


def test_strided_golden_fixture_through_the_c_abi() -> None:
    cases = np.load(GOLDEN / "gemm_cases.npz")
    a = torch.from_numpy(cases["strided_a_full"]).cuda()[:, ::2]
    b = torch.from_numpy(cases["strided_b_full"]).cuda()[::2, ::2]
    for family in ("tile", "split_k", "stream"):
        out = _abi_gemm(ABI_CONFIGS[family], a, b).cpu().numpy()
        assert oracle.within_tolerance(out, cases["strided_c"], atol=1e-2, rtol=1e-2)


@pytest.mark.parametrize(
    "candidate",
    [
        ActionCandidate(KernelConfig(128, 256, 64, 8, 4)),
        ActionCandidate(KernelConfig(64, 64, 64, 4, 2)),
        *[c for c in ALL_CANDIDATES if c.family in ("persistent", "split_k")][:3],
        ActionCandidate(StreamConfig(32, 128, 64, 4, 8, 0)),
        ActionCandidate(StreamConfig(32, 128, 64, 4, 6, 8)),
        ActionCandidate(StreamConfig(128, 256, 64, 4, 3, 4)),
        ActionCandidate(PairConfig(256, 256, 64, 4, 6, 8)),
        ActionCandidate(PairConfig(256, 256, 64, 4, 6, 8, PAIR_STREAM_K)),
        ActionCandidate(PairConfig(256, 512, 64, 4, 4, 16)),
        PAIR_DEEP_K,
        PAIR_NARROW,
    ],
    ids=lambda c: c.key,
)
def test_bitwise_reproducible_and_inputs_untouched(candidate: ActionCandidate) -> None:
    if candidate.family == "split_k":
        m = 31
    elif candidate.family == "stream":
        m = min(candidate.config.block_m, 100) - 1
    else:
        m = 300
    k, n = 4096, 3584
    g = torch.Generator(device="cuda").manual_seed(5)
    a = scaled_normal((m, k), k, g)
    b = scaled_normal((k, n), k, g)
    a0, b0 = a.clone(), b.clone()
    first = launch(a, b, candidate)
    for _ in range(3):
        again = launch(a, b, candidate)
        assert torch.equal(first.view(torch.int16), again.view(torch.int16))
    assert torch.equal(a.view(torch.int16), a0.view(torch.int16))
    assert torch.equal(b.view(torch.int16), b0.view(torch.int16))


def test_empty_and_degenerate_extents() -> None:
    a = torch.zeros((0, 64), device="cuda", dtype=torch.float16)
    b = torch.zeros((64, 32), device="cuda", dtype=torch.float16)
    assert launch(a, b, NON_SPLIT_CANDIDATES[0]).shape == (0, 32)
    a = torch.zeros((5, 0), device="cuda", dtype=torch.float16)
    b = torch.zeros((0, 16), device="cuda", dtype=torch.float16)
    out = matmul(a, b, KernelConfig(128, 128, 64, 4, 5))
    assert out.shape == (5, 16) and bool((out == 0).all())
    with pytest.raises(ValueError, match="split-K requires"):
        launch(torch.zeros((32, 64), device="cuda", dtype=torch.float16), torch.zeros((64, 16), device="cuda", dtype=torch.float16), SPLIT_K_CANDIDATES[0])


def test_pre_timing_gate_passes_every_family_and_journals_failures(monkeypatch: pytest.MonkeyPatch) -> None:
    """The reference's gate (hopper_kernel.py:498-623) over every family of this library on the
    edge shapes; a wrong kernel is a journal entry, and the asserting form raises on it."""
    from heliostune_b200 import action_expansion
    from heliostune_b200.action_configs import pair_candidates_for, stream_candidates_for
    from heliostune_b200.errors import ProtocolError
    from heliostune_b200.hopper_kernel import assert_candidate_kernels_correct, validate_candidate_kernels

    def every_family(w: Workload) -> tuple[ActionCandidate, ...]:
        frozen = tuple(c for c in ALL_CANDIDATES if c.family != "split_k" or w.m <= 31)
        pairs = (*PAIR_CANDIDATES, PAIR_DEEP_K, PAIR_NARROW) if w.m > 128 else ()
        return (*frozen, *stream_candidates_for(w), *pairs)

    results = assert_candidate_kernels_correct("B200", candidates_for=every_family, workloads=EDGE_WORKLOADS)
    assert len(results) == sum(len(every_family(w)) for w in EDGE_WORKLOADS)
    assert {r.kernel for r in results} == {"tile", "persistent", "split_k", "stream", "pair"}
    real = action_expansion.launch

    def wrong_pair(a, b, candidate):  # type: ignore[no-untyped-def]
        out = real(a, b, candidate)
        return out + 1 if candidate.family == "pair" else out

    monkeypatch.setattr(action_expansion, "launch", wrong_pair)
    journal = validate_candidate_kernels(candidates_for=every_family, workloads=EDGE_WORKLOADS)
    assert {r.kernel for r in journal if not r.correct} == {"pair"}
    assert all(r.error and "correctness check failed" in r.error for r in journal if not r.correct)
    with pytest.raises(ProtocolError, match="candidate kernel checks failed"):
        assert_candidate_kernels_correct(candidates_for=every_family, workloads=EDGE_WORKLOADS)
