"""Column-parallel GEMM: sharding arithmetic and the all-gather layout on world-size-2 gloo
ranks (CPU, host implementations of the GEMM and the assembly), plus the GPU assembly kernel."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from heliostune_b200.column_parallel import ColumnShard, column_parallel_matmul


def _host_gemm(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    return (a.double() @ b.double()).to(torch.float16)


def _host_assemble(gathered: torch.Tensor) -> torch.Tensor:
    parts, rows, cols = gathered.shape
    return gathered.permute(1, 0, 2).reshape(rows, parts * cols).contiguous()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank: int, world: int, port: int, queue) -> None:  # type: ignore[no-untyped-def]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(11)
        m, k, n = 37, 96, 80
        a = (torch.randn((m, k), generator=g) / k**0.5).to(torch.float16)
        b = (torch.randn((k, n), generator=g) / k**0.5).to(torch.float16)
        shard = ColumnShard(n, world, rank)
        c = column_parallel_matmul(a, shard.take(b), gemm=_host_gemm, assemble=_host_assemble)
        expected = _host_gemm(a, b)
        queue.put((rank, bool(torch.equal(c, expected)), tuple(c.shape)))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_assemble_the_full_product() -> None:
    world = 2
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    results = [queue.get(timeout=10) for _ in range(world)]
    assert sorted(r for r, _, _ in results) == [0, 1]
    for _, equal, shape in results:
        assert equal and shape == (37, 80)


def test_shard_arithmetic() -> None:
    shards = [ColumnShard(57344, 8, r) for r in range(8)]
    assert [s.start for s in shards] == [r * 7168 for r in range(8)]
    assert shards[-1].stop == 57344
    with pytest.raises(ValueError):
        ColumnShard(100, 3, 0)
    with pytest.raises(ValueError):
        ColumnShard(96, 4, 4)
    b = torch.arange(4 * 12).reshape(4, 12)
    parts = [ColumnShard(12, 3, r).take(b) for r in range(3)]
    assert torch.equal(torch.cat(parts, dim=1), b)


@pytest.mark.gpu
def test_assembly_kernel_and_single_rank_path() -> None:
    if not torch.cuda.is_available():
        pytest.skip("CUDA is unavailable")
    from heliostune_b200.column_parallel import assemble_columns
    from tests.gpu_helpers import assert_gemm_parity

    for parts, rows, cols in ((4, 33, 64), (3, 5, 7), (8, 128, 7168 // 8)):
        gathered = torch.randn((parts, rows, cols), device="cuda").to(torch.float16)
        out = assemble_columns(gathered)
        assert torch.equal(out, _host_assemble(gathered.cpu()).cuda())
    g = torch.Generator(device="cuda").manual_seed(3)
    a = (torch.randn((512, 1024), generator=g, device="cuda") / 32).to(torch.float16)
    b = (torch.randn((1024, 2048), generator=g, device="cuda") / 32).to(torch.float16)
    c = column_parallel_matmul(a, b)
    assert_gemm_parity(c, a, b)
    assert np.isfinite(c.float().cpu().numpy()).all()


def _fused_rank(rank: int, world: int, port: int, queue, peer_writes: str) -> None:  # type: ignore[no-untyped-def]
    from datetime import timedelta

    from heliostune_b200.action_expansion import fp32_reference
    from heliostune_b200.column_parallel import FusedColumnParallel

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    device = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=device)
    from heliostune_b200.action_expansion import launch
    from heliostune_b200.column_parallel import COLUMN_PARALLEL_CANDIDATE, COLUMN_PARALLEL_WIDE

    try:
        results = []
        cases = (
            (1000, 1032, 2 * 1024, None),
            (512, 4096, 2 * 1536, None),
            (1000, 520, 2 * 1280, COLUMN_PARALLEL_WIDE),  # 256 x 512 tiles, ragged last tile
            (600, 1024, 2 * 3072, COLUMN_PARALLEL_CANDIDATE),
        )
        for m, k, n, candidate in cases:
            g = torch.Generator(device=device).manual_seed(m + k)
            a = (torch.randn((m, k), generator=g, device=device) / k**0.5).to(torch.float16)
            b = (torch.randn((k, n), generator=g, device=device) / k**0.5).to(torch.float16)
            shard = ColumnShard(n, world, rank)
            fused = FusedColumnParallel(m, n, device=device, candidate=candidate, peer_writes=peer_writes)
            expected = fp32_reference(a, b)
            gemm = None if candidate is None else (lambda x, y, c=candidate: launch(x, y, c))
            plain = column_parallel_matmul(a, shard.take(b), gemm=gemm)
            for _ in range(2):  # the second call reuses the mapped outputs
                c = fused(a, shard.take(b)).clone()
                close = bool(torch.allclose(c.float(), expected, atol=1e-2, rtol=1e-2))
                results.append(close and bool(torch.equal(c, plain)))
            fused.close()
        queue.put((rank, all(results)))
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
@pytest.mark.parametrize("peer_writes", ("stores", "bulk"))
def test_fused_column_parallel_on_two_gpus(peer_writes: str) -> None:
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_fused_rank, args=(r, world, port, queue, peer_writes)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    results = [queue.get(timeout=10) for _ in range(world)]
    assert sorted(r for r, _ in results) == [0, 1]
    assert all(ok for _, ok in results)


def test_default_peer_writes_by_rank_count() -> None:
    from heliostune_b200.column_parallel import PEER_WRITES, default_peer_writes

    assert set(PEER_WRITES) == {"stores", "bulk"}
    assert default_peer_writes(2) == "bulk"
    assert [default_peer_writes(n) for n in (1, 4, 8)] == ["stores"] * 3


@pytest.mark.gpu
@pytest.mark.parametrize("peer_writes", ("stores", "bulk"))
@pytest.mark.parametrize(("m", "k", "n_total", "block_n"), ((1000, 1032, 2 * 1024, 256), (600, 520, 2 * 1280, 512)))
def test_fanout_writes_on_one_gpu(peer_writes: str, m: int, k: int, n_total: int, block_n: int) -> None:
    """hst_matmul_pair_fanout as rank 0 of two whose "peer" output is a second buffer on the same
    GPU: one launch, no cross-kernel wait. Both outputs hold the same bits in rank 0's columns,
    equal to the plain pair GEMM's and within the FP32 reference's tolerance; nothing else is
    written."""
    import ctypes

    from heliostune_b200 import _native
    from heliostune_b200.action_configs import ActionCandidate, PairConfig
    from heliostune_b200.action_expansion import fp32_reference, launch
    from heliostune_b200.column_parallel import PEER_WRITES

    if not torch.cuda.is_available():
        pytest.skip("CUDA is unavailable")
    g = torch.Generator(device="cuda").manual_seed(m + k)
    a = (torch.randn((m, k), generator=g, device="cuda") / k**0.5).to(torch.float16)
    cols = n_total // 2
    b0 = (torch.randn((k, cols), generator=g, device="cuda") / k**0.5).to(torch.float16)
    sentinel = torch.tensor(-7.0, dtype=torch.float16)
    c0 = torch.full((m, n_total), sentinel.item(), dtype=torch.float16, device="cuda")
    c1 = torch.full((m, n_total), sentinel.item(), dtype=torch.float16, device="cuda")
    config = PairConfig(256, block_n, 64, 4, 4 if block_n == 512 else 6, 8)
    outputs = (ctypes.c_void_p * 2)(c0.data_ptr(), c1.data_ptr())
    _native.check(
        _native.library().hst_matmul_pair_fanout(
            config.block_n, config.block_k, config.num_stages, config.group_m, a.data_ptr(), b0.data_ptr(),
            outputs, 2, 0, m, n_total, k, PEER_WRITES[peer_writes], torch.cuda.current_stream().cuda_stream,
        )
    )
    plain = launch(a, b0, ActionCandidate(config))
    torch.cuda.synchronize()
    assert torch.equal(c0[:, :cols], plain) and torch.equal(c1[:, :cols], plain)
    torch.testing.assert_close(plain.float(), fp32_reference(a, b0), atol=1e-2, rtol=1e-2)
    assert bool((c0[:, cols:] == sentinel.item()).all()) and bool((c1[:, cols:] == sentinel.item()).all())
    assert _native.status(torch.cuda.current_device()) == 0


@pytest.mark.gpu
def test_peer_barrier_passes_when_the_peer_has_arrived() -> None:
    """hst_peer_barrier for rank 0 of two on one GPU with the peer's entry already stored: the
    wait ends at once, the store into the other rank's words lands, no status bit is set."""
    import ctypes

    from heliostune_b200 import _native

    if not torch.cuda.is_available():
        pytest.skip("CUDA is unavailable")
    device = torch.cuda.current_device()
    _native.status(device, clear=True)
    mine = torch.tensor([0, 0, 0, 9], dtype=torch.int64, device="cuda")  # slot 1, entry of rank 1
    other = torch.zeros(4, dtype=torch.int64, device="cuda")
    words = (ctypes.c_void_p * 2)(mine.data_ptr(), other.data_ptr())
    _native.check(_native.library().hst_peer_barrier(words, 2, 0, 1, 9, 0, torch.cuda.current_stream().cuda_stream))
    assert other.tolist() == [0, 0, 9, 0]
    assert _native.status(device) == 0
