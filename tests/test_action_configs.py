"""Frozen candidate manifests: the reference's own tests (tests/test_action_configs.py:21-120)
ported onto heliostune_b200, plus equality with the manifests the reference itself emits."""

from __future__ import annotations

import subprocess
import sys
from dataclasses import FrozenInstanceError, replace

import pytest

from heliostune_b200.action_configs import (
    ALL_CANDIDATES,
    B200_FROZEN_KEPT,
    NON_SPLIT_CANDIDATES,
    PAIR_DEEP_K,
    PAIR_NARROW,
    SPLIT_K_CANDIDATES,
    ActionCandidate,
    SplitKConfig,
    StreamConfig,
    action_set_manifest,
    b200_candidates_for,
    candidates_for,
    PairConfig,
    pair_candidates_for,
    pair_stream_k_tiles,
    pair_tiles_underfill,
    split_plan,
    stream_block_m,
    stream_candidates_for,
    stream_splits,
    wave_fill,
)
from heliostune_b200.configs import (
    DEFAULT_CONFIGS,
    DEFAULT_WORKLOADS,
    EDGE_WORKLOADS,
    GRID_WORKLOADS,
    SWEEP_WORKLOADS,
    HopperGemmConfig,
    KernelConfig,
    Workload,
)
from heliostune_b200.errors import SchemaError
from tests.conftest import ROOT, load_golden


def test_enumeration_does_not_import_gpu_dependencies() -> None:
    code = (
        "import sys; "
        "from heliostune_b200.action_configs import candidates_for, b200_candidates_for; "
        "from heliostune_b200.configs import DEFAULT_WORKLOADS, GRID_WORKLOADS; "
        "assert all(candidates_for(w) for w in DEFAULT_WORKLOADS); "
        "assert all(b200_candidates_for(w) for w in GRID_WORKLOADS); "
        "import heliostune_b200.bandit, heliostune_b200.tuner; "
        "assert 'torch' not in sys.modules; "
        "assert 'heliostune_b200.action_expansion' not in sys.modules"
    )
    subprocess.run([sys.executable, "-c", code], check=True, cwd=ROOT)


def test_exact_non_split_candidates_are_frozen() -> None:
    tiles = {c.config for c in NON_SPLIT_CANDIDATES if c.family == "tile"}
    persistent = {c.config for c in NON_SPLIT_CANDIDATES if c.family == "persistent"}
    assert tiles == {
        KernelConfig(128, 128, 64, 4, 5),
        KernelConfig(128, 256, 64, 8, 4),
        KernelConfig(256, 128, 64, 8, 4),
        KernelConfig(128, 128, 128, 8, 3),
    }
    assert persistent == {HopperGemmConfig(128, 128, 64, 4, 4), HopperGemmConfig(128, 256, 64, 8, 3)}
    assert len(NON_SPLIT_CANDIDATES) == 6


def test_exact_split_candidates_are_frozen() -> None:
    assert {c.config for c in SPLIT_K_CANDIDATES} == {
        SplitKConfig(16, 64, 64, 4, 3, 4),
        SplitKConfig(16, 64, 64, 4, 3, 16),
        SplitKConfig(16, 128, 64, 4, 3, 4),
        SplitKConfig(16, 128, 64, 4, 3, 16),
    }


def test_every_workload_gets_only_its_applicable_candidates() -> None:
    assert len(DEFAULT_WORKLOADS) == 96
    for workload in DEFAULT_WORKLOADS:
        candidates = candidates_for(workload)
        assert candidates is (ALL_CANDIDATES if workload.m <= 31 else NON_SPLIT_CANDIDATES)
    edge = replace(DEFAULT_WORKLOADS[0], m=32)
    assert candidates_for(edge) is NON_SPLIT_CANDIDATES
    assert candidates_for(replace(edge, m=31)) is ALL_CANDIDATES


def test_candidate_ids_are_sorted_unique_and_disjoint_from_old_actions() -> None:
    keys = tuple(c.key for c in ALL_CANDIDATES)
    assert keys == tuple(sorted(keys))
    assert len(set(keys)) == 10
    assert set(keys).isdisjoint(c.key for c in DEFAULT_CONFIGS)
    for candidate in ALL_CANDIDATES:
        assert candidate.key == f"{candidate.family}:{candidate.config.key}"
        assert candidate.to_dict() == candidate.config.to_dict()


def test_candidates_are_immutable() -> None:
    candidate = SPLIT_K_CANDIDATES[0]
    with pytest.raises(FrozenInstanceError):
        candidate.config = candidate.config  # type: ignore[misc]
    with pytest.raises(TypeError):
        ActionCandidate("m16")  # type: ignore[arg-type]


@pytest.mark.parametrize(
    "fields",
    [
        dict(block_m=24),
        dict(block_m=8),
        dict(split_k=1),
        dict(split_k=3),
        dict(num_warps=3),
        dict(block_n=True),
    ],
)
def test_split_k_config_validation(fields: dict[str, object]) -> None:
    base = dict(block_m=16, block_n=64, block_k=64, num_warps=4, num_stages=3, split_k=4)
    base.update(fields)
    with pytest.raises(SchemaError):
        SplitKConfig(**base)  # type: ignore[arg-type]


def test_manifests_match_the_reference() -> None:
    golden = load_golden("manifest.json")
    assert action_set_manifest() == golden["action_set"]
    assert [c.key for c in ALL_CANDIDATES] == golden["all_candidate_keys"]
    assert [c.key for c in DEFAULT_CONFIGS] == golden["default_config_keys"]
    assert [[w.key, w.m, w.n, w.k, w.flops] for w in DEFAULT_WORKLOADS] == golden["default_workloads"]
    assert [w.key for w in EDGE_WORKLOADS] == golden["edge_workloads"]
    assert {w.key: [c.key for c in candidates_for(w)] for w in DEFAULT_WORKLOADS} == golden[
        "candidates_by_workload"
    ]


def test_config_round_trips() -> None:
    for config in DEFAULT_CONFIGS:
        assert KernelConfig.from_dict(config.to_dict()) == config
    persistent = HopperGemmConfig(128, 256, 64, 8, 3)
    assert HopperGemmConfig.from_dict(persistent.to_dict()) == persistent
    for workload in GRID_WORKLOADS[:5]:
        assert Workload.from_dict(workload.to_dict()) == workload
    with pytest.raises(SchemaError):
        KernelConfig.from_dict({"block_m": 16})


def test_measurement_grids() -> None:
    assert len(GRID_WORKLOADS) == 96
    assert len({w.key for w in GRID_WORKLOADS}) == 96
    assert sorted({(w.k, w.n) for w in GRID_WORKLOADS}) == sorted(
        [(4096, 6144), (4096, 4096), (4096, 28672), (14336, 4096), (3584, 4608), (3584, 3584),
         (3584, 37888), (18944, 3584)]
    )
    assert sorted({w.m for w in GRID_WORKLOADS}) == [1, 2, 4, 8, 16, 31, 32, 64, 128, 512, 2048, 8192]
    assert len(SWEEP_WORKLOADS) == 28


def test_stream_family() -> None:
    assert stream_block_m(1) == 16 and stream_block_m(17) == 32 and stream_block_m(256) == 256
    w = GRID_WORKLOADS[0]
    assert all(c.family == "stream" for c in stream_candidates_for(w))
    assert stream_candidates_for(replace(w, m=512)) == ()
    # the B200 pool keeps the split-K candidates of the frozen set that ever won on a B200
    kept = {c for c in candidates_for(w) if c.key in B200_FROZEN_KEPT and c.family == "split_k"}
    assert kept and kept <= set(b200_candidates_for(w))
    assert not any(c.family in ("tile", "persistent") for c in b200_candidates_for(w))  # M = 1
    assert set(stream_candidates_for(w)) <= set(b200_candidates_for(w))
    with pytest.raises(SchemaError):
        StreamConfig(16, 64, 64, 4, 8, 0)
    with pytest.raises(SchemaError):
        StreamConfig(16, 256, 64, 4, 8, 0)
    with pytest.raises(SchemaError):
        StreamConfig(16, 128, 64, 4, 8, 9)
    # The automatic split is the largest power of two <= 8 whose clusters are all resident
    # (148 / 74 / 33 / 15 clusters of 1 / 2 / 4 / 8 CTAs on a B200).
    config = StreamConfig(16, 128, 64, 4, 8, 0)
    assert stream_splits(1, 3584, 18944, config, 148) == 4  # 28 tiles: 28 clusters of four
    assert stream_splits(1, 1024, 18944, config, 148) == 8  # 8 tiles: 8 clusters of eight
    assert stream_splits(1, 37888, 3584, config, 148) == 1  # 296 tiles already fill the GPU
    assert stream_splits(1, 8192, 4096, config, 148) == 2  # 64 tiles: 64 pairs
    assert stream_splits(1, 4608, 4096, config, 148) == 3  # 36 tiles: 36 of the 45 clusters of three
    assert stream_splits(64, 4096, 4096, StreamConfig(64, 256, 64, 4, 4, 0), 148) == 6  # 16 tiles
    assert stream_splits(64, 6144, 4096, StreamConfig(64, 256, 64, 4, 4, 0), 148) == 5  # 24 tiles
    # every split owns K blocks: K = 100 is two blocks of 64
    assert stream_splits(1, 256, 100, StreamConfig(16, 128, 64, 4, 8, 8), 148) == 2


def test_split_plan_matches_the_reference_interval_rule() -> None:
    # tiles_per_split = cdiv(cdiv(K, BK), S); splits past K are dropped.
    assert split_plan(1543, 64, 16) == (2, 13)
    assert split_plan(17, 64, 16) == (1, 1)
    assert split_plan(18944, 64, 4) == (74, 4)


def _pair_work(tiles: int, k_blocks: int, pairs: int, sk_tiles: int, pair: int) -> list[tuple[int, int, int]]:
    """Segments (tile, kb0, kb1) of one pair, in order, as the pair kernel's PairWork walks them."""
    total = sk_tiles * k_blocks
    it, hi = total * (pairs - 1 - pair) // pairs, total * (pairs - pair) // pairs
    out = []
    while it < hi:
        tile, kb0 = divmod(it, k_blocks)
        kb1 = min(k_blocks, kb0 + hi - it)
        out.append((tile, kb0, kb1))
        it += kb1 - kb0
    out += [(t, 0, k_blocks) for t in range(sk_tiles + pair, tiles, pairs)]
    return out


@pytest.mark.parametrize(
    ("tiles", "k_blocks"),
    ((32, 64), (128, 64), (112, 56), (448, 296), (512, 224), (28, 296), (74, 64), (3, 5), (80, 2)),
)
def test_pair_stream_k_schedule_covers_every_k_block_once(tiles: int, k_blocks: int) -> None:
    pairs = 74
    sk = pair_stream_k_tiles(tiles, k_blocks, pairs)
    launched = pairs if sk else min(tiles, pairs)
    owners: dict[tuple[int, int], int] = {}
    pieces: dict[int, list[tuple[int, int, int]]] = {}
    work = [0] * launched
    for pair in range(launched):
        segs = _pair_work(tiles, k_blocks, launched, sk, pair)
        for i, (tile, kb0, kb1) in enumerate(segs):
            assert 0 <= kb0 < kb1 <= k_blocks
            if kb0 > 0:
                assert i == 0  # only a pair's first segment publishes a partial
            if kb0 == 0 and kb1 < k_blocks:
                # a finisher is the pair's last stream-K segment: whole tiles follow
                assert tile < sk and all(t >= sk for t, _, _ in segs[i + 1 :])
            for kb in range(kb0, kb1):
                assert (tile, kb) not in owners
                owners[(tile, kb)] = pair
            pieces.setdefault(tile, []).append((kb0, kb1, pair))
            work[pair] += kb1 - kb0
    assert len(owners) == tiles * k_blocks
    for tile, ps in pieces.items():
        ps.sort()
        if len(ps) > 1:
            assert tile < sk
            # the first K range is the finisher; the later ranges belong to ever lower pairs
            assert [p for _, _, p in ps] == sorted((p for _, _, p in ps), reverse=True)
            assert all(ps[i][1] == ps[i + 1][0] for i in range(len(ps) - 1))
    if sk:
        # stream-K balances the K blocks per pair to within one tile's depth
        assert max(work) - min(work) <= k_blocks
        assert max(len(ps) for ps in pieces.values()) <= max(2, -(-pairs // max(sk, 1)) + 1)


def test_pair_stream_k_rule() -> None:
    assert pair_stream_k_tiles(148, 64, 74) == 0  # whole waves
    assert pair_stream_k_tiles(32, 64, 74) == 32  # under one wave: every tile
    assert pair_stream_k_tiles(128, 64, 74) == 54  # the part-filled wave
    assert pair_stream_k_tiles(448, 296, 74) == 78  # 4 left over: one full wave joins them
    assert pair_stream_k_tiles(3, 5, 74) == 0  # under two K blocks per pair
    w = Workload(2048, 4096, 4096, "x", "y", "z")
    assert any(c.key.endswith("-streamk") for c in pair_candidates_for(w))
    assert "pair:pair-m256n256k128-w4s3g8-streamk" in {c.key for c in pair_candidates_for(w)}
    # 32 x 37 tiles of 256 x 256 are 16 whole waves
    assert "pair:pair-m256n256k128-w4s3g8-streamk" not in {c.key for c in pair_candidates_for(replace(w, m=8192, n=9472))}


def test_wide_pair_candidates_need_well_filled_waves() -> None:
    def keys(m: int, n: int, k: int) -> set[str]:
        return {c.key for c in pair_candidates_for(Workload(m, n, k, "x", "y", "z"))}

    assert wave_fill(72, 74) == 72 / 74 and wave_fill(96, 74) == 96 / 148 and wave_fill(0, 74) == 0.0
    assert "pair:pair-m256n512k64-w4s4g16" not in keys(512, 4096, 4096)  # 16 wide tiles
    assert "pair:pair-m256n512k64-w4s4g16" in keys(2048, 4096, 4096)  # 64 of 74 pairs busy
    assert "pair:pair-m256n512k64-w4s4g16" not in keys(2048, 6144, 4096)  # 96 = 74 + 22
    assert "pair:pair-m256n512k64-w4s4g16" in keys(8192, 4096, 4096)  # 256 wide tiles
    assert "pair:pair-m256n512k64-w4s4g8-streamk" in keys(8192, 4096, 14336)  # 256 = 3 x 74 + 34
    assert "pair:pair-m256n512k64-w4s4g8-streamk" not in keys(8192, 37888, 3584)  # 32 x 74 exactly


def test_deep_k_and_narrow_pair_candidates() -> None:
    def pool(m: int, n: int, k: int) -> set[str]:
        return {c.key for c in b200_candidates_for(Workload(m, n, k, "x", "y", "z"))}

    for shape in ((512, 4608, 3584), (2048, 6144, 4096), (8192, 37888, 3584)):
        assert PAIR_DEEP_K.key in pool(*shape)
        assert "tile:m128n256k64-w8s4g8" not in pool(*shape)
    # 256 x 256 tiles: 36 for M = 512, N = 4608 (half the pairs idle); 224 for N = 28672.
    assert pair_tiles_underfill(Workload(512, 4608, 3584, "x", "y", "z"))
    assert {PAIR_NARROW.key, "tile:m128n128k128-w8s3g8"} <= pool(512, 4608, 3584)
    assert not pair_tiles_underfill(Workload(512, 28672, 4096, "x", "y", "z"))
    assert not {PAIR_NARROW.key, "tile:m128n128k128-w8s3g8"} & pool(512, 28672, 4096)
    assert not pair_tiles_underfill(Workload(2048, 1024, 4096, "x", "y", "z"))  # M above 1024
    assert "tile:m128n256k64-w8s4g8" in pool(128, 28672, 4096)
    for m, n, k in ((512, 3584, 3584), (512, 28672, 4096), (2048, 4608, 3584), (8192, 4096, 14336)):
        assert len(pool(m, n, k)) <= 8  # every candidate gets one of the bandit's probes


    with pytest.raises(SchemaError):
        PairConfig(256, 512, 128, 4, 4, 8)
    with pytest.raises(SchemaError):
        PairConfig(256, 512, 64, 4, 4, 8, 2)


def test_validation_sample_is_the_reference_gate_sample() -> None:
    """The pre-timing gate's workload sample equals the one the reference's own
    ``validation_workloads`` picks (tests/golden/validation_workloads.json)."""
    from heliostune_b200.configs import EDGE_WORKLOADS, GRID_WORKLOADS, validation_workloads
    from heliostune_b200.errors import ProtocolError
    from tests.conftest import load_golden

    assert [w.key for w in validation_workloads()] == load_golden("validation_workloads.json")["keys"]
    grid = validation_workloads(GRID_WORKLOADS)
    assert len(grid) == 2 * 12 + len(EDGE_WORKLOADS)
    assert {w.m for w in grid} >= {1, 8192}
    with pytest.raises(ProtocolError):
        validation_workloads(())
