"""The frozen action-expansion candidates plus the B200 weight-streaming family.

``SplitKConfig``, ``ActionCandidate``, the frozen candidate tuples, ``candidates_for`` and
``action_set_manifest`` keep the reference's names, keys and membership
(``src/heliostune/action_configs.py:17-131``). Enumeration imports neither torch nor the native
library, as in the reference.

:class:`StreamConfig` is new: a swap-AB tcgen05 weight-streaming GEMM for ``M <= 256`` whose
split factor can be chosen per shape so the grid fills the 148 SMs. It is offered to the bandit
next to the frozen candidates by :func:`b200_candidates_for`.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass
from typing import Any, Literal

from heliostune_b200.configs import DEFAULT_CONFIGS, HopperGemmConfig, KernelConfig, Workload
from heliostune_b200.errors import SchemaError
from heliostune_b200.validation import exact_int

#: Largest M the reference's split-K launcher accepts (``action_configs.py:17``).
SPLIT_K_M_LIMIT = 31

#: Largest M the B200 weight-streaming kernel accepts (the UMMA N of its swapped MMA).
STREAM_M_LIMIT = 256


def _power_of_two(value: int) -> bool:
    return value > 0 and value & (value - 1) == 0


@dataclass(frozen=True, slots=True)
class SplitKConfig:
    """Split-K GEMM for ``1 <= M <= 31``: FP32 partials, then a fixed-order reduction.

    On a B200 (swap-AB tcgen05): ``block_n`` is the UMMA M, i.e. the columns of C one CTA owns
    (64 or 128); ``block_m`` is the granularity the rows of A are padded to for the UMMA N (all
    ``M <= 31`` rows are held by one CTA); ``block_k`` is the K extent of one shared-memory stage;
    ``num_stages`` is the depth of the TMA ring; ``split_k`` is the number of contiguous
    ``block_k``-aligned K intervals, each written to its own FP32 partial and summed in split
    order by a second kernel. ``num_warps`` is kept for the key.
    """

    block_m: int
    block_n: int
    block_k: int
    num_warps: int
    num_stages: int
    split_k: int

    def __post_init__(self) -> None:
        for name in ("block_m", "block_n", "block_k", "num_warps", "num_stages", "split_k"):
            exact_int(getattr(self, name), context=f"split-K config {name}", minimum=1)
        for name in ("block_m", "block_n", "block_k", "split_k"):
            if not _power_of_two(getattr(self, name)):
                raise SchemaError(f"{name} must be a power of two")
        for name in ("block_m", "block_n", "block_k"):
            if getattr(self, name) < 16:
                raise SchemaError(f"{name} must be at least 16")
        if self.num_warps not in (1, 2, 4, 8):
            raise SchemaError("num_warps must be one of 1, 2, 4, or 8")
        if self.split_k < 2:
            raise SchemaError("split_k must be at least 2")

    @property
    def key(self) -> str:
        return (
            f"m{self.block_m}n{self.block_n}k{self.block_k}"
            f"-w{self.num_warps}s{self.num_stages}-split{self.split_k}"
        )

    def to_dict(self) -> dict[str, int]:
        return asdict(self)


@dataclass(frozen=True, slots=True)
class StreamConfig:
    """B200 weight-streaming GEMM for ``1 <= M <= 256`` (no reference counterpart).

    A CTA owns ``block_n`` columns of C (128, or 256 as two UMMA atoms sharing the A tile, for
    ``block_m`` 64 or 128) and all M rows, padded to ``block_m`` (a power of two >= 16, the UMMA
    N of the swapped MMA). ``block_k`` and ``num_stages`` shape the TMA ring. ``split_k`` CTAs
    (1..8; 0 asks for the count that puts the most CTAs in one wave, see :func:`stream_splits`)
    divide K and form a thread-block cluster that sums their FP32 partials in split order through
    distributed shared memory, so no workspace and no second kernel are needed.
    """

    block_m: int
    block_n: int
    block_k: int
    num_warps: int
    num_stages: int
    split_k: int = 0

    def __post_init__(self) -> None:
        for name in ("block_m", "block_n", "block_k", "num_warps", "num_stages"):
            exact_int(getattr(self, name), context=f"stream config {name}", minimum=1)
        exact_int(self.split_k, context="stream config split_k", minimum=0)
        for name in ("block_m", "block_n", "block_k"):
            if not _power_of_two(getattr(self, name)):
                raise SchemaError(f"{name} must be a power of two")
        if not 16 <= self.block_m <= STREAM_M_LIMIT:
            raise SchemaError(f"block_m must be between 16 and {STREAM_M_LIMIT}")
        if self.block_n not in (128, 256):
            raise SchemaError("block_n must be 128 or 256")
        if self.block_n == 256 and self.block_m not in (64, 128):
            raise SchemaError("block_n 256 needs block_m 64 or 128")
        if self.block_k not in (64, 128):
            raise SchemaError("block_k must be 64 or 128")
        if self.split_k > 8:
            raise SchemaError("split_k must be 0 (automatic) or 1..8")
        if self.num_warps not in (1, 2, 4, 8):
            raise SchemaError("num_warps must be one of 1, 2, 4, or 8")

    @property
    def key(self) -> str:
        split = "auto" if self.split_k == 0 else str(self.split_k)
        return (
            f"stream-m{self.block_m}n{self.block_n}k{self.block_k}"
            f"-w{self.num_warps}s{self.num_stages}-split{split}"
        )

    def to_dict(self) -> dict[str, int]:
        return asdict(self)


#: ``PairConfig.split_k`` value selecting the stream-K schedule (HST_PAIR_STREAM_K in the C ABI).
PAIR_STREAM_K = -1


@dataclass(frozen=True, slots=True)
class PairConfig:
    """B200 CTA-pair GEMM (no reference counterpart): 256 x ``block_n`` tiles per two SMs.

    A cluster of two CTAs shares one ``tcgen05.mma.cta_group::2`` (UMMA M = 256): each CTA
    loads its 128 rows of A and half of the tile's ``block_n`` columns of B, so each SM moves
    half the B bytes of a single-SM tile. Persistent over the tiles in ``group_m`` raster order
    with two TMEM accumulators; ``num_stages`` is the ring depth per CTA. ``num_warps`` is kept
    for the key (the CTA runs six warps). ``split_k`` 2 or 4 (0 = automatic, only when the tiles
    would leave most SMs idle) lets 2 x ``split_k`` CTAs share one tile and sum their FP32
    partials in split order through distributed shared memory. ``split_k`` -1
    (:data:`PAIR_STREAM_K`) balances a part-filled last wave by stream-K: the tiles
    :func:`pair_stream_k_tiles` names are cut along K into one equal run of K blocks per pair,
    whose pieces meet through FP32 partial tiles in the workspace.
    """

    block_m: int
    block_n: int
    block_k: int
    num_warps: int
    num_stages: int
    group_m: int = 8
    split_k: int = 1

    def __post_init__(self) -> None:
        for name in ("block_m", "block_n", "block_k", "num_warps", "num_stages", "group_m"):
            exact_int(getattr(self, name), context=f"pair config {name}", minimum=1)
        if self.block_m != 256:
            raise SchemaError("block_m must be 256 (two SMs x 128 rows)")
        if self.block_n not in (128, 256, 512):
            raise SchemaError("block_n must be 128, 256 or 512")
        if self.block_k not in (64, 128):
            raise SchemaError("block_k must be 64 or 128")
        if self.block_n == 512 and (self.block_k != 64 or self.split_k > 1):
            raise SchemaError("the 512-wide pair tile has block_k 64 and no cluster split-K")
        if self.num_warps not in (1, 2, 4, 8):
            raise SchemaError("num_warps must be one of 1, 2, 4, or 8")
        exact_int(self.split_k, context="pair config split_k", minimum=PAIR_STREAM_K)
        if self.split_k not in (PAIR_STREAM_K, 0, 1, 2, 4):
            raise SchemaError("split_k must be -1 (stream-K), 0 (automatic), 1, 2 or 4")

    @property
    def key(self) -> str:
        split = {1: "", 0: "-splitauto", PAIR_STREAM_K: "-streamk"}.get(self.split_k, f"-split{self.split_k}")
        return (
            f"pair-m{self.block_m}n{self.block_n}k{self.block_k}"
            f"-w{self.num_warps}s{self.num_stages}g{self.group_m}{split}"
        )

    def to_dict(self) -> dict[str, int]:
        return asdict(self)


ActionConfig = KernelConfig | HopperGemmConfig | SplitKConfig | StreamConfig | PairConfig


@dataclass(frozen=True, slots=True)
class ActionCandidate:
    """An immutable launch configuration with a family-qualified identity."""

    config: ActionConfig

    def __post_init__(self) -> None:
        if not isinstance(
            self.config, KernelConfig | HopperGemmConfig | SplitKConfig | StreamConfig | PairConfig
        ):
            raise TypeError("candidate config must be a tile, persistent, split-K, stream or pair config")

    @property
    def family(self) -> Literal["tile", "persistent", "split_k", "stream", "pair"]:
        if isinstance(self.config, KernelConfig):
            return "tile"
        if isinstance(self.config, HopperGemmConfig):
            return "persistent"
        if isinstance(self.config, SplitKConfig):
            return "split_k"
        if isinstance(self.config, StreamConfig):
            return "stream"
        return "pair"

    @property
    def key(self) -> str:
        return f"{self.family}:{self.config.key}"

    def to_dict(self) -> dict[str, int | bool]:
        return dict(self.config.to_dict())


def _sorted(candidates: tuple[ActionCandidate, ...]) -> tuple[ActionCandidate, ...]:
    return tuple(sorted(candidates, key=lambda c: c.key))


#: The six ordinary/persistent candidates (``action_configs.py:88-101``).
NON_SPLIT_CANDIDATES: tuple[ActionCandidate, ...] = _sorted(
    (
        ActionCandidate(KernelConfig(128, 128, 64, 4, 5)),
        ActionCandidate(KernelConfig(128, 256, 64, 8, 4)),
        ActionCandidate(KernelConfig(256, 128, 64, 8, 4)),
        ActionCandidate(KernelConfig(128, 128, 128, 8, 3)),
        ActionCandidate(HopperGemmConfig(128, 128, 64, 4, 4)),
        ActionCandidate(HopperGemmConfig(128, 256, 64, 8, 3)),
    )
)
#: The four split-K candidates for ``M <= 31`` (``action_configs.py:102-111``).
SPLIT_K_CANDIDATES: tuple[ActionCandidate, ...] = _sorted(
    (
        ActionCandidate(SplitKConfig(16, 64, 64, 4, 3, 4)),
        ActionCandidate(SplitKConfig(16, 64, 64, 4, 3, 16)),
        ActionCandidate(SplitKConfig(16, 128, 64, 4, 3, 4)),
        ActionCandidate(SplitKConfig(16, 128, 64, 4, 3, 16)),
    )
)
ALL_CANDIDATES: tuple[ActionCandidate, ...] = _sorted((*NON_SPLIT_CANDIDATES, *SPLIT_K_CANDIDATES))


def candidates_for(workload: Workload) -> tuple[ActionCandidate, ...]:
    """The reference's frozen candidates for a workload; no measurement influences them."""
    return ALL_CANDIDATES if workload.m <= SPLIT_K_M_LIMIT else NON_SPLIT_CANDIDATES


def stream_block_m(m: int) -> int:
    """Padded row count of the weight-streaming kernel: the next multiple of 16 as power of 2."""
    block = 16
    while block < m:
        block *= 2
    return block


def stream_candidates_for(workload: Workload) -> tuple[ActionCandidate, ...]:
    """B200 weight-streaming candidates for ``M <= 256`` (empty above)."""
    if workload.m > STREAM_M_LIMIT:
        return ()
    bm = stream_block_m(workload.m)
    wide = ()
    if bm in (64, 128):
        # 256 columns per CTA: both column atoms share each A^T tile, halving the A bytes per
        # byte of B that matter once M approaches the column tile.
        wide = (ActionCandidate(StreamConfig(bm, 256, 64, 4, 4, 0)),)
    return _sorted(
        (
            ActionCandidate(StreamConfig(bm, 128, 64, 4, 8, 0)),
            ActionCandidate(StreamConfig(bm, 128, 128, 4, 4, 0)),
            ActionCandidate(StreamConfig(bm, 128, 64, 4, 4, 0)),
            *wide,
        )
    )


#: Smallest M the CTA-pair family is offered for (one 256-row tile is half empty below).
PAIR_M_MINIMUM = 129

PAIR_CANDIDATES: tuple[ActionCandidate, ...] = _sorted(
    (
        ActionCandidate(PairConfig(256, 256, 64, 4, 6, 8)),
        ActionCandidate(PairConfig(256, 256, 64, 4, 6, 16)),
        ActionCandidate(PairConfig(256, 256, 64, 4, 6, 4)),
    )
)
#: Split-K pair candidates: a (2, S) cluster per tile. At most 33 clusters of four and 15 of eight
#: CTAs are resident on a B200 at once, so split 2 is offered while the 256 x 256 tiles fit 33
#: clusters and split 4 while they fit 15.
PAIR_SPLIT2 = ActionCandidate(PairConfig(256, 256, 64, 4, 6, 8, 2))
PAIR_SPLIT4 = ActionCandidate(PairConfig(256, 256, 64, 4, 6, 8, 4))
PAIR_SPLIT_CANDIDATES: tuple[ActionCandidate, ...] = _sorted((PAIR_SPLIT2, PAIR_SPLIT4))


#: Stream-K pair candidate with 64-deep K blocks, for where the 256 x 256 tiles leave the last
#: wave of pairs part-filled (see :func:`pair_stream_k_tiles`). The tuner's pool offers the
#: 128-deep form (:data:`PAIR_DEEP_K_STREAM_K`); this one stays for forced runs and the tests.
PAIR_STREAM_K_CANDIDATE = ActionCandidate(PairConfig(256, 256, 64, 4, 6, 8, PAIR_STREAM_K))


def pair_stream_k_tiles(tiles: int, k_blocks: int, pairs: int) -> int:
    """Tiles the stream-K pair schedule shares out along K over ``pairs`` persistent pairs.

    None when the tiles fill whole waves; all of them below one wave; otherwise the part-filled
    last wave, plus one full wave when the last wave holds under a quarter of the pairs (so no
    tile is cut into more than about five pieces); none when a pair would get under two of the
    shared K blocks. The native planner applies the same rule (``hst_pair_stream_k_tiles``).
    """
    if tiles <= 0 or k_blocks <= 0 or pairs <= 0:
        return 0
    waves, rest = divmod(tiles, pairs)
    if rest == 0:
        return 0
    shared = tiles if waves == 0 else (rest if rest * 4 >= pairs else rest + pairs)
    return shared if shared * k_blocks >= 2 * pairs else 0


#: 512-wide pair tiles (a quarter fewer L2-to-SM bytes per FLOP, single-buffered accumulator),
#: offered while the 256 x 512 tiles keep at least :data:`PAIR_MIN_FILL` of the pairs busy over
#: their waves; the stream-K form where they leave the last wave part-filled.
PAIR_WIDE = ActionCandidate(PairConfig(256, 512, 64, 4, 4, 16))
PAIR_WIDE_STREAM_K = ActionCandidate(PairConfig(256, 512, 64, 4, 4, 8, PAIR_STREAM_K))
#: Busy fraction of the pairs (:func:`wave_fill`) under which a tile shape counts as underfilling.
PAIR_MIN_FILL = 0.75
#: 128-deep K blocks on the 256 x 256 tile: half the ring waits per multiply-add (three stages).
PAIR_DEEP_K = ActionCandidate(PairConfig(256, 256, 128, 4, 3, 8))
#: Its stream-K form, offered instead of :data:`PAIR_STREAM_K_CANDIDATE` (2-8% faster on 7 of 8
#: part-filled-wave grid and sweep shapes measured, 5% slower at M=2048 N=3584 K=18944).
PAIR_DEEP_K_STREAM_K = ActionCandidate(PairConfig(256, 256, 128, 4, 3, 8, PAIR_STREAM_K))
#: 256 x 128 tiles with 128-deep K blocks, twice as many tiles as 256 x 256: offered (with the
#: frozen 128 x 128 tile) while the 256 x 256 tiles underfill the pairs and M is at most
#: :data:`PAIR_NARROW_M_MAXIMUM`.
PAIR_NARROW = ActionCandidate(PairConfig(256, 128, 128, 4, 4, 8))
PAIR_NARROW_M_MAXIMUM = 1024


def wave_fill(tiles: int, slots: int) -> float:
    """Busy fraction of ``slots`` persistent workers over the waves ``tiles`` equal tiles take."""
    if tiles <= 0 or slots <= 0:
        return 0.0
    return tiles / (slots * -(-tiles // slots))


def pair_tiles_underfill(workload: Workload, sm_count: int = 148) -> bool:
    """Whether narrower tiles than 256 x 256 are worth offering (see :data:`PAIR_NARROW`)."""
    tiles = -(-workload.m // 256) * -(-workload.n // 256)
    return (
        workload.m <= PAIR_NARROW_M_MAXIMUM
        and wave_fill(tiles, resident_clusters(2, sm_count)) < PAIR_MIN_FILL
    )


def pair_candidates_for(workload: Workload, sm_count: int = 148) -> tuple[ActionCandidate, ...]:
    """B200 CTA-pair candidates for ``M > 128`` (empty below)."""
    if workload.m < PAIR_M_MINIMUM:
        return ()
    tiles = -(-workload.m // 256) * -(-workload.n // 256)
    wide_tiles = -(-workload.m // 256) * -(-workload.n // 512)
    k_blocks = -(-workload.k // 64)
    pairs = resident_clusters(2, sm_count)
    extra = (PAIR_DEEP_K,)
    if tiles <= 33:
        extra += (PAIR_SPLIT2,)
    if tiles <= 15:
        extra += (PAIR_SPLIT4,)
    if pair_stream_k_tiles(tiles, -(-workload.k // 128), pairs) > 0:
        extra += (PAIR_DEEP_K_STREAM_K,)
    if wave_fill(wide_tiles, pairs) >= PAIR_MIN_FILL:
        extra += (PAIR_WIDE,)
        if pair_stream_k_tiles(wide_tiles, k_blocks, pairs) > 0:
            extra += (PAIR_WIDE_STREAM_K,)
    if pair_tiles_underfill(workload, sm_count):
        extra += (PAIR_NARROW,)
    return _sorted((*PAIR_CANDIDATES, *extra))


#: Frozen candidates the B200 tuner keeps beside the B200 families. The others never won a grid
#: shape on the B200 (the CTA-pair family beats every single-SM tile above M = 128, the stream
#: family every tile and all but one split-K configuration below); leaving them out gives the
#: bandit's eight probes to the variants that compete.
B200_FROZEN_KEPT = frozenset(
    {
        "tile:m128n128k128-w8s3g8",
        "tile:m128n256k64-w8s4g8",
        "split_k:m16n64k64-w4s3-split4",
        "split_k:m16n128k64-w4s3-split4",
    }
)


#: The frozen tile that still wins a grid shape beside the CTA-pair family (M = 512), offered
#: where :func:`pair_tiles_underfill`; elsewhere above M = 128 the pair family alone is offered.
B200_FROZEN_KEPT_WITH_PAIRS = frozenset({"tile:m128n128k128-w8s3g8"})


def b200_candidates_for(workload: Workload) -> tuple[ActionCandidate, ...]:
    """Everything the B200 tuner may probe: the frozen candidates of :data:`B200_FROZEN_KEPT`
    that apply to the workload, plus the B200 families."""
    frozen = tuple(c for c in candidates_for(workload) if c.key in B200_FROZEN_KEPT)
    if workload.m <= 31:
        frozen = tuple(c for c in frozen if c.family == "split_k")
    elif workload.m >= PAIR_M_MINIMUM:
        keep = B200_FROZEN_KEPT_WITH_PAIRS if pair_tiles_underfill(workload) else frozenset()
        frozen = tuple(c for c in frozen if c.key in keep)
    return _sorted((*frozen, *stream_candidates_for(workload), *pair_candidates_for(workload)))


def action_set_manifest() -> dict[str, list[dict[str, Any]]]:
    """The frozen old/new action identities (``action_configs.py:122-131``)."""
    return {
        "old": [
            {"family": "old", "config_key": c.key, "config": c.to_dict()} for c in DEFAULT_CONFIGS
        ],
        "new": [
            {"family": c.family, "config_key": c.key, "config": c.to_dict()} for c in ALL_CANDIDATES
        ],
    }


# --------------------------------------------------------------------------------------------
# Launch planning of the weight-streaming kernels, shared by the launcher and the features.
# --------------------------------------------------------------------------------------------

#: Shared memory of one B200 SM and the per-CTA share the runtime reserves.
SMEM_PER_SM = 233472
SMEM_RESERVED_PER_CTA = 1024
#: Bytes of barriers, the TMEM address slot and alignment slack in a streaming CTA.
STREAM_SMEM_OVERHEAD = 2048


def stream_smem_bytes(block_m: int, block_n: int, block_k: int, stages: int) -> int:
    """Dynamic shared memory of one streaming CTA: the TMA ring, reused after the main loop for
    the FP32 partial the cluster reduction reads."""
    ring = stages * (block_n + block_m) * block_k * 2
    partial = block_n * block_m * 4
    return max(ring, partial) + STREAM_SMEM_OVERHEAD


def stream_ctas_per_sm(block_m: int, block_n: int, block_k: int, stages: int) -> int:
    per_cta = stream_smem_bytes(block_m, block_n, block_k, stages) + SMEM_RESERVED_PER_CTA
    by_smem = SMEM_PER_SM // per_cta
    columns = (block_n // 128) * block_m
    by_tmem = 512 // max(32, columns)
    return max(1, min(by_smem, by_tmem, 4))


def split_plan(k: int, block_k: int, splits: int) -> tuple[int, int]:
    """``(k_blocks_per_split, effective_splits)`` for contiguous block-aligned K intervals.

    Restates the reference's interval rule (``action_expansion.py:79-80``):
    ``tiles_per_split = cdiv(cdiv(K, BK), S)``. Splits that would start past K are dropped,
    so every launched split owns at least one K block.
    """
    k_blocks = -(-k // block_k)
    per_split = -(-k_blocks // splits)
    return per_split, -(-k_blocks // per_split)


def resident_clusters(size: int, sm_count: int) -> int:
    """Clusters of ``size`` CTAs (one per SM) a B200 keeps resident at once.

    ``cudaOccupancyMaxActiveClusters`` on the 148-SM B200 gives 148, 74, 45, 33, 26, 22, 15 and
    15 for clusters of 1 to 8 CTAs (the GPCs fit fewer large clusters); scaled to ``sm_count``.
    """
    per148 = {1: 148, 2: 74, 3: 45, 4: 33, 5: 26, 6: 22, 7: 15, 8: 15}[size]
    return per148 * sm_count // 148


def stream_splits(m: int, n: int, k: int, config: StreamConfig, sm_count: int) -> int:
    """The cluster size (K splits) a :class:`StreamConfig` launches with on ``sm_count`` SMs.

    Automatic: of 1..8, the split count giving the most CTAs (column tiles x splits) whose
    clusters are all resident in one wave, the smallest on a tie. As the launcher does, a count
    must give every split K blocks and all but the last the same number (else the next lower).
    """
    k_blocks = -(-k // config.block_k)

    def k_splits_ok(s: int) -> bool:
        return s <= k_blocks and -(-k_blocks // -(-k_blocks // s)) == s

    splits = config.split_k
    if splits == 0:
        n_tiles = -(-n // config.block_n)
        splits = 1
        for s in range(2, 9):
            if n_tiles <= resident_clusters(s, sm_count) and k_splits_ok(s) and s > splits:
                splits = s
    while splits > 1 and not k_splits_ok(splits):
        splits -= 1
    return splits
