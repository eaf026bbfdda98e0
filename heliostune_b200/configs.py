"""Launch configurations and the projection workloads of the FP16 matmul path.

The dataclasses keep the reference's field names, validation rules and ``key`` strings
(``src/heliostune/configs.py:11-51`` for :class:`KernelConfig`, ``:54-96`` for :class:`Workload`,
``:269-356`` for :class:`HopperGemmConfig`) so manifests, checkpoints and bandit features written
against the reference stay valid. What a field means on a B200 is stated on each class.
"""

from __future__ import annotations

from dataclasses import asdict, dataclass

from heliostune_b200.errors import SchemaError
from heliostune_b200.validation import exact_bool, exact_fields, exact_int, nonblank_string

#: A TMA tensor map needs 16-byte aligned row strides: FP16 rows of a multiple of 8 elements.
TENSOR_DESCRIPTOR_ALIGNMENT = 8

#: Smallest block edge the reference accepts for a tensor-core tile.
TENSOR_CORE_MIN_DOT_DIMENSION = 16


def _power_of_two(value: int) -> bool:
    return value > 0 and value & (value - 1) == 0


@dataclass(frozen=True, slots=True)
class KernelConfig:
    """One tile-GEMM launch configuration (the reference's "old"/"tile" family).

    On a B200 the configuration selects an instantiation of the tcgen05 tile kernel:

    * ``block_m`` -- rows of C per CTA. 16..64 run one M=64 UMMA atom, 128 one M=128 atom and
      256 two M=128 atoms (two TMEM accumulators) in one CTA.
    * ``block_n`` -- columns of C per CTA and the UMMA N; 32 is widened to 64 (one 128-byte
      swizzle atom of B).
    * ``block_k`` -- K extent of one shared-memory stage; 32 is widened to 64 (one 128-byte
      swizzle atom of A).
    * ``num_stages`` -- depth of the TMA -> UMMA shared-memory ring.
    * ``group_m`` -- raster group of the tile order, exactly as the reference's 1-D grid.
    * ``num_warps`` -- kept for the key and the bandit features; the B200 CTA always runs one
      TMA warp, one UMMA warp and four epilogue warps.
    """

    block_m: int
    block_n: int
    block_k: int
    num_warps: int
    num_stages: int
    group_m: int = 8

    def __post_init__(self) -> None:
        for name in ("block_m", "block_n", "block_k", "num_warps", "num_stages", "group_m"):
            exact_int(getattr(self, name), context=f"kernel config {name}", minimum=1)
        for name in ("block_m", "block_n", "block_k"):
            if not _power_of_two(getattr(self, name)):
                raise SchemaError(f"{name} must be a power of two")
        if self.num_warps not in (1, 2, 4, 8):
            raise SchemaError("num_warps must be one of 1, 2, 4, or 8")

    @property
    def key(self) -> str:
        return (
            f"m{self.block_m}n{self.block_n}k{self.block_k}"
            f"-w{self.num_warps}s{self.num_stages}g{self.group_m}"
        )

    def to_dict(self) -> dict[str, int]:
        return asdict(self)

    @classmethod
    def from_dict(cls, value: object) -> KernelConfig:
        names = ("block_m", "block_n", "block_k", "num_warps", "num_stages", "group_m")
        data = exact_fields(value, required=names, context="kernel config")
        return cls(**{n: exact_int(data[n], context=f"kernel config {n}", minimum=1) for n in names})


@dataclass(frozen=True, slots=True)
class Workload:
    """A row-major ``A[M,K] @ B[K,N]`` projection."""

    m: int
    n: int
    k: int
    model: str
    projection: str
    regime: str

    def __post_init__(self) -> None:
        for name in ("m", "n", "k"):
            exact_int(getattr(self, name), context=f"workload {name}", minimum=1)
        for name in ("model", "projection", "regime"):
            nonblank_string(getattr(self, name), context=f"workload {name}")

    @property
    def key(self) -> str:
        return f"{self.model}-{self.projection}-{self.regime}-m{self.m}-n{self.n}-k{self.k}"

    @property
    def flops(self) -> int:
        return 2 * self.m * self.n * self.k

    @property
    def ideal_bytes(self) -> int:
        """Algorithmic FP16 traffic: read A and B once, write C once."""
        return 2 * (self.m * self.k + self.k * self.n + self.m * self.n)

    def to_dict(self) -> dict[str, int | str]:
        return asdict(self)

    @classmethod
    def from_dict(cls, value: object) -> Workload:
        data = exact_fields(
            value, required=("m", "n", "k", "model", "projection", "regime"), context="workload"
        )
        return cls(
            m=exact_int(data["m"], context="workload m", minimum=1),
            n=exact_int(data["n"], context="workload n", minimum=1),
            k=exact_int(data["k"], context="workload k", minimum=1),
            model=nonblank_string(data["model"], context="workload model"),
            projection=nonblank_string(data["projection"], context="workload projection"),
            regime=nonblank_string(data["regime"], context="workload regime"),
        )


@dataclass(frozen=True, slots=True)
class ModelSpec:
    """Public decoder dimensions a projection corpus is derived from."""

    name: str
    hidden_size: int
    intermediate_size: int
    attention_heads: int
    key_value_heads: int

    @property
    def key_value_size(self) -> int:
        return self.hidden_size // self.attention_heads * self.key_value_heads


def projection_shapes(model: ModelSpec) -> tuple[tuple[str, int, int], ...]:
    """``(projection, N, K)`` of the four decoder projections (fused QKV, out, up, down)."""
    return (
        ("attention-qkv", model.hidden_size + 2 * model.key_value_size, model.hidden_size),
        ("attention-out", model.hidden_size, model.hidden_size),
        ("ffn-up", model.intermediate_size, model.hidden_size),
        ("ffn-down", model.hidden_size, model.intermediate_size),
    )


#: The reference's corpus models (``src/heliostune/configs.py:130-163``).
MODEL_SPECS: tuple[ModelSpec, ...] = (
    ModelSpec("mistral-7b", 4096, 14336, 32, 8),
    ModelSpec("qwen2.5-7b", 3584, 18944, 28, 4),
    ModelSpec("phi-3-mini", 3072, 8192, 32, 32),
    ModelSpec("granite-3.1-8b", 4096, 12800, 32, 8),
)

#: Token regimes of the reference corpus (``src/heliostune/configs.py:220-227``).
TOKEN_REGIMES: tuple[tuple[str, int], ...] = (
    ("decode-1", 1),
    ("decode-7", 7),
    ("mixed-31", 31),
    ("mixed-96", 96),
    ("prefill-257", 257),
    ("prefill-1024", 1024),
)

#: The reference's 96 published workloads, in its order (``src/heliostune/configs.py:239-251``).
DEFAULT_WORKLOADS: tuple[Workload, ...] = tuple(
    Workload(m=tokens, n=n, k=k, model=model.name, projection=projection, regime=regime)
    for model in MODEL_SPECS
    for projection, n, k in projection_shapes(model)
    for regime, tokens in TOKEN_REGIMES
)


def _tile_warps(block_m: int, block_n: int) -> int:
    return 8 if block_m * block_n >= 8192 else 4


_OLD_TILES = tuple((bm, bn) for bm in (16, 32, 64, 128) for bn in (32, 64, 128))

#: The 36 stock tile configurations (``src/heliostune/configs.py:166-186``), in the same order.
DEFAULT_CONFIGS: tuple[KernelConfig, ...] = (
    tuple(KernelConfig(bm, bn, 32, _tile_warps(bm, bn), 3, 8) for bm, bn in _OLD_TILES)
    + tuple(KernelConfig(bm, bn, 64, _tile_warps(bm, bn), 2, 8) for bm, bn in _OLD_TILES)
    + tuple(KernelConfig(bm, bn, 32, _tile_warps(bm, bn), 4, 4) for bm, bn in _OLD_TILES)
)


@dataclass(frozen=True, slots=True)
class HopperGemmConfig:
    """A persistent tile-scheduler GEMM configuration (the reference's "persistent" family).

    The name is the reference's (``src/heliostune/configs.py:269-356``); on a B200 it selects the
    persistent tcgen05 kernel: a grid of one CTA per SM walks the tiles in ``group_m`` raster order
    with two TMEM accumulators, so the epilogue of one tile overlaps the main loop of the next.
    ``epilogue_subtile`` and ``warp_specialize`` are accepted for manifest compatibility; the B200
    kernel is always warp-specialised and always drains the accumulator in 64-column sub-tiles.
    """

    block_m: int
    block_n: int
    block_k: int
    num_warps: int
    num_stages: int
    group_m: int = 8
    epilogue_subtile: bool = False
    warp_specialize: bool = False

    def __post_init__(self) -> None:
        for name in ("block_m", "block_n", "block_k", "num_warps", "num_stages", "group_m"):
            exact_int(getattr(self, name), context=f"hopper gemm config {name}", minimum=1)
        for name in ("epilogue_subtile", "warp_specialize"):
            exact_bool(getattr(self, name), context=f"hopper gemm config {name}")
        for name in ("block_m", "block_n", "block_k"):
            if not _power_of_two(getattr(self, name)):
                raise SchemaError(f"{name} must be a power of two")
        if self.num_warps not in (1, 2, 4, 8):
            raise SchemaError("num_warps must be one of 1, 2, 4, or 8")
        for name in ("block_m", "block_n", "block_k"):
            if getattr(self, name) < TENSOR_CORE_MIN_DOT_DIMENSION:
                raise SchemaError(f"{name} must be at least {TENSOR_CORE_MIN_DOT_DIMENSION}")
        for name in ("block_n", "block_k"):
            if getattr(self, name) % TENSOR_DESCRIPTOR_ALIGNMENT:
                raise SchemaError(
                    f"{name} must be a multiple of {TENSOR_DESCRIPTOR_ALIGNMENT} elements"
                )
        if self.epilogue_subtile and (self.block_n // 2) % TENSOR_DESCRIPTOR_ALIGNMENT:
            raise SchemaError(
                "a subtiled epilogue stores block_n // 2 columns, which must be a "
                f"multiple of {TENSOR_DESCRIPTOR_ALIGNMENT} elements"
            )

    @property
    def key(self) -> str:
        return (
            f"hopper-m{self.block_m}n{self.block_n}k{self.block_k}"
            f"-w{self.num_warps}s{self.num_stages}g{self.group_m}"
            f"-sub{int(self.epilogue_subtile)}-ws{int(self.warp_specialize)}"
        )

    def to_dict(self) -> dict[str, int | bool]:
        return asdict(self)

    @classmethod
    def from_dict(cls, value: object) -> HopperGemmConfig:
        ints = ("block_m", "block_n", "block_k", "num_warps", "num_stages", "group_m")
        flags = ("epilogue_subtile", "warp_specialize")
        data = exact_fields(value, required=ints + flags, context="hopper gemm config")
        kwargs: dict[str, int | bool] = {
            n: exact_int(data[n], context=f"hopper gemm config {n}", minimum=1) for n in ints
        }
        for n in flags:
            kwargs[n] = exact_bool(data[n], context=f"hopper gemm config {n}")
        return cls(**kwargs)  # type: ignore[arg-type]


#: Shapes the published corpus never produces (``src/heliostune/hopper_spec.py:19-23``):
#: a minimum descriptor, partial N/K tiles, and partial rows.
EDGE_WORKLOADS: tuple[Workload, ...] = (
    Workload(m=1, n=8, k=8, model="synthetic", projection="descriptor-minimum", regime="edge"),
    Workload(m=7, n=136, k=264, model="synthetic", projection="partial-tiles", regime="edge"),
    Workload(m=131, n=1032, k=520, model="synthetic", projection="partial-rows", regime="edge"),
)


def validation_workloads(
    workloads: tuple[Workload, ...] | list[Workload] = DEFAULT_WORKLOADS,
    *,
    edges: tuple[Workload, ...] | list[Workload] = EDGE_WORKLOADS,
) -> tuple[Workload, ...]:
    """The pre-timing gate's sample (``hopper_spec.py:26-55``): per token regime the workloads with
    the smallest and the largest N x K, then the edge shapes, each once, in that order."""
    from heliostune_b200.errors import ProtocolError

    if not workloads:
        raise ProtocolError("validation workload manifest must not be empty")
    regimes: dict[str, list[Workload]] = {}
    for workload in workloads:
        if type(workload) is not Workload:
            raise ProtocolError("validation workload manifest must contain only Workload values")
        regimes.setdefault(workload.regime, []).append(workload)
    chosen: dict[str, Workload] = {}
    for regime in sorted(regimes):
        by_size = sorted(regimes[regime], key=lambda w: (w.n * w.k, w.key))
        chosen.setdefault(by_size[0].key, by_size[0])
        chosen.setdefault(by_size[-1].key, by_size[-1])
    for workload in edges:
        if type(workload) is not Workload:
            raise ProtocolError("validation edge manifest must contain only Workload values")
        chosen.setdefault(workload.key, workload)
    return tuple(chosen.values())


# --------------------------------------------------------------------------------------------
# The measurement grids of this build (Llama-3-8B and Qwen2.5-7B projections).
# --------------------------------------------------------------------------------------------

LLAMA3_8B_PAIRS: tuple[tuple[str, int, int], ...] = (
    ("attention-qkv", 4096, 6144),
    ("attention-out", 4096, 4096),
    ("ffn-gate-up", 4096, 28672),
    ("ffn-down", 14336, 4096),
)
QWEN25_7B_PAIRS: tuple[tuple[str, int, int], ...] = (
    ("attention-qkv", 3584, 4608),
    ("attention-out", 3584, 3584),
    ("ffn-gate-up", 3584, 37888),
    ("ffn-down", 18944, 3584),
)

GRID_M: tuple[int, ...] = (1, 2, 4, 8, 16, 31, 32, 64, 128, 512, 2048, 8192)
SWEEP_M: tuple[int, ...] = (1, 16, 31, 64, 256, 1024, 4096)


def _grid(pairs: tuple[tuple[str, str, int, int], ...], ms: tuple[int, ...]) -> tuple[Workload, ...]:
    return tuple(
        Workload(m=m, n=n, k=k, model=model, projection=projection, regime=f"m{m}")
        for model, projection, k, n in pairs
        for m in ms
    )


_GRID_PAIRS = tuple(("llama-3-8b", p, k, n) for p, k, n in LLAMA3_8B_PAIRS) + tuple(
    ("qwen2.5-7b", p, k, n) for p, k, n in QWEN25_7B_PAIRS
)

#: The 96-shape FP16 grid: 8 (K, N) pairs x 12 values of M.
GRID_WORKLOADS: tuple[Workload, ...] = _grid(_GRID_PAIRS, GRID_M)

#: The 28-shape Llama-3-8B projection sweep.
SWEEP_WORKLOADS: tuple[Workload, ...] = _grid(_GRID_PAIRS[:4], SWEEP_M)

#: The single decode GEMM sized like Qwen2.5-7B FFN-down at M=1.
DECODE_WORKLOAD = Workload(
    m=1, n=3584, k=18944, model="qwen2.5-7b", projection="ffn-down", regime="m1"
)

#: The column-parallel GEMM sized like Llama-3-70B gate-up.
COLUMN_PARALLEL_WORKLOAD = Workload(
    m=8192, n=57344, k=8192, model="llama-3-70b", projection="ffn-gate-up", regime="m8192"
)
