"""Column-parallel (N-sharded) GEMM across the GPUs of one node, joined by an all-gather.

No reference counterpart: the reference has no multi-GPU code. Rank ``r`` of ``P`` holds the
replicated A ``[M, K]`` and the column slice ``B[:, r*N/P : (r+1)*N/P]``; it computes its slice
``C_r = A @ B_r`` with the B200 GEMM, the slices are all-gathered over NVLink (NCCL), and
``hst_column_assemble`` writes the rank-ordered ``[P, M, N/P]`` chunks into the columns of a
row-major ``C [M, N]``. Every rank ends with the full C. Each GEMM is a single-GPU launch on
local memory; no TMA load in this library reads another GPU's memory or feeds several CTAs.
"""

from __future__ import annotations

from collections.abc import Callable
from dataclasses import dataclass

import torch
import torch.distributed as dist

from heliostune_b200 import _native
from heliostune_b200.action_configs import ActionCandidate, PairConfig
from heliostune_b200.kernel import _device_guard, _stream

#: The GEMM configurations a rank uses for its slice (large M, wide N): CTA-pair 256 x 256
#: tiles, or 256 x 512 tiles (a quarter fewer L2-to-SM bytes per FLOP, about 7% faster per FLOP
#: on the B200) when their coarser last wave does not give that back.
COLUMN_PARALLEL_CANDIDATE = ActionCandidate(PairConfig(256, 256, 64, 4, 6, 8))
COLUMN_PARALLEL_WIDE = ActionCandidate(PairConfig(256, 512, 64, 4, 4, 16))


def column_parallel_candidate(m: int, cols: int, sm_count: int = 148) -> ActionCandidate:
    """The slice GEMM's configuration: whole waves of 74 pairs, a 256 x 512 tile costing 1.86
    256 x 256 tiles."""
    pairs = sm_count // 2

    def waves(tiles: int) -> int:
        return -(-tiles // pairs)

    rows = -(-m // 256)
    wide = waves(rows * -(-cols // 512)) * 1.86
    return COLUMN_PARALLEL_WIDE if wide < waves(rows * -(-cols // 256)) else COLUMN_PARALLEL_CANDIDATE


@dataclass(frozen=True)
class ColumnShard:
    """The columns of C (and of B) rank ``rank`` of ``world`` owns."""

    n_total: int
    world: int
    rank: int

    def __post_init__(self) -> None:
        if self.world < 1 or not 0 <= self.rank < self.world:
            raise ValueError("rank must be in [0, world)")
        if self.n_total < 1 or self.n_total % self.world:
            raise ValueError(f"N={self.n_total} must split evenly over {self.world} ranks")

    @property
    def cols(self) -> int:
        return self.n_total // self.world

    @property
    def start(self) -> int:
        return self.rank * self.cols

    @property
    def stop(self) -> int:
        return self.start + self.cols

    def take(self, b: torch.Tensor) -> torch.Tensor:
        """This rank's slice of a full ``B [K, N]`` as a contiguous ``[K, N/P]`` tensor."""
        return b[:, self.start : self.stop].contiguous()


def assemble_columns(gathered: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """``out[:, p*Nc:(p+1)*Nc] = gathered[p]`` on the GPU (``hst_column_assemble``)."""
    if gathered.ndim != 3 or gathered.dtype != torch.float16 or not gathered.is_contiguous():
        raise ValueError("gathered must be a contiguous FP16 [parts, rows, cols] tensor")
    parts, rows, cols = gathered.shape
    if out is None:
        out = torch.empty((rows, parts * cols), dtype=torch.float16, device=gathered.device)
    if out.shape != (rows, parts * cols) or out.stride(1) != 1:
        raise ValueError("out must be [rows, parts * cols] with unit column stride")
    with _device_guard(gathered.device):
        _native.check(
            _native.library().hst_column_assemble(
                gathered.data_ptr(),
                out.data_ptr(),
                parts,
                rows,
                cols,
                out.stride(0),
                _stream(gathered.device),
            )
        )
    return out


#: How the fused GEMM writes into the peers' C: coalesced 16-byte stores from the epilogue warps,
#: or one TMA tensor store per peer of every staged sub-tile.
PEER_WRITES = {"stores": _native.HST_PEER_STORES, "bulk": _native.HST_PEER_BULK}


def default_peer_writes(world: int) -> str:
    """The peer-write form measured fastest at this rank count: TMA tensor stores at two ranks
    (1-3% shorter steps on the B200), the epilogue warps' stores otherwise (the form measured at
    four and eight)."""
    return "bulk" if world == 2 else "stores"


class FusedColumnParallel:
    """Column-parallel GEMM whose all-gather is fused into the GEMM epilogue.

    Every rank allocates its full output ``C [M, N]`` once (``torch.empty``), exports its CUDA
    IPC handle, and maps every peer's output (``hst_ipc_*``). A call runs the persistent CTA-pair
    GEMM on this rank's column slice; each finished sub-tile goes to the local C by TMA and to
    every peer's C over NVLink while the next tiles compute (``hst_matmul_pair_fanout``), by
    coalesced stores from the epilogue warps or by TMA tensor stores (``peer_writes``). Barriers
    on the stream before and after the launch order the ranks without NCCL
    (``hst_peer_barrier``: each rank stores the call's epoch into barrier words kept behind every
    peer's C and waits for the peers' stores into its own): no peer writes into a C that is still
    being read, and C is complete when the call returns.
    The returned tensor is this object's buffer and is overwritten by the next call.
    """

    def __init__(
        self,
        m: int,
        n_total: int,
        *,
        group: dist.ProcessGroup | None = None,
        candidate: ActionCandidate | None = None,
        device: torch.device | None = None,
        peer_writes: str | None = None,
    ) -> None:
        import ctypes

        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if peer_writes is None:
            peer_writes = default_peer_writes(self.world)
        if peer_writes not in PEER_WRITES:
            raise ValueError(f"peer_writes must be one of {tuple(PEER_WRITES)}, not {peer_writes!r}")
        self.peer_writes = peer_writes
        self.shard = ColumnShard(n_total, self.world, self.rank)
        if candidate is None:
            candidate = column_parallel_candidate(m, self.shard.cols)
        if not isinstance(candidate.config, PairConfig):
            raise ValueError("the fused column-parallel GEMM runs the CTA-pair kernel")
        self.candidate = candidate
        self.device = device or torch.device("cuda", torch.cuda.current_device())
        # One allocation per rank, so one IPC mapping per peer: C, then (256-byte aligned) the
        # 2 x world barrier words of hst_peer_barrier, zero before the first barrier.
        c_bytes = m * n_total * 2
        words_offset = -(-c_bytes // 256) * 256
        storage = torch.empty(words_offset + 2 * self.world * 8, dtype=torch.uint8, device=self.device)
        self.out = storage[:c_bytes].view(torch.float16).view(m, n_total)
        self._words = storage[words_offset:].view(torch.int64)
        self._words.zero_()
        self._epoch = 0
        torch.cuda.synchronize(self.device)  # zero before any peer can write into it
        lib = _native.library()
        handle = (ctypes.c_char * 64)()
        offset = ctypes.c_uint64(0)
        _native.check(lib.hst_ipc_export(self.out.data_ptr(), handle, ctypes.byref(offset)))
        mine = (bytes(handle), offset.value)
        gathered: list[object] = [None] * self.world
        if self.world > 1:
            dist.all_gather_object(gathered, mine, group=group)
        else:
            gathered = [mine]
        self._bases: list[int] = []
        pointers = []
        for q, (raw, off) in enumerate(gathered):  # type: ignore[misc]
            if q == self.rank:
                pointers.append(self.out.data_ptr())
                continue
            base = ctypes.c_void_p()
            _native.check(lib.hst_ipc_import(raw, ctypes.byref(base)))
            self._bases.append(base.value)
            pointers.append(base.value + off)
        self._pointers = (ctypes.c_void_p * self.world)(*pointers)
        self._word_pointers = (ctypes.c_void_p * self.world)(*(p + words_offset for p in pointers))

    def _barrier(self, slot: int) -> None:
        """Every rank's stream reaches this point before work after it runs (hst_peer_barrier:
        stores into the peers' barrier words over NVLink and a bounded wait on its own)."""
        if self.world > 1:
            _native.check(
                _native.library().hst_peer_barrier(
                    self._word_pointers, self.world, self.rank, slot, self._epoch, 0, _stream(self.device)
                )
            )

    def __call__(
        self,
        a: torch.Tensor,
        b_shard: torch.Tensor,
        phase_events: list[torch.cuda.Event] | None = None,
    ) -> torch.Tensor:
        config = self.candidate.config
        m, k = a.shape
        if b_shard.shape != (k, self.shard.cols) or m != self.out.shape[0]:
            raise ValueError("operand shapes do not match this column-parallel plan")
        if not (a.is_contiguous() and b_shard.is_contiguous()):
            raise ValueError("operands must be row-major contiguous")
        if phase_events:
            phase_events[0].record()
        self._epoch += 1
        self._barrier(0)  # every rank is done reading the previous result
        _native.check(
            _native.library().hst_matmul_pair_fanout(
                config.block_n,
                config.block_k,
                config.num_stages,
                config.group_m,
                a.data_ptr(),
                b_shard.data_ptr(),
                self._pointers,
                self.world,
                self.rank,
                m,
                self.shard.n_total,
                k,
                PEER_WRITES[self.peer_writes],
                _stream(self.device),
            )
        )
        if phase_events:
            phase_events[1].record()
        self._barrier(1)  # every rank's slices have landed everywhere
        if phase_events:
            phase_events[2].record()
        return self.out

    def close(self) -> None:
        lib = _native.library()
        torch.cuda.synchronize(self.device)
        for base in self._bases:
            _native.check(lib.hst_ipc_close(base))
        self._bases = []


def _default_gemm(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    from heliostune_b200.action_expansion import launch

    return launch(a, b, column_parallel_candidate(a.shape[0], b.shape[1]))


def column_parallel_matmul(
    a: torch.Tensor,
    b_shard: torch.Tensor,
    *,
    group: dist.ProcessGroup | None = None,
    gemm: Callable[[torch.Tensor, torch.Tensor], torch.Tensor] | None = None,
    assemble: Callable[[torch.Tensor], torch.Tensor] | None = None,
    phase_events: list[torch.cuda.Event] | None = None,
) -> torch.Tensor:
    """Full ``C = A @ B`` on every rank from this rank's column slice of B.

    ``gemm`` and ``assemble`` default to the B200 kernels; tests on CPU ranks pass host
    implementations to exercise the sharding and gather logic. ``phase_events`` (three CUDA
    events) are recorded before the GEMM, after the GEMM and after the assembly, so callers can
    time the two phases on the launching stream.
    """
    gemm = gemm or _default_gemm
    assemble = assemble or assemble_columns
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    if phase_events:
        phase_events[0].record()
    local = gemm(a, b_shard)
    if phase_events:
        phase_events[1].record()
    if world == 1:
        if phase_events:
            phase_events[2].record()
        return local  # one rank: the slice is the whole product
    else:
        rows, cols = local.shape
        flat = torch.empty((world * rows, cols), dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(flat, local.contiguous(), group=group)
        gathered = flat.view(world, rows, cols)
    out = assemble(gathered)
    if phase_events:
        phase_events[2].record()
    return out
