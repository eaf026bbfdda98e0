"""Device timing with CUDA events, the role ``triton.testing.do_bench`` plays in the reference.

``do_bench`` follows the protocol the reference times every action with
(``src/heliostune/kernel.py:141-158``, warm-up 25 ms, repetition 100 ms, quantiles p20/p50/p80):
estimate one call, run enough warm-up calls to fill ``warmup_ms``, then time enough calls to fill
``rep_ms``, each one preceded by a write of a 256 MiB buffer so L2 (126 MB on a B200) holds
nothing of the previous call. Each call is bracketed by events on the current stream.
"""

from __future__ import annotations

from collections.abc import Callable, Sequence

import torch

_FLUSH_BYTES = 256 * 1024 * 1024
_flush_buffers: dict[int, torch.Tensor] = {}


def flush_buffer(device: torch.device | None = None) -> torch.Tensor:
    index = torch.cuda.current_device() if device is None or device.index is None else device.index
    buffer = _flush_buffers.get(index)
    if buffer is None:
        buffer = torch.empty(_FLUSH_BYTES // 4, dtype=torch.int32, device=f"cuda:{index}")
        _flush_buffers[index] = buffer
    return buffer


def flush_l2(device: torch.device | None = None) -> None:
    flush_buffer(device).zero_()


def quantiles_of(values: Sequence[float], qs: Sequence[float]) -> list[float]:
    ordered = torch.tensor(sorted(values), dtype=torch.float64)
    return [float(torch.quantile(ordered, q)) for q in qs]


def do_bench(
    fn: Callable[[], object],
    *,
    warmup_ms: float = 25.0,
    rep_ms: float = 100.0,
    quantiles: Sequence[float] = (0.2, 0.5, 0.8),
    max_reps: int = 1000,
) -> list[float]:
    """Latency quantiles in milliseconds of ``fn`` with a cold L2 before every call."""
    buffer = flush_buffer()
    fn()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(5):
        buffer.zero_()
        fn()
    end.record()
    torch.cuda.synchronize()
    estimate = max(start.elapsed_time(end) / 5, 1e-3)
    n_warmup = max(1, int(warmup_ms / estimate))
    n_repeat = max(1, min(max_reps, int(rep_ms / estimate)))
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(n_repeat)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(n_repeat)]
    for _ in range(n_warmup):
        fn()
    for i in range(n_repeat):
        buffer.zero_()
        starts[i].record()
        fn()
        ends[i].record()
    torch.cuda.synchronize()
    times = [s.elapsed_time(e) for s, e in zip(starts, ends, strict=True)]
    return quantiles_of(times, quantiles)
