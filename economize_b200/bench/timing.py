"""Device timing of GPU work (economize ``bench/timing.py:1-252``, re-done for multi-GPU runs).

:func:`time_call` brackets ``iters`` calls with CUDA events on the launching stream after ``warmup`` calls, with a
synchronize on both sides, optionally overwriting a buffer larger than L2 before every timed call (``flush_l2``) so
that each call reads its inputs from HBM. Under ``torch.distributed`` the per-rank times are reduced with MAX:
a multi-GPU step is as slow as its slowest rank.
"""

from __future__ import annotations

import statistics
from collections.abc import Callable
from dataclasses import dataclass, field

import torch
import torch.distributed as dist

__all__ = ["Timing", "max_over_ranks", "time_call", "time_graph"]

L2_BYTES = 126 * 1024 * 1024


@dataclass
class Timing:
    """Per-call device times in milliseconds (max over ranks when distributed)."""

    times_ms: list[float] = field(default_factory=list)

    @property
    def mean_ms(self) -> float:
        return statistics.fmean(self.times_ms) if self.times_ms else float("nan")

    @property
    def median_ms(self) -> float:
        return statistics.median(self.times_ms) if self.times_ms else float("nan")

    @property
    def min_ms(self) -> float:
        return min(self.times_ms) if self.times_ms else float("nan")


def max_over_ranks(value: float, device: torch.device | None = None) -> float:
    """``value`` maxed over the ranks of the default process group (itself when not distributed)."""
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device or "cpu")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


_flush_buf: dict[torch.device, torch.Tensor] = {}


def flush_l2(device: torch.device) -> None:
    """Overwrite a buffer 2x the L2 size so that the next kernel starts from a cold cache."""
    buf = _flush_buf.get(device)
    if buf is None:
        buf = _flush_buf[device] = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=device)
    buf.fill_(1.0)


def time_call(fn: Callable[[], object], iters: int = 20, warmup: int = 3, flush: bool = True,
              device: torch.device | str | None = None) -> Timing:
    """Time ``fn`` on the current CUDA stream; each timed call has its own event pair so an L2 flush between calls
    is not counted."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize(dev)
    if dist.is_available() and dist.is_initialized():
        dist.barrier()
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(iters)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(iters)]
    for i in range(iters):
        if flush:
            flush_l2(dev)
        starts[i].record()
        fn()
        ends[i].record()
    torch.cuda.synchronize(dev)
    times = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    return Timing([max_over_ranks(t, dev if dist.is_initialized() and dist.get_backend() == "nccl" else None)
                   for t in times])


def time_graph(calls: list[Callable[[], object]], replays: int = 10, warmup: int = 3) -> float:
    """Device milliseconds per call of ``calls`` captured back to back in one CUDA graph (launch overhead excluded).

    Give the calls distinct inputs whose total size exceeds L2 (rotating weight copies) so that every call reads
    from HBM, as it would inside a model step.
    """
    for fn in calls:
        fn()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for fn in calls:
            fn()
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(replays):
        graph.replay()
    end.record()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end) / (replays * len(calls))
    del graph
    return max_over_ranks(ms)
