"""Fused collectives over NVLink peer memory for tensor parallelism.

:class:`FusedAllReduce` allocates one IPC-exportable buffer per rank (``csrc/comm.cu``), exchanges the handles
once through ``torch.distributed`` and maps every peer's buffer. Each all-reduce of a row-parallel projection is
then two kernels on the rank's stream: ``push`` stores the rank's partial into its slot of every peer's buffer with
P2P stores and signals arrival with system-scope atomics; ``reduce_rmsnorm`` waits (bounded) for all ranks, sums the
slots in rank order, adds the residual and applies the next RMSNorm. No NCCL call and no host synchronization is
involved, so the sequence is captured in the cycle's CUDA graph. Every forward pass issues an even number of
all-reduces (two per block), so the alternating buffer parity is the same at capture and at every replay.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from .. import ops
from ..errors import CommTimeoutError, ConfigError

__all__ = ["FusedAllReduce", "Pushed"]


class Pushed:
    """A row-parallel projection output that its GEMM already stored into every peer's slot (push mode)."""

    def __init__(self, rows: int, shape: torch.Size, like: torch.Tensor, parity: int) -> None:
        self.rows, self.shape, self.like, self.parity = rows, shape, like, parity


class FusedAllReduce:
    """NVLink push / reduce runtime of one tensor-parallel group.

    Args:
        tp: The group (its ranks must share a node and see each other over NVLink).
        hidden: Width of the reduced rows.
        max_tokens: Most rows one all-reduce carries (larger passes fall back to NCCL).
    """

    def __init__(self, tp, hidden: int, max_tokens: int = 4096) -> None:
        if tp.size > 8:
            raise ConfigError("the fused all-reduce supports up to 8 ranks")
        self.tp = tp
        self.hidden = hidden
        self.max_tokens = max_tokens
        self.slot_elems = max_tokens * hidden
        ext = ops.require()
        self.ext = ext
        nbytes = ext.symm_control_bytes() + 2 * tp.size * self.slot_elems * 2
        self.own, handle = ext.symm_alloc(nbytes)
        handles: list = [None] * tp.size
        dist.all_gather_object(handles, handle, group=tp.group)
        self.ptrs = [self.own if r == tp.rank else ext.symm_open(h) for r, h in enumerate(handles)]
        dist.barrier(group=tp.group)
        self.calls = 0

    def fits(self, rows: int) -> bool:
        return rows <= self.max_tokens

    def gemm_push(self, x: torch.Tensor, weight: torch.Tensor) -> Pushed:
        """Row-parallel ``x @ weight.T`` whose output tiles the GEMM stores straight into every peer's slot (the
        GEMM -> all-reduce fusion); :meth:`reduce_rmsnorm` consumes the result."""
        shape = (*x.shape[:-1], weight.shape[0])
        rows = x.numel() // x.shape[-1]
        parity = self.calls % 2
        self.calls += 1
        self.ext.linear_push(x.reshape(rows, x.shape[-1]), weight, self.ptrs, self.tp.rank, parity,
                             self.slot_elems)
        return Pushed(rows, torch.Size(shape), x, parity)

    def reduce_rmsnorm(self, partial: torch.Tensor | Pushed, weight: torch.Tensor, eps: float,
                       residual: torch.Tensor | None) -> tuple[torch.Tensor, torch.Tensor]:
        """``(rmsnorm(sum_ranks(partial) + residual) * weight, sum_ranks(partial) + residual)``."""
        if isinstance(partial, Pushed):
            shape, rows, parity, like = partial.shape, partial.rows, partial.parity, partial.like
        else:
            shape = partial.shape
            rows = partial.numel() // self.hidden
            parity = self.calls % 2
            self.calls += 1
            like = partial
            self.ext.push(partial.reshape(rows, self.hidden), self.ptrs, self.tp.rank, parity, self.slot_elems)
        res = None if residual is None else residual.reshape(rows, self.hidden)
        out, resid = self.ext.reduce_rmsnorm(self.ptrs, self.tp.rank, parity, self.slot_elems, res, weight,
                                             float(eps), rows, self.hidden, like)
        return out.reshape(shape), resid.reshape(shape)

    def check(self) -> None:
        """Raise :class:`CommTimeoutError` if a bounded wait of this device gave up since the last check."""
        status = self.ext.status(torch.cuda.current_device())
        if status & 8:
            raise CommTimeoutError(f"a peer's partial did not arrive in time (status {status})")

    def close(self) -> None:
        for r, p in enumerate(self.ptrs):
            if r != self.tp.rank:
                self.ext.symm_close(p)
        self.ext.symm_free(self.own)
        self.ptrs = []
