"""Sequence-parallel fused tensor parallelism: GEMM -> reduce-scatter and all-gather -> GEMM over NVLink.

Megatron-style sharding of the weights (:func:`~economize_b200.parallel.tp.shard_model`) with the residual stream
split by token between the sublayers (``csrc/tp_sp.cu``). Per sublayer and rank:

    y_part = x @ W_row.T            GEMM whose epilogue stores row m into the partial slot of rank m // s
    r, n   = reduce_norm(...)       the owner sums the P partials of its rows, adds its residual rows, applies
                                    the next RMSNorm and pushes the normed rows into every rank's buffer
    z      = ag_gemm(W_col)         GEMM whose TMA producer waits until every rank's rows arrived, then streams
                                    the full [M, H] activations from local memory

No NCCL call and no host synchronization runs inside a pass, so the whole cycle is captured in one CUDA graph; the
round parities are device counters. Economize's own tensor parallelism is ``transformers``' ``tp_plan="auto"``
with an NCCL all-reduce after every row-parallel projection (``src/economize/distributed/tp.py:117-138``).
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from .. import ops
from ..errors import CommTimeoutError, ConfigError

__all__ = ["SequenceParallel"]


class SequenceParallel:
    """The buffers and collective kernels of one tensor-parallel group.

    Args:
        tp: The group (its ranks share a node and reach each other over NVLink).
        hidden: Width of the residual stream.
        max_rows: Most tokens one pass carries (larger passes take the NCCL path).
        captures: Block outputs per pass that can be gathered in full for a drafter.
    """

    def __init__(self, tp, hidden: int, max_rows: int = 4096, captures: int = 4) -> None:
        if tp.size > 8:
            raise ConfigError("the fused sequence-parallel collectives support up to 8 ranks")
        self.tp = tp
        self.hidden = hidden
        self.max_rows = max_rows
        self.n_cap = captures
        ext = ops.require()
        self.ext = ext
        nbytes = ext.sp_buffer_bytes(tp.size, tp.rank, hidden, max_rows, captures)
        self.own, handle = ext.symm_alloc(nbytes)
        handles: list = [None] * tp.size
        dist.all_gather_object(handles, handle, group=tp.group)
        self.ptrs = [self.own if r == tp.rank else ext.symm_open(h) for r, h in enumerate(handles)]
        dist.barrier(group=tp.group)

    def _args(self):
        return self.ptrs, self.tp.rank, self.hidden, self.max_rows, self.n_cap

    def fits(self, rows: int) -> bool:
        return 1 <= rows <= self.max_rows

    def shard(self, rows: int) -> tuple[int, int]:
        """``(first row, row count)`` of this rank's token shard of a pass of ``rows`` tokens."""
        per = -(-rows // self.tp.size)
        lo = min(rows, self.tp.rank * per)
        return lo, min(rows, lo + per) - lo

    def reduce_norm(self, resid: torch.Tensor, weight: torch.Tensor, eps: float, rows: int, partials: bool = True,
                    capture: int = -1) -> torch.Tensor:
        """Finish a reduce-scatter round (``partials``) on this rank's residual rows ``resid [n, H]``, RMSNorm, and
        all-gather the normed rows; returns the new residual rows. ``capture >= 0`` also gathers the residual rows
        into that capture slot."""
        lo, _ = self.shard(rows)
        return self.ext.sp_reduce_norm(*self._args(), partials, resid, weight, float(eps), lo, int(capture))

    def ag_linear(self, weight: torch.Tensor, rows: int) -> torch.Tensor:
        """All-gather -> GEMM: ``X @ weight.T`` for the current all-gather round's ``[rows, H]`` activations."""
        return self.ext.sp_linear_ag(*self._args(), rows, weight)

    def ag_linear_parts(self, weight: torch.Tensor, rows: int, lead: tuple[int, ...]) -> torch.Tensor | ops.Partials:
        """:meth:`ag_linear` for a consumer that sums split-K partials (``ops.rope_store``, ``ops.glu``): the
        swap-AB GEMM's :class:`~economize_b200.ops.Partials` shaped ``[*lead, N]`` (the decode path's kernel;
        passes of more than 64 tokens take :meth:`ag_linear`)."""
        if rows > 64:
            return self.ag_linear(weight, rows).reshape(*lead, -1)
        y = self.ext.sp_linear_ag_parts(*self._args(), rows, weight)
        if y.dtype == torch.bfloat16:
            return y.reshape(*lead, -1)
        return ops.Partials(y.reshape(y.shape[0], *lead, y.shape[-1]))

    def rs_linear(self, x: torch.Tensor, weight: torch.Tensor) -> None:
        """GEMM -> reduce-scatter: ``x @ weight.T`` with every output row sent to its owner's partial slot."""
        self.ext.sp_linear_rs(*self._args(), x.reshape(-1, x.shape[-1]), weight)

    def fetch(self, rows: int, like: torch.Tensor) -> torch.Tensor:
        """The current all-gather round's rows ``[rows, H]`` (the round's consumer)."""
        return self.ext.sp_fetch(*self._args(), rows, like)

    def captured(self, slot: int, rows: int, like: torch.Tensor) -> torch.Tensor:
        """The residual rows gathered into ``slot`` this pass (read after the pass's last all-gather round)."""
        return self.ext.sp_capture(*self._args(), slot, rows, like)

    def check(self) -> None:
        """Raise :class:`CommTimeoutError` if a bounded wait of this device gave up since the last check."""
        status = self.ext.status(torch.cuda.current_device())
        if status & 8:
            raise CommTimeoutError(f"a peer's rows did not arrive in time (status {status})")

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's. Every rank calls it (it waits for the others first, so no
        peer still stores into a buffer being freed)."""
        if not self.ptrs:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.tp.group)
        for r, p in enumerate(self.ptrs):
            if r != self.tp.rank:
                self.ext.symm_close(p)
        self.ext.symm_free(self.own)
        self.ptrs = []
