"""Decoding phases: which kind of forward pass is running (economize ``runtime/phase.py``).

The engine marks every pass it runs: ``"prefill"`` (the exact pass over the prompt), ``"refresh"`` (a later exact
pass that verifies drafts), ``"decode"`` (a later exact pass without a drafter, one token per row) and ``"draft"``
(drafter steps). Techniques that act per phase (activation sparsity) read :func:`current_phase`; outside the engine
it is ``None``. CUDA graphs are captured inside the same markers, so a captured graph holds the path of its phase.
On CUDA every phase is also an NVTX range (``economize:<phase>``) for timeline profilers.
"""

from __future__ import annotations

from collections.abc import Iterator
from contextlib import contextmanager
from contextvars import ContextVar

from ..errors import ConfigError

__all__ = ["PHASES", "current_phase", "phase"]

PHASES = ("prefill", "refresh", "decode", "draft")

_PHASE: ContextVar[str | None] = ContextVar("economize_b200_phase", default=None)


def current_phase() -> str | None:
    """The phase of the pass in progress, or ``None`` outside the engine."""
    return _PHASE.get()


@contextmanager
def phase(name: str | None) -> Iterator[None]:
    """Mark the passes inside the block as phase ``name``."""
    if name is not None and name not in PHASES:
        raise ConfigError(f"unknown phase {name!r}; expected one of {PHASES}")
    token = _PHASE.set(name)
    marked = name is not None and _nvtx_enabled()
    if marked:  # an NVTX range per phase, for timeline profilers
        import torch

        torch.cuda.nvtx.range_push(f"economize:{name}")
    try:
        yield
    finally:
        if marked:
            import torch

            torch.cuda.nvtx.range_pop()
        _PHASE.reset(token)


def _nvtx_enabled() -> bool:
    import torch

    return torch.cuda.is_available()
