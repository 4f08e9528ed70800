"""The protocol between the engine and a drafting technique.

A drafter keeps its own state on the device (e.g. EAGLE-3's draft KV cache) and is driven by the engine with
fixed-shape tensors, so a whole cycle can be recorded as one CUDA graph:

* :meth:`DraftModel.observe` writes the drafter's state for the columns the exact pass committed and runs the
  root step (the first draft step after the exact token), returning the root's logits over the draft vocabulary.
* :meth:`DraftModel.tree_step` runs one draft step over a frontier of ``W`` nodes (a chain is a frontier of one).

This replaces economize's observe/step/tree_step drafter calls (``src/economize/techniques/_draft_layer/
drafter.py:118-190``) with calls that never synchronize with the host.
"""

from __future__ import annotations

from typing import Protocol, runtime_checkable

import torch

__all__ = ["DraftModel"]


@runtime_checkable
class DraftModel(Protocol):
    #: Block outputs of the target that :meth:`observe` reads (``0`` = embeddings, ``i`` = output of ``i`` blocks).
    capture_layers: tuple[int, ...]
    #: Width of the per-row carry (the fused state of the last committed token), or 0 without one.
    carry_size: int

    def begin(self, batch: int, capacity: int) -> None:
        """Allocate (or reuse) per-generation device state for ``batch`` rows of ``capacity`` positions."""

    def fuse(self, aux: dict[int, torch.Tensor]) -> torch.Tensor:
        """The drafter's per-token source ``[B, C, d]`` from the captured target states ``{layer: [B, C, H]}``."""

    def observe(self, tokens: torch.Tensor, sources: torch.Tensor, kv_len: torch.Tensor, n_valid: torch.Tensor,
                root: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """Process columns ``0..n_valid[b]-1`` of ``tokens [B, C]`` at positions ``kv_len[b] + i`` with source
        ``sources[:, i]``; column ``root[b] = n_valid[b] - 1`` is the root step. Returns the root's logits
        ``[B, V_d]`` (fp32) and its output state ``[B, d]``."""

    def tree_step(self, tokens: torch.Tensor, states: torch.Tensor, positions: torch.Tensor, kv_base: torch.Tensor,
                  n_forwarded: int, q_offset: int, mask: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """One draft step over ``tokens [B, W]`` whose parents' outputs are ``states [B, W, d]``. The frontier
        nodes are forwarded nodes ``q_offset .. q_offset + W - 1`` of a region of ``n_forwarded`` slots starting at
        ``kv_base``; ``mask [B, W]`` holds their ancestor bits within that region. Returns fp32 logits
        ``[B, W, V_d]`` and the frontier's output states ``[B, W, d]``."""

    def to_target(self, draft_ids: torch.Tensor) -> torch.Tensor:
        """Map draft-vocabulary ids to target ids."""
