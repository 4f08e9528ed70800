"""Running ranges of decoder layers (economize ``runtime/runner.py``: ``LayerRunner.run / forward / replay``).

The engine's executor (:class:`~economize_b200.models.llama.CausalLM`) already runs any contiguous layer range on
given residual-stream inputs (``forward_step(layers=, hidden=)``); :class:`LayerRunner` is the public face of that
for drafters and tools: a range of layers (1-indexed, inclusive) on a batch's slot cache, with ``overrides`` that
substitute callables for some layers (trainable copies, skipped layers), captures of block outputs, the exact pass,
logits, and a replay that rebuilds the cache over committed tokens.
"""

from __future__ import annotations

from collections.abc import Callable, Mapping
from dataclasses import dataclass, field

import torch

from ..errors import ConfigError
from .cache import KVCache, StepBatch

__all__ = ["ExactPass", "LayerCall", "LayerRunner"]

#: A stand-in for decoder layer ``i``: ``(hidden [B, T, H], batch, cache) -> hidden``, the residual stream in and out.
LayerCall = Callable[[torch.Tensor, StepBatch, KVCache], torch.Tensor]


@dataclass
class ExactPass:
    """One pass of the unmodified model: the final-normed hidden states, the captured block outputs (``i``: the
    stream entering block ``i + 1``, ``0`` the embeddings, ``-1`` the final-normed states) and the pass's batch."""

    final: torch.Tensor
    hidden: dict[int, torch.Tensor] = field(default_factory=dict)
    batch: StepBatch | None = None


class LayerRunner:
    """Runs the decoder layers of an engine model on its slot cache."""

    def __init__(self, model) -> None:
        self.model = model

    @property
    def num_layers(self) -> int:
        return self.model.config.num_layers

    def new_cache(self, batch: int, capacity: int) -> KVCache:
        return self.model.new_cache(batch, capacity)

    def embed(self, tokens: torch.Tensor) -> torch.Tensor:
        return self.model.embed_tokens(tokens)

    def run(self, hidden: torch.Tensor, batch: StepBatch, cache: KVCache, first: int, last: int,
            overrides: Mapping[int, LayerCall] | None = None, capture: tuple[int, ...] = ()
            ) -> tuple[torch.Tensor, dict[int, torch.Tensor]]:
        """Layers ``first .. last`` (1-indexed, inclusive) on the residual stream ``hidden [B, T, H]``; returns the
        stream after layer ``last`` (not normed) and the requested block outputs (keys as in :class:`ExactPass`).
        Layer ``i`` in ``overrides`` runs the given callable instead of the model's layer."""
        if not 1 <= first <= last + 1 <= self.num_layers + 1:
            raise ConfigError(f"layer range {first}..{last} is outside 1..{self.num_layers}")
        overrides = dict(overrides or {})
        stray = [i for i in overrides if not first <= i <= last]
        if stray:
            raise ConfigError(f"overrides for layers {sorted(stray)} outside the range {first}..{last}")
        aux: dict[int, torch.Tensor] = {}
        h = hidden
        dummy = torch.zeros(hidden.shape[:2], dtype=torch.int64, device=hidden.device)
        i = first
        while i <= last:
            if (i - 1) in capture:
                aux[i - 1] = h
            if i in overrides:
                h = overrides[i](h, batch, cache)
                i += 1
                continue
            j = i
            while j + 1 <= last and (j + 1) not in overrides and j not in capture:
                j += 1
            # layers i .. j of the model (0-based i - 1 .. j - 1): the stream after them is the pre-norm residual
            _, got = self.model.forward_step(dummy, batch, cache, capture=(-2,), layers=range(i - 1, j), hidden=h)
            h = got[-2]
            i = j + 1
        if last in capture:
            aux[last] = h
        return h, aux

    def forward(self, tokens: torch.Tensor, batch: StepBatch, cache: KVCache,
                capture: tuple[int, ...] = ()) -> ExactPass:
        """The exact pass over ``tokens [B, T]`` (every layer, the model's own weights)."""
        final, hidden = self.model.forward_step(tokens, batch, cache, capture)
        return ExactPass(final, hidden, batch)

    def logits(self, final: torch.Tensor) -> torch.Tensor:
        return self.model.logits(final)

    def replay(self, tokens: torch.Tensor, cache: KVCache, lengths: torch.Tensor) -> ExactPass:
        """Rebuild ``cache`` from slot 0 over committed ``tokens [B, P]`` (``lengths`` valid per row), e.g. after
        the cache was reset or a technique changed the layers that wrote it."""
        batch = StepBatch.prefill(lengths.to(torch.int32), tokens.shape[1])
        return self.forward(tokens, batch, cache)
