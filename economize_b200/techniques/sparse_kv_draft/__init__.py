"""Self-speculation on a sparse view of the KV cache (``magicdec`` and ``triforce``; economize
``techniques/sparse_kv_draft``): the drafter is the target model itself, attending only to a StreamingLLM-style
subset of the context (``sink`` first tokens plus the ``window`` most recent ones), so at long context a draft
step reads a fraction of the KV bytes while its weights are the target's (MagicDec, Chen et al. 2024). TriForce
(Sun et al. 2024) retrieves chunks instead of a fixed window: ``triforce`` keeps, besides the sinks and the recent
window, the ``chunks`` prompt chunks whose mean key has the largest inner product with the last prompt token's
queries.

The view runs on the engine's kernels with its own KV cache (slot-addressed like the target's) and hides the other
prompt slots with the attention kernel's per-head keep bitmap, set when the view processes the prompt; generated
tokens stay visible (at the long contexts these drafters target they are a small addition to the window).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import ClassVar

import torch

from ...core.technique import TechniqueConfig, register_technique
from ...validation import check_positive
from .._self_draft import SelfDraftTechnique, layer_view
from ..kv_evict import keep_words

__all__ = ["MagicDecConfig", "SparseViewEvictor", "TriForceConfig"]


@dataclass(frozen=True)
class MagicDecConfig(TechniqueConfig):
    technique: ClassVar[str] = "magicdec"
    sink: int = 16
    window: int = 256

    def __post_init__(self) -> None:
        check_positive("window", self.window)


@dataclass(frozen=True)
class TriForceConfig(MagicDecConfig):
    technique: ClassVar[str] = "triforce"
    chunk: int = 64
    chunks: int = 8


class SparseViewEvictor:
    """The draft view's keep policy: sinks + a window that slides with the committed length (+ retrieved chunks)."""

    def __init__(self, config: MagicDecConfig, num_layers: int) -> None:
        self.config = config
        self.num_layers = num_layers
        self.keep: torch.Tensor | None = None
        self.chunk_keep: torch.Tensor | None = None  # [L, B, H_kv, S] retrieved chunks (triforce)

    def keep_for(self, layer: int, k_cache: torch.Tensor, q=None, batch=None) -> torch.Tensor | None:
        return None if self.keep is None or self.keep.shape[3] * 32 != k_cache.shape[2] else self.keep[layer]

    @torch.no_grad()
    def observe_prefill(self, layer, q, k_cache, v_cache, batch) -> None:
        c = self.config
        b, length = q.shape[0], q.shape[1]
        hkv, s = k_cache.shape[1], k_cache.shape[2]
        slots = torch.arange(s, device=q.device)
        lengths = batch.n_new
        keep = (slots[None] < c.sink) | (slots[None] >= lengths[:, None] - c.window)
        keep = keep[:, None].expand(b, hkv, s).clone()
        if isinstance(c, TriForceConfig):
            n_chunks = s // c.chunk
            keys = k_cache.float().reshape(b, hkv, n_chunks, c.chunk, -1).mean(3)  # [B, Hkv, C, D]
            group = q.shape[2] // hkv
            last = q[:, length - 1].float().reshape(b, hkv, group, -1).mean(2)  # [B, Hkv, D]
            score = torch.einsum("bhcd,bhd->bhc", keys, last)
            valid = (torch.arange(n_chunks, device=q.device)[None] * c.chunk) < lengths[:, None]
            score = score.masked_fill(~valid[:, None], float("-inf"))
            top = score.topk(min(c.chunks, n_chunks), -1).indices
            chosen = torch.zeros(b, hkv, n_chunks, dtype=torch.bool, device=q.device).scatter_(-1, top, True)
            keep |= chosen.repeat_interleave(c.chunk, -1) & (slots[None, None] < lengths[:, None, None])
        keep |= slots[None, None] >= lengths[:, None, None]  # generated tokens: decided by the window below
        if self.keep is None or self.keep.shape[1:] != (b, hkv, s // 32):
            self.keep = torch.full((self.num_layers, b, hkv, s // 32), -1, dtype=torch.int32, device=q.device)
        self.keep[layer] = keep_words(keep)


class _SparseViewTechnique(SelfDraftTechnique):
    def view_layers(self) -> list[int]:
        return list(range(self.model.config.num_layers))

    def attach(self) -> None:
        super().attach()
        self._view[0].kv_evictor = SparseViewEvictor(self.config, self.model.config.num_layers)


@register_technique
class MagicDecTechnique(_SparseViewTechnique):
    config_class = MagicDecConfig


@register_technique
class TriForceTechnique(_SparseViewTechnique):
    config_class = TriForceConfig
