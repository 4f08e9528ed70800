"""A draft model on another device (``placed_draft_model``; economize ``techniques/placed_draft``,
``drafter.py:23-80``): the draft LM runs on its own GPU with its own KV cache; every draft call moves its inputs
there (``non_blocking`` peer copies) and the logits back, so the draft GPU's weight streaming does not compete
with the target's. Cycles run without CUDA graphs (a graph belongs to one device)."""

from __future__ import annotations

from dataclasses import dataclass
from typing import ClassVar

import torch

from ...core.technique import register_technique
from ...decoding.config import DecodeConfig
from ...errors import ConfigError
from ..draft_model import DraftLMDrafter, DraftModelConfig, DraftModelTechnique, install_view, load_draft

__all__ = ["PlacedDraftModelConfig", "PlacedDraftModelTechnique", "PlacedDrafter"]


@dataclass(frozen=True)
class PlacedDraftModelConfig(DraftModelConfig):
    """``device``: where the draft model runs (e.g. ``"cuda:1"``)."""

    technique: ClassVar[str] = "placed_draft_model"
    device: str = "cuda:1"


class PlacedDrafter(DraftLMDrafter):
    graph_safe = False

    def __init__(self, draft, target_hidden: int, home: torch.device) -> None:
        super().__init__(draft, target_hidden)
        self.home = home
        self.there = draft.device

    def _to(self, *ts):
        return tuple(t.to(self.there, non_blocking=True) if isinstance(t, torch.Tensor) else t for t in ts)

    def fuse(self, aux):
        states = aux[-1]
        return torch.zeros(*states.shape[:2], 1, dtype=self.draft.dtype, device=self.home)

    def observe(self, tokens, sources, kv_len, n_valid, root):
        tokens, kv_len, n_valid, root = self._to(tokens, kv_len, n_valid, root)
        logits, _ = super().observe(tokens, None, kv_len, n_valid, root)
        state = torch.zeros(tokens.shape[0], self.target_hidden, dtype=self.draft.dtype, device=self.home)
        return logits.to(self.home, non_blocking=True), state

    def tree_step(self, tokens, states, positions, kv_base, n_forwarded, q_offset, mask):
        tokens, positions, kv_base, mask = self._to(tokens, positions, kv_base, mask)
        logits, _ = super().tree_step(tokens, None, positions, kv_base, n_forwarded, q_offset, mask)
        return logits.to(self.home, non_blocking=True), states


@register_technique
class PlacedDraftModelTechnique(DraftModelTechnique):
    config_class = PlacedDraftModelConfig

    def __init__(self, config: PlacedDraftModelConfig, model) -> None:
        super(DraftModelTechnique, self).__init__(config, model)
        device = torch.device(config.device)
        if device.type == "cuda" and device.index is None:  # "cuda": the current device
            device = torch.device("cuda", torch.cuda.current_device() if torch.cuda.is_available() else 0)
        if device.type == "cuda" and (not torch.cuda.is_available() or device.index >= torch.cuda.device_count()):
            raise ConfigError(f"placed_draft_model: device {config.device} is not available")
        self._draft = [load_draft(config, model).to(device)]
        install_view(self.draft, config)

    def drafter(self) -> PlacedDrafter:
        return PlacedDrafter(self.draft, self.model.config.hidden_size, self.model.device)

    def default_decoding(self) -> DecodeConfig:
        return DecodeConfig(cycle_length=5)
