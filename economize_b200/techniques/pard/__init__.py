"""PARD (``pard``; An et al., 2025; economize ``techniques/pard``): a draft LM that proposes ``k`` tokens in one
forward pass. After the committed tokens (the catch-up) the drafter appends ``k - 1`` mask tokens in the same call:
the logits at the last real token give the first draft and the logits at the ``i``-th mask the draft ``i + 1``. The
mask positions are scratch in the draft LM's cache: the next cycle's catch-up overwrites them. The target verifies
(lossless).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import ClassVar

import torch

from ...core.technique import register_technique
from ...decoding.config import DecodeConfig
from ...errors import ConfigError
from ...runtime.cache import StepBatch
from ..draft_model import DraftLMDrafter, DraftModelConfig, DraftModelTechnique

__all__ = ["PardConfig", "PardDrafter", "PardTechnique"]


@dataclass(frozen=True)
class PardConfig(DraftModelConfig):
    """``mask_token_id``: the draft LM's mask token (``None``: its vocabulary's last id); ``max_drafts``: tokens
    proposed per call."""

    technique: ClassVar[str] = "pard"
    mask_token_id: int | None = None
    max_drafts: int = 8

    def __post_init__(self) -> None:
        super().__post_init__()
        if self.max_drafts < 1:
            raise ConfigError("max_drafts must be positive")


class PardDrafter(DraftLMDrafter):
    def __init__(self, draft, target_hidden: int, mask_id: int, k: int) -> None:
        super().__init__(draft, target_hidden)
        self.mask_id = mask_id
        self.k = k
        self.stash: torch.Tensor | None = None
        self._step = 0

    def draft_depth(self, decode: DecodeConfig) -> int:
        self.k = min(self.k, max(1, decode.cycle_length - 1))
        return self.k

    def draft_nodes(self, decode: DecodeConfig) -> int:
        return self.draft_depth(decode)

    def begin(self, batch: int, capacity: int) -> None:
        super().begin(batch, capacity + self.k)  # room for the mask positions past the committed tokens
        v = self.draft.config.vocab_size
        if self.stash is None or self.stash.shape[0] != batch or self.stash.shape[1] != self.k:
            self.stash = torch.zeros(batch, self.k, v, dtype=torch.float32, device=self.draft.device)

    def observe(self, tokens, sources, kv_len, n_valid, root):
        batch, width = tokens.shape
        dev = tokens.device
        k = self.k
        ext = torch.cat([tokens, torch.full((batch, k - 1), self.mask_id, dtype=tokens.dtype, device=dev)], 1)
        cols = torch.arange(width + k - 1, device=dev)
        offs = cols[None] - root.long()[:, None]  # masks right after each row's root column
        ext = torch.where((offs >= 1) & (offs < k), torch.full_like(ext, self.mask_id), ext)
        n_ext = (n_valid + k - 1).to(torch.int32)
        pos = (kv_len[:, None] + cols[None]).to(torch.int32)
        first, self._prompt_pass = getattr(self, "_prompt_pass", False), False
        hidden, _ = self.draft.forward_step(ext, StepBatch(kv_len, n_ext, pos.contiguous(), is_prefill=first),
                                            self.cache)
        idx = (root.long()[:, None] + torch.arange(k, device=dev)[None])  # root, then the k - 1 masks
        picked = hidden.gather(1, idx[..., None].expand(batch, k, hidden.shape[-1]))
        self.stash.copy_(self.draft.logits(picked).float())
        self._step = 0
        return self.stash[:, 0], torch.zeros(batch, self.target_hidden, dtype=self.draft.dtype, device=dev)

    def tree_step(self, tokens, states, positions, kv_base, n_forwarded, q_offset, mask):
        self._step = min(self._step + 1, self.k - 1)
        return self.stash[:, self._step][:, None].expand(-1, tokens.shape[1], -1), states


@register_technique
class PardTechnique(DraftModelTechnique):
    config_class = PardConfig

    def drafter(self) -> PardDrafter:
        mask = self.config.mask_token_id
        if mask is None:
            mask = self.draft.config.vocab_size - 1
        return PardDrafter(self.draft, self.model.config.hidden_size, int(mask), self.config.max_drafts)

    def default_decoding(self) -> DecodeConfig:
        return DecodeConfig(cycle_length=self.config.max_drafts + 1)
