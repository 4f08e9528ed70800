"""Frequency-ranked speculative sampling (``frspec``; Zhao et al., 2025; economize ``techniques/frspec``): the
drafter's LM head is restricted to the ``vocab_size`` most frequent tokens of a corpus (the calibration tokens), so
the draft head reads ``vocab_size / V`` of the full head's bytes. Wraps an attached ``eagle3`` drafter: its head
rows, ``d2t`` and ``t2d`` are rebuilt for the frequent subset. Lossless (the target verifies every token)."""

from __future__ import annotations

from dataclasses import dataclass
from typing import ClassVar

import torch
from torch import nn

from ...core.technique import Capability, Family, Technique, TechniqueConfig, register_technique
from ...errors import ConfigError
from ...validation import check_positive

__all__ = ["FRSpecConfig", "FRSpecTechnique", "frequent_tokens"]


@dataclass(frozen=True)
class FRSpecConfig(TechniqueConfig):
    technique: ClassVar[str] = "frspec"
    vocab_size: int = 32768

    def __post_init__(self) -> None:
        check_positive("vocab_size", self.vocab_size)


def frequent_tokens(tokens: torch.Tensor, vocab: int, k: int) -> torch.Tensor:
    """The ``k`` most frequent ids of ``tokens`` (unseen ids fill up in id order)."""
    counts = torch.bincount(tokens.reshape(-1).long().cpu(), minlength=vocab)[:vocab].float()
    order = torch.argsort(-counts, stable=True)
    return order[:k].sort().values


@register_technique
class FRSpecTechnique(Technique):
    config_class = FRSpecConfig
    capabilities = Capability.NONE
    family = Family.OTHER
    lossless = True

    def __init__(self, config: FRSpecConfig, model) -> None:
        super().__init__(config, model)
        self._calibration = None
        self.register_buffer("token_ids", torch.zeros(0, dtype=torch.int64, device=model.device))

    def calibrate(self, calibration) -> None:
        self._calibration = calibration

    def after_drafter(self, technique: nn.Module) -> None:
        """Restrict ``technique``'s head (called once the drafter is attached)."""
        while hasattr(technique, "wrapped_drafter"):  # a hybrid's fallback
            technique = technique.wrapped_drafter
        if technique.name != "eagle3":
            raise ConfigError(f"frspec restricts an eagle3 draft head, not {technique.name}")
        if self.token_ids.numel() == 0:
            cal = self._calibration
            if cal is None:
                raise ConfigError("frspec needs calibration tokens to rank the vocabulary (apply(..., calibration=))")
            toks = cal if isinstance(cal, torch.Tensor) else torch.cat([torch.as_tensor(c).reshape(-1) for c in cal])
            vocab = self.model.config.vocab_size
            self.token_ids = frequent_tokens(toks, vocab, min(self.config.vocab_size, vocab)).to(self.model.device)
        restrict_eagle3_head(technique, self.token_ids)


@torch.no_grad()
def restrict_eagle3_head(tech, ids: torch.Tensor) -> None:
    ids = ids.to(tech.d2t.device).long().sort().values
    full_rows = tech.model.head_weight.detach()[ids].to(tech.lm_head.dtype) if tech.shared_head else None
    if tech.shared_head:
        tech.shared_head = False
        tech.norm = nn.Parameter(tech.model.norm.detach().clone().to(full_rows.dtype))
        tech.lm_head = nn.Parameter(full_rows)
    else:
        # keep the trained rows of ids the head already had; others start from the target's head
        old_ids = torch.arange(tech.draft_vocab, device=ids.device) + tech.d2t
        rows = tech.model.head_weight.detach()[ids].to(tech.lm_head.dtype).clone()
        pos = torch.searchsorted(old_ids, ids).clamp(max=old_ids.numel() - 1)
        hit = old_ids[pos] == ids
        rows[hit] = tech.lm_head.detach()[pos[hit]]
        tech.lm_head = nn.Parameter(rows)
    tech.draft_vocab = ids.numel()
    tech.d2t = ids - torch.arange(ids.numel(), device=ids.device)
    t2d = torch.zeros_like(tech.t2d)
    t2d[ids] = True
    tech.t2d = t2d
