"""Prompt-lookup decoding (``lookup``): drafts the tokens that followed an earlier occurrence of the context's last
n-gram (Saxena 2023; economize ``techniques/lookup``). The search runs on the device (``csrc/ngram.cu``) over the
engine's token history, so it is part of the captured cycle."""

from __future__ import annotations

from dataclasses import dataclass
from typing import ClassVar

import torch

from ... import ops
from ...core.technique import Capability, Family, Technique, TechniqueConfig, register_technique
from ...decoding.config import DecodeConfig
from ...errors import ConfigError
from ...validation import check_choice, check_positive

__all__ = ["LookupConfig", "LookupDrafter", "LookupTechnique"]


@dataclass(frozen=True)
class LookupConfig(TechniqueConfig):
    """Attributes: ``max_ngram`` / ``min_ngram`` (longest match tried first), ``max_proposal`` drafts per cycle
    (``None``: ``cycle_length - 1``), ``match`` ``"earliest"`` or ``"latest"`` occurrence."""

    technique: ClassVar[str] = "lookup"
    max_ngram: int = 3
    min_ngram: int = 1
    max_proposal: int | None = None
    match: str = "earliest"

    def __post_init__(self) -> None:
        check_positive("max_ngram", self.max_ngram)
        check_positive("min_ngram", self.min_ngram)
        if self.min_ngram > self.max_ngram:
            raise ConfigError("min_ngram exceeds max_ngram")
        if self.max_proposal is not None:
            check_positive("max_proposal", self.max_proposal)
        check_choice("match", self.match, ("earliest", "latest"))


@register_technique
class LookupTechnique(Technique):
    config_class = LookupConfig
    capabilities = Capability.DRAFTER
    family = Family.DRAFTER

    def drafter(self) -> LookupDrafter:
        return LookupDrafter(self.config)

    def default_decoding(self) -> DecodeConfig:
        return DecodeConfig(cycle_length=4)


class LookupDrafter:
    observes = False
    capture_layers: tuple[int, ...] = ()
    carry_size = 0

    def __init__(self, config: LookupConfig) -> None:
        self.config = config
        self.k = 1

    def begin(self, batch: int, capacity: int) -> None:
        pass

    def draft_depth(self, decode: DecodeConfig) -> int:
        self.k = self.config.max_proposal or max(1, decode.cycle_length - 1)
        return self.k

    def draft_nodes(self, decode: DecodeConfig) -> int:
        return self.draft_depth(decode)

    def propose(self, history: torch.Tensor, length: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        c = self.config
        drafts = ops.ngram(history, length, self.k, c.min_ngram, c.max_ngram, c.match == "earliest")
        parents = (torch.arange(self.k, device=history.device) - 1).expand(history.shape[0], self.k).contiguous()
        return drafts, parents

    def to_target(self, ids: torch.Tensor) -> torch.Tensor:
        return ids
