"""Kangaroo self-drafting (``kangaroo``; Liu et al., 2024; economize ``techniques/kangaroo``): a shallow sub-network
(the target's first ``exit_layer`` blocks) followed by a small trained adapter block, read out by the target's LM
head. The adapter is a full decoder block owned by the technique, initialised as a copy of the target's block
``exit_layer`` (so an untrained adapter already drafts like a one-block-deeper exit) and trained with
``train.fit`` under the ``kangaroo_distill`` objective (KL to the target's next-token distribution)."""

from __future__ import annotations

import copy
from dataclasses import dataclass
from typing import ClassVar

import torch
from torch import nn

from ...core.technique import TechniqueConfig, register_technique
from ...errors import ConfigError
from .._self_draft import SelfDraftTechnique

__all__ = ["KangarooConfig", "KangarooTechnique"]


@dataclass(frozen=True)
class KangarooConfig(TechniqueConfig):
    technique: ClassVar[str] = "kangaroo"
    exit_layer: int = 2
    adapter_layers: int = 1

    def __post_init__(self) -> None:
        if self.exit_layer < 1 or self.adapter_layers < 1:
            raise ConfigError("exit_layer and adapter_layers must be >= 1")

    def validate(self, model) -> None:
        if self.exit_layer + self.adapter_layers > model.config.num_layers:
            raise ConfigError("exit_layer + adapter_layers exceeds the model's depth")


@register_technique
class KangarooTechnique(SelfDraftTechnique):
    config_class = KangarooConfig
    objective_name = "kangaroo_distill"

    def __init__(self, config: KangarooConfig, model) -> None:
        super().__init__(config, model)
        with torch.no_grad():
            self.adapter = nn.ModuleList(copy.deepcopy(model.layers[config.exit_layer + i])
                                         for i in range(config.adapter_layers))

    def view_layers(self) -> list[int]:
        return list(range(self.config.exit_layer))

    def extra_layers(self) -> list[nn.Module]:
        return list(self.adapter)
