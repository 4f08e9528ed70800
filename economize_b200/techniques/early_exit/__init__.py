"""Early-exit self-drafting (``early_exit``): the draft is the target's first ``exit_layer`` blocks read out by the
target's final norm and LM head (LayerSkip, Elhoushi et al. 2024; economize ``techniques/early_exit``, whose
optional LoRA/full readout adaptation is trained with the ``layerskip`` objective). The exit's KV cache is the
drafter's own, so verification never reuses draft keys."""

from __future__ import annotations

from dataclasses import dataclass
from typing import ClassVar

from ...core.technique import TechniqueConfig, register_technique
from ...errors import ConfigError
from .._self_draft import SelfDraftTechnique

__all__ = ["EarlyExitConfig", "EarlyExitTechnique"]


@dataclass(frozen=True)
class EarlyExitConfig(TechniqueConfig):
    """``exit_layer``: number of leading blocks the draft runs (``None``: half the depth)."""

    technique: ClassVar[str] = "early_exit"
    exit_layer: int | None = None

    def __post_init__(self) -> None:
        if self.exit_layer is not None and self.exit_layer < 1:
            raise ConfigError("exit_layer must be >= 1")

    def validate(self, model) -> None:
        if self.exit_layer is not None and self.exit_layer >= model.config.num_layers:
            raise ConfigError(f"exit_layer {self.exit_layer} must be below the model's {model.config.num_layers} "
                              "layers")


@register_technique
class EarlyExitTechnique(SelfDraftTechnique):
    config_class = EarlyExitConfig

    def view_layers(self) -> list[int]:
        k = self.config.exit_layer or max(1, self.model.config.num_layers // 2)
        return list(range(k))
