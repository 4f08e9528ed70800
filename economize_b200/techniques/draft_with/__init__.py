"""Draft views (``draft_with``; economize ``techniques/draft_with``): a self-speculative drafter that runs the
target with other techniques applied to the draft path only (sparse activations, quantized or pruned weights, an
evicted or compressed KV cache), while the unmodified target verifies. Greedy decoding returns the target's tokens;
rejection sampling keeps its distribution.

The draft path is a :func:`~economize_b200.techniques._self_draft.layer_view` over every layer: its layer
references hold their own attributes, so the listed techniques are attached to the view and leave the target's
layers untouched. For weight techniques the view first gets its own copies of the projection weights, which the
techniques then rewrite (the draft path's quantized or pruned copy is extra memory, as a separate draft copy).
"""

from __future__ import annotations

from collections.abc import Iterable
from dataclasses import dataclass
from typing import Any, ClassVar

import torch
from torch import nn

from ...core.technique import CAPABILITY_ORDER, Capability, TechniqueConfig, register_technique, technique_for
from ...errors import ConfigError
from .._self_draft import SelfDraftTechnique, layer_view

__all__ = ["DraftWith", "DraftWithConfig", "DraftWithTechnique"]

PROJECTIONS = ("wqkv", "wo", "w_gate_up", "w_down")
#: Techniques that cannot run on a draft view: drafters, and transforms that rewrite tensors the view shares with
#: the target (the embedding, norms and head).
_REFUSED = ("rotate", "draft_with", "draft_quant", "frspec")


@dataclass(frozen=True)
class DraftWithConfig(TechniqueConfig):
    """Attributes: ``techniques``: the configurations the draft path runs (at least one, distinct names; a list or
    the JSON entries ``{"technique": name, "config": fields}``)."""

    technique: ClassVar[str] = "draft_with"
    techniques: tuple = ()

    def __post_init__(self) -> None:
        from ...core.serialization import nested_config

        value: Any = self.techniques
        if isinstance(value, (TechniqueConfig, dict)) or not isinstance(value, Iterable):
            raise ConfigError(f"techniques must be a sequence of technique configurations, got {type(value).__name__}")
        configs = [nested_config(v) if isinstance(v, dict) else v for v in value]
        if any(not isinstance(c, TechniqueConfig) for c in configs):
            raise ConfigError("techniques must hold technique configurations")
        if not configs:
            raise ConfigError("draft_with needs at least one technique to apply to the draft path")
        names = [c.technique for c in configs]
        repeated = sorted({n for n in names if names.count(n) > 1})
        if repeated:
            raise ConfigError(f"draft_with lists the technique(s) {repeated} more than once")
        for c in configs:
            cls = technique_for(c)
            if Capability.DRAFTER in cls.capabilities or c.technique in _REFUSED:
                raise ConfigError(f"{c.technique!r} cannot run on a draft view")
        object.__setattr__(self, "techniques", tuple(configs))

    def validate(self, model) -> None:
        for c in self.techniques:
            c.validate(model)

    def to_dict(self) -> dict[str, Any]:
        from ...core.serialization import nested_dict

        return {"techniques": [nested_dict(c) for c in self.techniques]}


def DraftWith(*techniques: TechniqueConfig) -> DraftWithConfig:
    """A drafter that runs the model with ``techniques`` applied, e.g. ``DraftWith(TealConfig(sparsity=0.5))``."""
    return DraftWithConfig(techniques=techniques)


def _rank(config: TechniqueConfig) -> int:
    caps = technique_for(config).capabilities
    return next((i for i, c in enumerate(CAPABILITY_ORDER) if c in caps or c == Capability.NONE), len(CAPABILITY_ORDER))


@register_technique
class DraftWithTechnique(SelfDraftTechnique):
    config_class = DraftWithConfig

    def __init__(self, config: DraftWithConfig, model) -> None:
        super().__init__(config, model)
        view = layer_view(model, list(range(model.config.num_layers)))
        ordered = sorted(config.techniques, key=_rank)
        if any(Capability.WEIGHTS in technique_for(c).capabilities for c in ordered):
            with torch.no_grad():
                for ref in view.layers:
                    target = ref._target[0]
                    for name in PROJECTIONS:
                        w = getattr(target, name)
                        if isinstance(w, torch.Tensor):
                            ref.register_parameter(name, nn.Parameter(w.detach().clone(), requires_grad=False))
        self._view = [view]
        self.inner = nn.ModuleDict({c.technique: technique_for(c)(c, view) for c in ordered})

    def calibrate(self, calibration) -> None:
        super().calibrate(calibration)
        for t in self.inner.values():
            if hasattr(t, "calibrate"):
                t.calibrate(calibration)

    def attach(self) -> None:
        for t in self.inner.values():
            t.attach()

    def detach(self) -> None:
        for t in reversed(list(self.inner.values())):
            t.detach()

    def technique_state(self) -> dict[str, torch.Tensor]:
        return {f"{n}.{k}": v for n, t in self.inner.items() for k, v in t.technique_state().items()}

    def export_state(self) -> dict[str, torch.Tensor]:
        return {f"{n}.{k}": v for n, t in self.inner.items() for k, v in t.export_state().items()}

    def load_technique_state(self, state: dict[str, torch.Tensor]) -> None:
        for n, t in self.inner.items():
            sub = {k[len(n) + 1:]: v for k, v in state.items() if k.startswith(n + ".")}
            if sub:
                t.load_technique_state(sub)
        unknown = sorted(k for k in state if k.split(".", 1)[0] not in self.inner)
        if unknown:
            raise ConfigError(f"draft_with: unexpected tensors {unknown[:5]}")

    def simulation(self):
        return None
