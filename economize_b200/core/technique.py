"""The technique contract: configuration, capabilities, attach order and the technique registry.

Mirrors economize's technique model (``src/economize/core/technique.py:47-372``): every technique is a
``TechniqueConfig`` dataclass (registered under ``config.technique``) plus a :class:`Technique` module that holds the
added parameters. Techniques attach in ``CAPABILITY_ORDER`` whatever order the user lists them in.
"""

from __future__ import annotations

import enum
from dataclasses import asdict, dataclass, fields
from typing import TYPE_CHECKING, Any, ClassVar

import torch
from torch import nn

from ..errors import ConfigError, IncompatibleTechniquesError
from ..registry import Registry
from ..validation import known_fields

if TYPE_CHECKING:
    from ..decoding.config import DecodeConfig
    from ..decoding.drafter import DraftModel
    from ..models.llama import CausalLM

__all__ = ["CAPABILITY_ORDER", "TECHNIQUES", "Capability", "Family", "Simulation", "Technique", "TechniqueConfig",
           "register_technique", "technique_for"]


class Capability(enum.Flag):
    """What a technique changes."""

    NONE = 0
    WEIGHTS = enum.auto()      # rewrites the model's weights (quantization, pruning, low rank)
    ACTIVATIONS = enum.auto()  # hooks on activations per token (activation sparsity)
    KV_CACHE = enum.auto()     # compresses or evicts the KV cache
    DEPTH = enum.auto()        # skips layers per token
    DRAFTER = enum.auto()      # proposes tokens the exact model verifies


#: Attach order: weight transforms first, the drafter last (it reads the transformed model).
CAPABILITY_ORDER = (Capability.WEIGHTS, Capability.ACTIVATIONS, Capability.KV_CACHE, Capability.DEPTH,
                    Capability.DRAFTER, Capability.NONE)


class Family(enum.Enum):
    """Techniques of one family exclude each other (two drafters, two weight quantizers, ...)."""

    DRAFTER = "drafter"
    QUANTIZATION = "quantization"
    DRAFT_COMPRESSION = "draft_compression"  # compresses the drafter's own weights (never the target's)
    PRUNING = "pruning"
    KV_COMPRESSION = "kv_compression"
    SPARSITY = "sparsity"
    DEPTH = "depth"
    OTHER = "other"


@dataclass(frozen=True)
class Simulation:
    """A saving a technique's current path does not realize (its outputs are exact)."""

    saving: str
    reason: str


@dataclass(frozen=True)
class TechniqueConfig:
    """Base of every technique configuration; subclasses set ``technique`` (the registry name)."""

    technique: ClassVar[str] = ""

    def to_dict(self) -> dict[str, Any]:
        out = {}
        for f in fields(self):
            v = getattr(self, f.name)
            out[f.name] = list(v) if isinstance(v, tuple) else v
        return out

    @classmethod
    def from_dict(cls, data: dict[str, Any]) -> TechniqueConfig:
        return cls(**known_fields(cls.__name__, data, {f.name for f in fields(cls)}))

    def validate(self, model: CausalLM) -> None:
        """Raise :class:`ConfigError` when this configuration does not fit ``model``."""


class Technique(nn.Module):
    """A technique attached to a model: holds its parameters and hooks into the engine.

    Subclasses set ``config_class``, ``capabilities``, ``family`` and ``lossless``, build their parameters in
    ``__init__(config, model)``, and override the hooks they need.
    """

    config_class: ClassVar[type[TechniqueConfig]] = TechniqueConfig
    capabilities: ClassVar[Capability] = Capability.NONE
    family: ClassVar[Family] = Family.OTHER
    lossless: ClassVar[bool] = True
    graph_safe: ClassVar[bool] = True

    def __init__(self, config: TechniqueConfig, model: CausalLM) -> None:
        super().__init__()
        config.validate(model)
        self.config = config
        self._model_ref = [model]  # not a submodule: the model's weights are not the technique's

    @property
    def name(self) -> str:
        return self.config.technique

    @property
    def model(self) -> CausalLM:
        return self._model_ref[0]

    def attach(self) -> None:
        """Hook the technique into the model (weight techniques rewrite weights here)."""

    def detach(self) -> None:
        """Undo :meth:`attach` where possible."""

    def inplace_targets(self) -> list[torch.Tensor]:
        """Tensors of the model that :meth:`attach` changes in place (rather than replacing them), so that a failed
        ``apply`` can restore their contents. Weight techniques that write into existing tensors list them."""
        return []

    def drafter(self) -> DraftModel | None:
        return None

    def default_decoding(self) -> DecodeConfig | None:
        return None

    def simulation(self) -> Simulation | None:
        return None

    def conflicts(self, other: Technique) -> str | None:
        """A reason why ``other`` cannot be attached with this technique, or ``None``."""
        if self.family == other.family and self.family in (Family.DRAFTER, Family.QUANTIZATION):
            return f"{self.name} and {other.name} are both {self.family.value} techniques"
        return None

    def technique_state(self) -> dict[str, torch.Tensor]:
        return {k: v.detach() for k, v in self.state_dict().items()}

    def export_state(self) -> dict[str, torch.Tensor]:
        """Tensors under economize's names (what checkpoints store); subclasses with fused layouts convert."""
        return self.technique_state()

    def load_technique_state(self, state: dict[str, torch.Tensor]) -> None:
        missing, unexpected = self.load_state_dict(state, strict=False)
        if unexpected:
            raise ConfigError(f"{self.name}: unexpected tensors {sorted(unexpected)[:5]}")
        if missing:
            raise ConfigError(f"{self.name}: missing tensors {sorted(missing)[:5]}")


TECHNIQUES: Registry[type[Technique]] = Registry("technique", "economize_b200.techniques")


def register_technique(cls: type[Technique]) -> type[Technique]:
    """Class decorator: register a technique under its config's ``technique`` name."""
    name = cls.config_class.technique
    if not name:
        raise ConfigError(f"{cls.__name__}.config_class has no technique name")
    TECHNIQUES.register(name, cls)
    return cls


def technique_for(config: TechniqueConfig) -> type[Technique]:
    if not isinstance(config, TechniqueConfig):
        raise ConfigError(f"expected a technique configuration, got {type(config).__name__}")
    return TECHNIQUES.get(config.technique)


def check_compatible(techniques: list[Technique]) -> None:
    names = [t.name for t in techniques]
    if len(set(names)) != len(names):
        raise IncompatibleTechniquesError(f"a technique is applied twice: {names}")
    drafters = [t.name for t in techniques if Capability.DRAFTER in t.capabilities]
    if len(drafters) > 1:
        raise IncompatibleTechniquesError(f"more than one drafting technique: {drafters}")
    for i, a in enumerate(techniques):
        for b in techniques[i + 1:]:
            reason = a.conflicts(b) or b.conflicts(a)
            if reason:
                raise IncompatibleTechniquesError(reason)
