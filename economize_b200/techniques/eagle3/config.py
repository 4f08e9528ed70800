"""Configuration of EAGLE-3 drafting (fields of economize's ``Eagle3Config``,
``src/economize/techniques/eagle3/config.py:17-58``)."""

from __future__ import annotations

from dataclasses import dataclass
from typing import TYPE_CHECKING, ClassVar

from ...errors import ConfigError
from ...validation import check_choice, check_indices, check_positive
from .._draft_layer.config import DraftLayerConfig

if TYPE_CHECKING:
    from ...models.llama import CausalLM

__all__ = ["EAGLE3_HEADS", "Eagle3Config", "default_aux_layers"]

EAGLE3_HEADS = ("own", "shared")


def default_aux_layers(num_layers: int) -> tuple[int, ...]:
    """The block outputs EAGLE-3 fuses for an ``num_layers``-block model: one after block 2, one halfway and one three
    blocks before the end. A shallow model keeps the distinct ones that exist (``0`` is the embedding output)."""
    wanted = (2, num_layers // 2, num_layers - 3)
    chosen: list[int] = []
    for layer in wanted:
        layer = num_layers if layer > num_layers else (0 if layer < 0 else layer)
        if layer not in chosen:
            chosen.append(layer)
    chosen.sort()
    return tuple(chosen)


@dataclass(frozen=True)
class Eagle3Config(DraftLayerConfig):
    """EAGLE-3 draft head (Li et al., 2025): ``g = fc([h_low; h_mid; h_high])`` of token ``t - 1`` and the token
    embedding of ``t`` feed one decoder layer whose output drafts ``t + 1`` and replaces ``g`` at the next step.

    Attributes:
        aux_layers: Fused block outputs (``None``: ``(2, L // 2, L - 3)``).
        head: ``"own"`` final norm + LM head (initialised from the model's) or ``"shared"`` (the model's).
        draft_vocab: Size of the own head's vocabulary (draft token ``i`` is model token ``i + d2t[i]``).
        norm_before_residual: The attention block's residual is ``norm_h(g)`` instead of ``g``.
    """

    technique: ClassVar[str] = "eagle3"

    aux_layers: tuple[int, ...] | None = None
    head: str = "own"
    draft_vocab: int | None = None
    norm_before_residual: bool = False

    def __post_init__(self) -> None:
        super().__post_init__()
        check_choice("head", self.head, EAGLE3_HEADS)
        if self.draft_vocab is not None:
            if self.head == "shared":
                raise ConfigError("a reduced draft vocabulary belongs to the drafter's own head; with head='shared' "
                                  "leave draft_vocab unset")
            check_positive("draft_vocab", self.draft_vocab)
        if self.aux_layers is None:
            return
        fused = tuple(int(index) for index in self.aux_layers)
        check_indices("aux_layers", fused, allow_empty=False)
        object.__setattr__(self, "aux_layers", fused)

    def layers(self, num_layers: int) -> tuple[int, ...]:
        return self.aux_layers if self.aux_layers is not None else default_aux_layers(num_layers)

    def validate(self, model: CausalLM) -> None:
        c = model.config
        if max(self.layers(c.num_layers)) > c.num_layers:
            raise ConfigError(f"aux_layers {self.layers(c.num_layers)} exceed the model's {c.num_layers} layers")
        if self.draft_vocab is not None and self.draft_vocab > c.vocab_size:
            raise ConfigError(f"draft_vocab {self.draft_vocab} exceeds the model's vocabulary ({c.vocab_size})")
        heads = self.num_heads or c.num_heads
        kv = self.num_kv_heads or (c.num_kv_heads if self.num_heads is None else heads)
        if heads % kv:
            raise ConfigError(f"the draft layer's {heads} heads are not a multiple of its {kv} KV heads")
