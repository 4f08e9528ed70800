"""Hydra drafting (``hydra``; Ankner et al., 2024; economize ``techniques/hydra``): Medusa-like heads where head
``j`` reads the target state ``h_t``, the embedding of the target's next token and the embeddings of the tokens that
heads ``1 .. j - 1`` drafted (sequential dependence), as an MLP of ``num_layers`` residual SiLU blocks over a linear
map of that concatenation, read out through the target's norm and LM head. Trained with ``step_distill``.

Not built: Hydra++'s prefix attention layer (``prefix_layer=True`` raises a ConfigError).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import ClassVar

import torch
import torch.nn.functional as F
from torch import nn

from ... import ops
from ...core.technique import TechniqueConfig, register_technique
from ...errors import ConfigError
from ...validation import check_choice, check_positive
from .._seq_heads import SequentialHeadTechnique

__all__ = ["HydraConfig", "HydraTechnique"]


@dataclass(frozen=True)
class HydraConfig(TechniqueConfig):
    """``num_heads``: draft steps; ``num_layers``: residual blocks per head; ``param_dtype``: ``"model"`` or
    ``"float32"``; ``prefix_layer``: Hydra++'s prefix attention (not built)."""

    technique: ClassVar[str] = "hydra"
    num_heads: int = 4
    num_layers: int = 1
    param_dtype: str = "model"
    prefix_layer: bool = False

    def __post_init__(self) -> None:
        check_positive("num_heads", self.num_heads)
        check_positive("num_layers", self.num_layers)
        check_choice("param_dtype", self.param_dtype, ("model", "float32"))
        if self.prefix_layer:
            raise ConfigError("hydra's prefix attention layer (Hydra++) is not built in this engine; use "
                              "prefix_layer=False")


class HydraHead(nn.Module):
    def __init__(self, inputs: int, hidden: int, layers: int) -> None:
        super().__init__()
        self.inp = nn.Linear(inputs * hidden, hidden, bias=False)
        with torch.no_grad():  # starts as the identity on h_t (a Medusa head with zero blocks)
            self.inp.weight.zero_()
            self.inp.weight[:, :hidden].copy_(torch.eye(hidden))
        self.blocks = nn.ModuleList(nn.Linear(hidden, hidden) for _ in range(layers))
        for b in self.blocks:
            nn.init.zeros_(b.weight)
            nn.init.zeros_(b.bias)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = F.linear(x, self.inp.weight)
        for b in self.blocks:
            x = x + F.silu(b(x))
        return x


@register_technique
class HydraTechnique(SequentialHeadTechnique):
    config_class = HydraConfig

    def __init__(self, config: HydraConfig, model) -> None:
        super().__init__(config, model)
        h = model.config.hidden_size
        dtype = model.dtype if config.param_dtype == "model" else torch.float32
        self.heads = nn.ModuleList(HydraHead(j + 2, h, config.num_layers) for j in range(config.num_heads)
                                   ).to(device=model.device, dtype=dtype)
        self.hidden = h

    def max_steps(self) -> int:
        return self.config.num_heads

    def depth_of(self, state: torch.Tensor) -> int:
        return state.shape[-1] // self.hidden - 2

    def start(self, h: torch.Tensor, e: torch.Tensor) -> torch.Tensor:
        return torch.cat([h.to(e.dtype), e], -1)

    def advance(self, state: torch.Tensor, e: torch.Tensor, depth: int) -> torch.Tensor:
        return torch.cat([state, e.to(state.dtype)], -1)

    def readout(self, state: torch.Tensor, depth: int) -> torch.Tensor:
        head = self.heads[min(depth, len(self.heads) - 1)]
        return head(state.to(head.inp.weight.dtype))
