"""ReDrafter (``redrafter``; Cheng et al., 2024; economize ``techniques/redrafter``): a recurrent draft head on the
target's last hidden state. The recurrent state starts from the target state and the target's next token,
``s_0 = tanh(W_h h + W_e e(x_{t+1}))``, advances with every drafted token, ``s_j = tanh(U s_{j-1} + W_e e(d_j))``,
and each step reads out ``MLP([h; s_j])`` through the target's norm and LM head. Beam search maps onto the engine's
dynamic tree (``beam_width`` top-k children per node, ``beam_length`` levels, verified as one tree). Trained with
``step_distill``.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import ClassVar

import torch
import torch.nn.functional as F
from torch import nn

from ...core.technique import TechniqueConfig, register_technique
from ...decoding.config import DecodeConfig
from ...validation import check_choice, check_positive
from .._seq_heads import SequentialHeadTechnique

__all__ = ["RedrafterConfig", "RedrafterTechnique"]


@dataclass(frozen=True)
class RedrafterConfig(TechniqueConfig):
    technique: ClassVar[str] = "redrafter"
    beam_width: int = 8
    beam_length: int = 5
    num_layers: int = 2
    param_dtype: str = "model"

    def __post_init__(self) -> None:
        check_positive("beam_width", self.beam_width)
        check_positive("beam_length", self.beam_length)
        check_positive("num_layers", self.num_layers)
        check_choice("param_dtype", self.param_dtype, ("model", "float32"))


@register_technique
class RedrafterTechnique(SequentialHeadTechnique):
    config_class = RedrafterConfig

    def __init__(self, config: RedrafterConfig, model) -> None:
        super().__init__(config, model)
        h = model.config.hidden_size
        dtype = model.dtype if config.param_dtype == "model" else torch.float32
        self.w_h = nn.Linear(h, h, bias=False)
        self.w_e = nn.Linear(h, h)
        self.u = nn.Linear(h, h, bias=False)
        self.mlp_in = nn.Linear(2 * h, h, bias=False)
        self.mlp = nn.ModuleList(nn.Linear(h, h) for _ in range(config.num_layers))
        with torch.no_grad():
            self.mlp_in.weight.zero_()
            self.mlp_in.weight[:, :h].copy_(torch.eye(h))  # starts as the target's own readout of h
            for b in self.mlp:
                nn.init.zeros_(b.weight)
                nn.init.zeros_(b.bias)
        self.to(device=model.device, dtype=dtype)
        self.hidden = h

    def max_steps(self) -> int:
        return self.config.beam_length

    def depth_of(self, state: torch.Tensor) -> int:
        return 0  # one recurrent cell for every step

    def start(self, h, e):
        dt = self.w_h.weight.dtype
        s = torch.tanh(self.w_h(h.to(dt)) + self.w_e(e.to(dt)))
        return torch.cat([h.to(dt), s], -1)

    def advance(self, state, e, depth):
        h, s = state[..., : self.hidden], state[..., self.hidden:]
        dt = self.u.weight.dtype
        s = torch.tanh(self.u(s.to(dt)) + self.w_e(e.to(dt)))
        return torch.cat([h, s], -1)

    def readout(self, state, depth):
        x = F.linear(state.to(self.mlp_in.weight.dtype), self.mlp_in.weight)
        for b in self.mlp:
            x = x + F.silu(b(x))
        return x

    def default_decoding(self) -> DecodeConfig:
        c = self.config
        return DecodeConfig(cycle_length=c.beam_length + 1, draft_policy="dynamic_tree",
                            draft_policy_options={"depth": c.beam_length, "topk": min(c.beam_width, 10),
                                                  "total_tokens": min(63, c.beam_width * c.beam_length)})
