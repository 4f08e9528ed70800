"""Hydra drafting (``hydra``; Ankner et al., 2024; economize ``techniques/hydra``): Medusa-like heads where head
``j`` reads the target state ``h_t``, the embedding of the target's next token and the embeddings of the tokens that
heads ``1 .. j - 1`` drafted (sequential dependence), as an MLP of ``num_layers`` residual SiLU blocks over a linear
map of that concatenation, read out through the target's norm and LM head. Trained with ``step_distill``.

With ``prefix_layer=True`` (Hydra++) the heads start from ``P_t`` instead of ``h_t``: the output at ``t`` of one
extra decoder layer with its own attention and KV cache over the target's last hidden states. The drafter runs it
over every committed position once (each cycle's observe step, at the positions of those states), so its cache
holds exactly the committed prefix; in training it runs causally over the teacher-forced sequence. Its attention
and MLP output projections start at zero, so a fresh prefix layer is the identity and heads trained without it keep
working.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import ClassVar

import torch
import torch.nn.functional as F
from torch import nn

from ... import ops
from ...core.technique import TechniqueConfig, register_technique
from ...validation import check_choice, check_positive
from ...runtime.cache import KVCache, StepBatch
from .._draft_layer.layer import DraftLayer
from .._seq_heads import SequentialHeadDrafter, SequentialHeadTechnique

__all__ = ["HydraConfig", "HydraTechnique"]


@dataclass(frozen=True)
class HydraConfig(TechniqueConfig):
    """``num_heads``: draft steps; ``num_layers``: residual blocks per head; ``param_dtype``: ``"model"`` or
    ``"float32"``; ``prefix_layer``: Hydra++'s prefix attention layer (the target's attention geometry;
    ``prefix_intermediate_size``: its MLP width, default the target's)."""

    technique: ClassVar[str] = "hydra"
    num_heads: int = 4
    num_layers: int = 1
    param_dtype: str = "model"
    prefix_layer: bool = False
    prefix_intermediate_size: int | None = None

    def __post_init__(self) -> None:
        check_positive("num_heads", self.num_heads)
        check_positive("num_layers", self.num_layers)
        check_choice("param_dtype", self.param_dtype, ("model", "float32"))
        if self.prefix_intermediate_size is not None:
            check_positive("prefix_intermediate_size", self.prefix_intermediate_size)


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
        self.prefix = None
        if config.prefix_layer:
            c = model.config
            self.prefix = DraftLayer(h, h, config.prefix_intermediate_size or c.intermediate_size, c.num_heads,
                                     c.num_kv_heads, c.head_dim, c.rms_norm_eps, False, model.dtype, model.device)
            self.prefix.set_rope(c)
            gen = torch.Generator().manual_seed(0)
            with torch.no_grad():
                for p in (self.prefix.wqkv, self.prefix.w_gate_up):
                    p.copy_(torch.randn(p.shape, generator=gen).mul_(0.02).to(p))
                self.prefix.wo.zero_()  # the residual passes through: P_t = h_t until trained
                self.prefix.w_down.zero_()

    def source_states(self, h: torch.Tensor) -> torch.Tensor:
        if self.prefix is None:
            return h
        from ..eagle import draft_layer_torch

        x = h.to(self.prefix.wqkv.dtype)
        return draft_layer_torch(self.prefix, x, x)

    def drafter(self):
        return HydraPrefixDrafter(self) if self.prefix is not None else super().drafter()

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


class HydraPrefixDrafter(SequentialHeadDrafter):
    """The sequential-head drafter with Hydra++'s prefix layer: observe runs the layer over the newly committed
    target states (columns ``1 ..`` of the observed block hold the states of positions ``kv_len ..``; column 0 is
    the previous cycle's last state, already in the cache) and starts the heads from its output at the root."""

    def __init__(self, tech) -> None:
        super().__init__(tech)
        self.cache: KVCache | None = None

    def begin(self, batch: int, capacity: int) -> None:
        layer = self.tech.prefix
        if self.cache is None or self.cache.batch != batch or self.cache.capacity < capacity:
            self.cache = KVCache(1, batch, layer.kv_heads, capacity, layer.head_dim, layer.wqkv.dtype,
                                 layer.wqkv.device)
        else:
            self.cache.reset()

    def observe(self, tokens, sources, kv_len, n_valid, root):
        tech = self.tech
        layer = tech.prefix
        batch, width = tokens.shape
        dev = tokens.device
        x = sources[:, 1:].to(layer.wqkv.dtype).contiguous()
        pos = (kv_len[:, None] + torch.arange(width - 1, device=dev, dtype=torch.int32)[None]).to(torch.int32)
        mlp, a = layer.run(x, x, self.cache, StepBatch(kv_len.to(torch.int32), (n_valid - 1).to(torch.int32),
                                                        pos.contiguous()))
        if isinstance(mlp, ops.Partials):
            mlp = mlp.sum()
        p = a + mlp
        rows = torch.arange(batch, device=dev)
        r = root.long()
        h = p[rows, r - 1]
        state = tech.start(h, tech.embed(tokens[rows, r]))
        if self.root_ext is None or self.root_ext.shape != state.shape:
            self.root_ext = torch.zeros_like(state)
        self.root_ext.copy_(state)
        return tech.readout_logits(state, 0), h.to(tech.model.dtype)
