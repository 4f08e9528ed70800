"""Hadamard rotation of the residual stream (``rotate``; QuaRot, Ashkboos et al. 2024; economize
``techniques/rotate``, ``HADAMARD_KERNELS``).

RMSNorm weights are folded into the projections that read the norm's output, after which the network is invariant
to any orthogonal ``Q`` applied to the residual stream: ``embed' = embed Q``, readers ``W' = W Q`` (QKV, gate/up,
LM head), writers ``W' = Q^T W`` (o, down). With ``Q`` a randomized Hadamard matrix (``H diag(+-1) / sqrt(n)``)
outlier features are spread over all channels, which makes the rotated weights and activations far easier to
quantize (apply ``rotate`` before ``quant``: both are weight transforms and attach in the given order). The
transform is exact in real arithmetic; it is computed in fp32 and rounded once to the model dtype.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import ClassVar

import torch
from torch import nn

from ...core.technique import Capability, Family, Technique, TechniqueConfig, register_technique
from ...errors import ConfigError

__all__ = ["RotateConfig", "RotateTechnique", "random_hadamard"]


def _hadamard(n: int) -> torch.Tensor:
    h = torch.ones(1, 1)
    while h.shape[0] < n:
        h = torch.cat([torch.cat([h, h], 1), torch.cat([h, -h], 1)], 0)
    return h


def random_hadamard(n: int, seed: int = 0) -> torch.Tensor:
    """An ``n x n`` orthogonal matrix: Sylvester Hadamard with random signs when ``n`` is a power of two, else a
    random orthogonal matrix (QR of a Gaussian)."""
    g = torch.Generator().manual_seed(seed)
    if n & (n - 1) == 0:
        signs = torch.randint(0, 2, (n,), generator=g).float() * 2 - 1
        return _hadamard(n) * signs[None, :] / n ** 0.5
    q, r = torch.linalg.qr(torch.randn(n, n, generator=g, dtype=torch.float64))
    return (q * torch.sign(torch.diagonal(r))[None, :]).float()


@dataclass(frozen=True)
class RotateConfig(TechniqueConfig):
    technique: ClassVar[str] = "rotate"
    seed: int = 0


@register_technique
class RotateTechnique(Technique):
    config_class = RotateConfig
    capabilities = Capability.WEIGHTS
    family = Family.OTHER
    lossless = True  # exact up to the final rounding

    def __init__(self, config: RotateConfig, model) -> None:
        super().__init__(config, model)
        if model.config.is_moe:
            raise ConfigError("rotate supports dense models")
        self.applied = False

    @torch.no_grad()
    def attach(self) -> None:
        if self.applied:
            return
        m = self.model
        if m.tp is not None and m.tp.size > 1:
            raise ConfigError("rotate before sharding the model")
        dev, dt = m.device, m.dtype
        q = random_hadamard(m.config.hidden_size, self.config.seed).to(dev)
        if m.lm_head is None:  # untie: the head is folded and rotated, the embedding only rotated
            m.lm_head = nn.Parameter(m.embed.detach().clone())
            m.config.tie_word_embeddings = False

        def set_(p: nn.Parameter, value: torch.Tensor) -> None:
            p.data = value.to(dt).contiguous()

        for layer in m.layers:
            set_(layer.wqkv, (layer.wqkv.float() * layer.attn_norm.float()[None]) @ q)
            set_(layer.w_gate_up, (layer.w_gate_up.float() * layer.mlp_norm.float()[None]) @ q)
            set_(layer.wo, q.t() @ layer.wo.float())
            set_(layer.w_down, q.t() @ layer.w_down.float())
            layer.attn_norm.data.fill_(1.0)
            layer.mlp_norm.data.fill_(1.0)
        set_(m.lm_head, (m.lm_head.float() * m.norm.float()[None]) @ q)
        m.norm.data.fill_(1.0)
        set_(m.embed, m.embed.float() @ q)
        self.applied = True

    def technique_state(self) -> dict[str, torch.Tensor]:
        return {}

    def load_technique_state(self, state: dict[str, torch.Tensor]) -> None:
        if state:
            raise ConfigError("rotate stores no tensors: it is recomputed from its seed")
