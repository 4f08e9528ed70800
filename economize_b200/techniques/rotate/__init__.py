"""Hadamard rotations that make weights and activations easier to quantize (``rotate``; QuaRot, Ashkboos et al.
2024; economize ``techniques/rotate/config.py:20-53``, ``hadamard.py``).

Three rotations, each exact in real arithmetic (computed in fp32, rounded once to the model dtype):

* residual (QuaRot's R1): RMSNorm weights are folded into the projections that read the norm's output, after which
  the network is invariant to any orthogonal ``Q`` applied to the residual stream: ``embed' = embed Q``, readers
  ``W' = W Q`` (QKV, gate/up, LM head), writers ``W' = Q^T W`` (o, down). ``Q`` is a randomized Hadamard matrix
  (``H diag(+-1) / sqrt(n)``). Dense pre-norm models only.
* values (R2): per KV head an orthogonal ``R`` (``head_dim`` square, randomized Hadamard) rotates the rows of the
  value projection (``W_v' = R^T W_v``, bias ``b_v R``) and the matching columns of ``wo`` for every query head of the
  group (``W_o' = W_o R``): every head's attention output is rotated by ``R`` and ``wo`` undoes it.
* online (R4 on ``mlp.down_proj``): ``w_down' = w_down H`` with ``H`` the block-diagonal normalized Sylvester matrix
  of the largest power-of-two block that divides the MLP width (at most ``block``, at most 8192), and the down
  projection's input is rotated at run time. On CUDA the rotation runs inside the gated-activation kernel that
  produces that input (``csrc/elementwise.cu:hadamard_kernel``), so the rotated activation is written once.

With rotated weights, outlier features are spread over all channels; apply ``rotate`` before ``quant`` (both are
weight transforms and attach in the given order).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import ClassVar

import torch
from torch import nn

from ...core.technique import Capability, Family, Technique, TechniqueConfig, register_technique
from ...errors import ConfigError
from ...ops import reference as ops_reference

__all__ = ["MAX_ONLINE_BLOCK", "ONLINE_MAPS", "RotateConfig", "RotateTechnique", "online_block", "random_hadamard"]


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
    """``online``: linear maps whose inputs are rotated online (``("mlp.down_proj",)`` or ``()``); ``values``: the
    value rotation; ``residual``: the residual-stream rotation (dense pre-norm models); ``layers``: 1-indexed layers
    of the value and online rotations (empty: all); ``block``: largest online Hadamard block, a power of two (0: the
    largest dividing the width, capped at 8192); ``seed``: seed of the random signs (``None``: plain Sylvester)."""

    technique: ClassVar[str] = "rotate"
    online: tuple[str, ...] = ("mlp.down_proj",)
    values: bool = True
    residual: bool = True
    layers: tuple[int, ...] = ()
    block: int = 0
    seed: int | None = 0

    def __post_init__(self) -> None:
        online = tuple(self.online)
        unknown = [name for name in online if name not in ONLINE_MAPS]
        if unknown:
            raise ConfigError(f"online rotations are built for {ONLINE_MAPS}, got {unknown}")
        object.__setattr__(self, "online", online)
        object.__setattr__(self, "layers", tuple(int(i) for i in self.layers))
        if any(i < 1 for i in self.layers):
            raise ConfigError(f"layers are 1-indexed, got {self.layers}")
        if self.block < 0 or (self.block and (self.block & (self.block - 1) or self.block < 8)):
            raise ConfigError(f"block must be 0 or a power of two >= 8, got {self.block}")
        if self.seed is not None and (isinstance(self.seed, bool) or not isinstance(self.seed, int)):
            raise ConfigError(f"seed must be an int or None, got {self.seed!r}")
        if not (online or self.values or self.residual):
            raise ConfigError("rotate with online=(), values=False and residual=False rotates nothing")


#: linear maps whose input can be rotated online (the down projection of dense gated MLPs)
ONLINE_MAPS = ("mlp.down_proj",)
#: largest online block the CUDA kernel transforms (its fp32 block sits in 32 KB of shared memory)
MAX_ONLINE_BLOCK = 8192


def online_block(width: int, cap: int = 0) -> int:
    """The block of the block-diagonal Hadamard rotation of a ``width``-wide input: the largest power of two that
    divides ``width``, at most ``cap`` (0: no cap of its own) and at most :data:`MAX_ONLINE_BLOCK`."""
    block = width & -width
    return min(block, cap or block, MAX_ONLINE_BLOCK)


def _sylvester_signed(n: int, seed: int | None) -> torch.Tensor:
    """The ``n x n`` normalized Sylvester matrix, columns multiplied by random signs of ``seed`` (``None``: none)."""
    h = _hadamard(n) / n ** 0.5
    if seed is None:
        return h
    g = torch.Generator().manual_seed(seed)
    return h * (torch.randint(0, 2, (n,), generator=g).float() * 2 - 1)[None, :]


@register_technique
class RotateTechnique(Technique):
    config_class = RotateConfig
    capabilities = Capability.WEIGHTS
    family = Family.OTHER
    lossless = True  # exact up to the final rounding

    def __init__(self, config: RotateConfig, model) -> None:
        super().__init__(config, model)
        if model.config.is_moe and config.residual:
            raise ConfigError("the residual rotation supports dense models (rotate with residual=False)")
        self.applied = False

    def _layer_ids(self) -> list[int]:
        n = len(self.model.layers)
        if any(i > n for i in self.config.layers):
            raise ConfigError(f"layers {self.config.layers} exceed the model's {n} layers")
        return [i - 1 for i in self.config.layers] if self.config.layers else list(range(n))

    @torch.no_grad()
    def attach(self) -> None:
        if self.applied:
            return
        m, c = self.model, self.config
        if m.tp is not None and m.tp.size > 1:
            raise ConfigError("rotate before sharding the model")
        dev, dt = m.device, m.dtype
        ids = self._layer_ids()
        if c.online:
            for i in ids:
                if getattr(m.layers[i], "mlp_rule", None) is not None:
                    raise ConfigError(f"layer {i + 1} runs an activation-sparse MLP, whose kernels read the down "
                                      "projection's input unrotated (rotate with online=() or apply rotate first)")

        def set_(p: nn.Parameter, value: torch.Tensor) -> None:
            p.data = value.to(dt).contiguous()

        if c.residual:
            n = m.config.hidden_size
            plain = c.seed is None and n & (n - 1) == 0
            q = (_sylvester_signed(n, None) if plain else random_hadamard(n, c.seed or 0)).to(dev)
            if m.lm_head is None:  # untie: the head is folded and rotated, the embedding only rotated
                m.lm_head = nn.Parameter(m.embed.detach().clone())
                m.config.tie_word_embeddings = False
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
        if c.values:
            self._rotate_values(ids, set_)
        if c.online:
            for i in ids:
                layer = m.layers[i]
                if layer.router is not None or layer.down_hadamard:
                    continue  # MoE experts keep unrotated inputs; a layer is rotated once
                block = online_block(layer.w_down.shape[1], c.block)
                if block < 8:
                    continue  # a width without a power-of-two factor of 8 keeps its input unrotated
                set_(layer.w_down, ops_reference.hadamard(layer.w_down.float(), block))
                layer.down_hadamard = block
        self.applied = True

    def _rotate_values(self, ids: list[int], set_) -> None:
        mc = self.model.config
        d, hq, hkv = mc.head_dim, mc.num_heads, mc.num_kv_heads
        if d & (d - 1):
            raise ConfigError(f"the value rotation needs a power-of-two head_dim, got {d}")
        r = _sylvester_signed(d, self.config.seed).to(self.model.device)
        for i in ids:
            layer = self.model.layers[i]
            w = layer.wqkv.float()
            v0 = mc.q_size + mc.kv_size
            v = w[v0:v0 + mc.kv_size].reshape(hkv, d, -1)
            w[v0:v0 + mc.kv_size] = torch.einsum("ji,hjk->hik", r, v).reshape(mc.kv_size, -1)
            set_(layer.wqkv, w)
            if layer.bqkv is not None:
                b = layer.bqkv.float()
                b[v0:v0 + mc.kv_size] = (b[v0:v0 + mc.kv_size].reshape(hkv, d) @ r).reshape(-1)
                set_(layer.bqkv, b)
            wo = layer.wo.float().reshape(-1, hq, d)
            set_(layer.wo, (wo @ r).reshape(-1, hq * d))

    def technique_state(self) -> dict[str, torch.Tensor]:
        return {}

    def load_technique_state(self, state: dict[str, torch.Tensor]) -> None:
        if state:
            raise ConfigError("rotate stores no tensors: it is recomputed from its seed")
