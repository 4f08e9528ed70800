"""EAGLE-1/2 drafting (``eagle``; Li et al., 2024; economize ``techniques/eagle``): one decoder layer on
``x = fc([embed(x_{t+1}); f_t])`` where ``f_t`` is the target's top-layer feature (the residual stream before the
final norm) of the previous token; the layer's output is the predicted next feature, read out by the target's own
final norm and LM head. Features of drafted tokens are the draft's own predictions (EAGLE's feature
autoregression); dynamic trees are EAGLE-2.

Parameter names follow the official EAGLE checkpoints with q/k/v and gate/up fused: ``fc.weight``/``fc.bias``
and the layer's projections and ``post_attention_layernorm`` (the first layer has no input norm).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import ClassVar

import torch
import torch.nn.functional as F
from torch import nn

from ... import ops
from ...core.technique import Capability, Family, Technique, register_technique
from ...decoding.config import DecodeConfig
from ...errors import ConfigError
from ...models.config import ModelConfig
from ...runtime.cache import KVCache, StepBatch
from ...train.objective import OBJECTIVES, Objective, OptimDefaults, teacher_pass
from .._draft_layer.config import DraftLayerConfig
from .._draft_layer.layer import DraftLayer

__all__ = ["EagleConfig", "EagleDrafter", "EagleFeatureLoss", "EagleTechnique"]


@dataclass(frozen=True)
class EagleConfig(DraftLayerConfig):
    """EAGLE-1/2 draft layer; the ``DraftLayerConfig`` fields size it (``None``: the target's)."""

    technique: ClassVar[str] = "eagle"
    fc_bias: bool = True


@register_technique
class EagleTechnique(Technique):
    config_class = EagleConfig
    capabilities = Capability.DRAFTER
    family = Family.DRAFTER
    lossless = True
    objective_name = "eagle_feature"

    def __init__(self, config: EagleConfig, model) -> None:
        super().__init__(config, model)
        c = model.config
        dtype = {"model": model.dtype, "float32": torch.float32, "bfloat16": torch.bfloat16,
                 "float16": torch.float16}[config.param_dtype]
        kw = dict(dtype=dtype, device=model.device)
        h = c.hidden_size
        heads = config.num_heads or c.num_heads
        kv_heads = config.num_kv_heads or (c.num_kv_heads if config.num_heads is None else heads)
        self.eps = config.rms_norm_eps or c.rms_norm_eps
        self.fc = nn.Parameter(torch.empty(h, 2 * h, **kw))
        self.fc_bias = nn.Parameter(torch.zeros(h, **kw)) if config.fc_bias else None
        bias = bool(config.attention_bias) if config.attention_bias is not None else c.attention_bias
        self.layer = DraftLayer(h, h, config.intermediate_size or c.intermediate_size, heads, kv_heads,
                                config.head_dim or c.head_dim, self.eps, bias, dtype, model.device)
        self.layer.set_rope(ModelConfig.from_dict({**c.to_dict(), "rope_theta": config.rope_theta or c.rope_theta}))
        self.reset_parameters()

    @torch.no_grad()
    def reset_parameters(self, seed: int | None = None, std: float = 0.02, identity: bool = False) -> None:
        """N(0, std) matrices; with ``identity`` the layer starts by passing the previous feature through (fc picks
        the feature half, attention and MLP outputs are zero)."""
        gen = None
        if seed is not None:
            gen = torch.Generator(device=self.fc.device)
            gen.manual_seed(seed)
        for p in (self.fc, self.layer.wqkv, self.layer.wo, self.layer.w_gate_up, self.layer.w_down):
            p.copy_(torch.randn(p.shape, generator=gen, device=p.device, dtype=torch.float32) * std)
        if identity:
            h = self.fc.shape[0]
            self.fc.zero_()
            self.fc[:, h:].copy_(torch.eye(h, device=self.fc.device, dtype=self.fc.dtype))
            self.layer.wo.zero_()
            self.layer.w_down.zero_()

    def validate_model(self) -> None:
        if self.model.config.num_layers < 1:
            raise ConfigError("eagle needs a model with layers")

    def default_decoding(self) -> DecodeConfig:
        return DecodeConfig(cycle_length=4)

    def drafter(self) -> EagleDrafter:
        return EagleDrafter(self)


class EagleDrafter:
    """Device drafter of :class:`EagleTechnique` (see :class:`~economize_b200.decoding.drafter.DraftModel`)."""

    def __init__(self, technique: EagleTechnique) -> None:
        self.t = technique
        self.capture_layers = (technique.model.config.num_layers,)  # the pre-norm top-layer feature
        self.carry_size = technique.model.config.hidden_size
        self.cache: KVCache | None = None

    def begin(self, batch: int, capacity: int) -> None:
        layer = self.t.layer
        if self.cache is None or self.cache.batch != batch or self.cache.capacity < capacity:
            self.cache = KVCache(1, batch, layer.kv_heads, capacity, layer.head_dim, layer.wqkv.dtype,
                                 layer.wqkv.device)
        else:
            self.cache.reset()

    def fuse(self, aux: dict[int, torch.Tensor]) -> torch.Tensor:
        return aux[self.capture_layers[0]].to(self.t.fc.dtype)

    def _step(self, tokens: torch.Tensor, features: torch.Tensor, batch: StepBatch):
        t = self.t
        emb = t.model.embed_tokens(tokens).to(t.fc.dtype)
        x = ops.linear(torch.cat([emb, features.to(t.fc.dtype)], -1), t.fc, t.fc_bias)
        mlp, a = t.layer.run(x, x, self.cache, batch)
        model = t.model
        normed, out = ops.rmsnorm(mlp, model.norm.to(a.dtype), model.config.rms_norm_eps, a)
        return ops.linear(normed, model.head_weight).float(), out

    def observe(self, tokens, sources, kv_len, n_valid, root):
        batch, width = tokens.shape
        dev = tokens.device
        pos = (kv_len[:, None] + torch.arange(width, device=dev, dtype=torch.int32)[None]).to(torch.int32)
        logits, out = self._step(tokens, sources, StepBatch(kv_len, n_valid.to(torch.int32), pos.contiguous()))
        rows = torch.arange(batch, device=dev)
        r = root.long()
        return logits[rows, r], out[rows, r]

    def tree_step(self, tokens, states, positions, kv_base, n_forwarded, q_offset, mask):
        batch = tokens.shape[0]
        n_new = torch.full((batch,), n_forwarded, dtype=torch.int32, device=tokens.device)
        sb = StepBatch(kv_base.to(torch.int32), n_new, positions.to(torch.int32), mask, q_offset)
        return self._step(tokens, states, sb)

    def to_target(self, ids: torch.Tensor) -> torch.Tensor:
        return ids


def draft_layer_torch(layer: DraftLayer, x: torch.Tensor, residual: torch.Tensor) -> torch.Tensor:
    """The draft layer in plain PyTorch with causal attention (autograd): returns ``a + mlp``."""
    from ...ops.reference import rmsnorm

    batch, length, _ = x.shape
    heads, kv_heads, hd = layer.heads, layer.kv_heads, layer.head_dim
    cos, sin = layer.rope()
    c, s = cos[:length][None, :, None].to(x.dtype), sin[:length][None, :, None].to(x.dtype)
    q, k, v = F.linear(x, layer.wqkv, layer.bqkv).split([heads * hd, kv_heads * hd, kv_heads * hd], -1)

    def rot(t):
        t = t.reshape(batch, length, -1, hd)
        a, b = t[..., : hd // 2], t[..., hd // 2:]
        return torch.cat([a * c - b * s, b * c + a * s], -1).transpose(1, 2)

    q, k = rot(q), rot(k)
    v = v.reshape(batch, length, kv_heads, hd).transpose(1, 2)
    g = heads // kv_heads
    o = F.scaled_dot_product_attention(q, k.repeat_interleave(g, 1), v.repeat_interleave(g, 1), is_causal=True)
    a = residual + F.linear(o.transpose(1, 2).reshape(batch, length, -1), layer.wo)
    gate, up = F.linear(rmsnorm(a, layer.post_norm, layer.eps)[0], layer.w_gate_up).chunk(2, -1)
    return a + F.linear(F.silu(gate) * up, layer.w_down)


@OBJECTIVES.register("eagle_feature")
class EagleFeatureLoss(Objective):
    """EAGLE-1's objective: smooth-L1 regression of the next top-layer feature plus ``ce_weight`` times the
    cross-entropy of its readout against the target's greedy token (teacher-forced features)."""

    name = "eagle_feature"
    defaults = OptimDefaults(lr=1e-3, warmup_steps=10)

    def __init__(self, model, ce_weight: float = 0.1) -> None:
        super().__init__(model)
        if "eagle" not in model.techniques:
            raise ConfigError("eagle_feature needs an attached eagle technique")
        self.tech = model.techniques["eagle"]
        self.ce_weight = ce_weight

    def parameters(self):
        return [p for p in self.tech.parameters() if p.requires_grad]

    def loss(self, tokens: torch.Tensor):
        from ...ops.reference import rmsnorm

        tech, target = self.tech, self.model.model
        key = target.config.num_layers
        aux, labels = teacher_pass(self.model, tokens, (key,))
        f = aux[key].detach().to(tech.fc.dtype)
        emb = target.embed_tokens(tokens[:, 1:]).to(tech.fc.dtype)
        x = F.linear(torch.cat([emb, f[:, :-1]], -1), tech.fc, tech.fc_bias)
        pred = draft_layer_torch(tech.layer, x, x)
        reg = F.smooth_l1_loss(pred.float(), f[:, 1:].float())
        logits = F.linear(rmsnorm(pred, target.norm.to(pred.dtype), target.config.rms_norm_eps)[0],
                          target.head_weight.to(pred.dtype)).float()
        ce = F.cross_entropy(logits.reshape(-1, logits.shape[-1]), labels[:, 1:].reshape(-1))
        loss = reg + self.ce_weight * ce
        with torch.no_grad():
            acc = (logits.argmax(-1) == labels[:, 1:]).float().mean()
        return loss, {"loss": float(loss.detach()), "reg": float(reg.detach()), "ce": float(ce.detach()),
                      "acc": float(acc)}
