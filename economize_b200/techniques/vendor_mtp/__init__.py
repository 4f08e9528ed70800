"""Multi-token-prediction heads as drafters (``vendor_mtp``; economize ``techniques/vendor_mtp``, whose
``MTP_FAMILIES`` read the MTP modules shipped with DeepSeek-V3, GLM-4.5, MiMo and Qwen3.5 checkpoints).

The DeepSeek-V3 MTP module (Liu et al., 2024): ``h' = Block(W_eh [RMSNorm_e(embed(t+1)); RMSNorm_h(h_t)])`` with a
full pre-norm decoder block, read out by the model's shared final norm and LM head; ``h_t`` is the model's top-layer
feature (before the final norm) and, at later draft steps, the module's own output. It drafts like EAGLE-1 (feature
autoregression) on the engine's kernels. Parameters: ``enorm``, ``hnorm``, ``eh_proj`` (``fc``), the block's
``input_norm`` and projections; the vendor checkpoint names map onto them in :data:`MTP_FAMILIES`.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import ClassVar

import torch
from torch import nn

from ... import ops
from ...core.technique import register_technique
from ...runtime.cache import StepBatch
from ...train.objective import OBJECTIVES
from ..eagle import EagleConfig, EagleDrafter, EagleFeatureLoss, EagleTechnique

__all__ = ["MTP_FAMILIES", "VendorMTPConfig", "VendorMTPTechnique"]

#: vendor module names of the MTP block (relative to the MTP layer prefix) -> this technique's parameters
MTP_FAMILIES = {
    "deepseek_v3": {"enorm.weight": "enorm", "hnorm.weight": "hnorm", "eh_proj.weight": "fc",
                    "input_layernorm.weight": "input_norm", "post_attention_layernorm.weight": "layer.post_norm",
                    "self_attn.o_proj.weight": "layer.wo", "mlp.down_proj.weight": "layer.w_down"},
}


@dataclass(frozen=True)
class VendorMTPConfig(EagleConfig):
    technique: ClassVar[str] = "vendor_mtp"
    family: str = "deepseek_v3"
    fc_bias: bool = False


@register_technique
class VendorMTPTechnique(EagleTechnique):
    config_class = VendorMTPConfig
    objective_name = "mtp_feature"

    def __init__(self, config: VendorMTPConfig, model) -> None:
        super().__init__(config, model)
        h = model.config.hidden_size
        kw = dict(dtype=self.fc.dtype, device=model.device)
        self.enorm = nn.Parameter(torch.ones(h, **kw))
        self.hnorm = nn.Parameter(torch.ones(h, **kw))
        self.input_norm = nn.Parameter(torch.ones(h, **kw))

    def drafter(self) -> MTPDrafter:
        return MTPDrafter(self)

    def fused_input(self, emb: torch.Tensor, h: torch.Tensor) -> torch.Tensor:
        e, _ = ops.rmsnorm(emb, self.enorm, self.eps)
        g, _ = ops.rmsnorm(h, self.hnorm, self.eps)
        return ops.linear(torch.cat([e, g], -1), self.fc, self.fc_bias)


class MTPDrafter(EagleDrafter):
    def _step(self, tokens: torch.Tensor, features: torch.Tensor, batch: StepBatch):
        t = self.t
        emb = t.model.embed_tokens(tokens).to(t.fc.dtype)
        x = t.fused_input(emb, features.to(t.fc.dtype))
        xn, _ = ops.rmsnorm(x, t.input_norm, t.eps)
        mlp, a = t.layer.run(xn, x, self.cache, batch)
        model = t.model
        normed, out = ops.rmsnorm(mlp, model.norm.to(a.dtype), model.config.rms_norm_eps, a)
        return ops.linear(normed, model.head_weight).float(), out


@OBJECTIVES.register("mtp_feature")
class MTPFeatureLoss(EagleFeatureLoss):
    """Next-feature regression plus readout cross-entropy for an MTP head (teacher-forced)."""

    name = "mtp_feature"

    def __init__(self, model, ce_weight: float = 0.1) -> None:
        from ...errors import ConfigError

        if "vendor_mtp" not in model.techniques:
            raise ConfigError("mtp_feature needs an attached vendor_mtp technique")
        self.model = model
        self.tech = model.techniques["vendor_mtp"]
        self.ce_weight = ce_weight

    def loss(self, tokens: torch.Tensor):
        import torch.nn.functional as F

        from ...ops.reference import rmsnorm
        from ...train.objective import teacher_pass
        from ..eagle import draft_layer_torch

        tech, target = self.tech, self.model.model
        key = target.config.num_layers
        aux, labels = teacher_pass(self.model, tokens, (key,))
        f = aux[key].detach().to(tech.fc.dtype)
        emb = target.embed_tokens(tokens[:, 1:]).to(tech.fc.dtype)
        x = F.linear(torch.cat([rmsnorm(emb, tech.enorm, tech.eps)[0], rmsnorm(f[:, :-1], tech.hnorm, tech.eps)[0]],
                               -1), tech.fc, tech.fc_bias)
        pred = draft_layer_torch(tech.layer, rmsnorm(x, tech.input_norm, tech.eps)[0], x)
        reg = F.smooth_l1_loss(pred.float(), f[:, 1:].float())
        logits = F.linear(rmsnorm(pred, target.norm.to(pred.dtype), target.config.rms_norm_eps)[0],
                          target.head_weight.to(pred.dtype)).float()
        ce = F.cross_entropy(logits.reshape(-1, logits.shape[-1]), labels[:, 1:].reshape(-1))
        loss = reg + self.ce_weight * ce
        return loss, {"loss": float(loss.detach()), "reg": float(reg.detach()), "ce": float(ce.detach())}
