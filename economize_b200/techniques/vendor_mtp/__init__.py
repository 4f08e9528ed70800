"""Multi-token-prediction modules as drafters (``vendor_mtp``; economize ``techniques/vendor_mtp``: the MTP modules
that DeepSeek-V3, GLM-4.5, MiMo, Qwen3-Next and Qwen3.5 checkpoints ship, and new ones in their layouts).

A module (DeepSeek-V3, arXiv 2412.19437, section 2.2) reads the state ``h`` of the previous position and the
embedding of the current token, mixes them as ``fc([enorm(embed(x)); hnorm(h)])`` (MiMo: ``[hnorm(h);
enorm(embed(x))]``), runs one pre-norm decoder block with its own KV cache, applies its own final norm and the
model's LM head. The first draft step reads the target's last hidden state (after the model's final norm by
default, as vLLM passes it; ``target_state="raw"``: the last block's output); later steps read the module's own
output, before its norm (``recycle="raw"``, DeepSeek-V3 / GLM-4.5) or after it (``"normed"``, MiMo / Qwen). Some
families zero the embedding of the token at position 0. The layout of each family lives in
:data:`~economize_b200.techniques.vendor_mtp.families.MTP_FAMILIES`; checkpoints that ship modules load through
:mod:`.formats` (``economize_b200.read_checkpoint(model_dir)`` then ``attach``).

Draft steps run on the engine's kernels (fused norms, the tcgen05 GEMMs and tree attention); the module drafts
like EAGLE-1 (state autoregression), chains and dynamic trees alike.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import ClassVar

import torch
import torch.nn.functional as F
from torch import nn

from ... import ops
from ...core.technique import register_technique
from ...errors import ConfigError
from ...runtime.cache import StepBatch
from ...train.objective import OBJECTIVES
from ..eagle import EagleConfig, EagleDrafter, EagleFeatureLoss, EagleTechnique
from .families import CONCAT_ORDERS, DEFAULT_FAMILY, MTP_FAMILIES, RECYCLE, MTPFamily, MTPLayout, family_for
from .formats import VendorMTPFormat, mtp_settings, state_from_vendor, state_to_vendor

__all__ = ["MTP_FAMILIES", "MTPFamily", "MTPLayout", "VendorMTPConfig", "VendorMTPFormat", "VendorMTPTechnique",
           "mtp_settings", "state_from_vendor", "state_to_vendor"]


@dataclass(frozen=True)
class VendorMTPConfig(EagleConfig):
    """An MTP module in a registered family's layout.

    Attributes:
        family: A registered family (``None``: the family of the target's ``model_type``, else DeepSeek-V3's).
        num_modules: Modules to draft with; this engine drafts with one (every released family ships one).
        concat_order, zero_first_embedding, recycle: Overrides of the family's layout.
        target_state: What the first draft step reads: ``"normed"`` (the model's final norm applied) or ``"raw"``.
    """

    technique: ClassVar[str] = "vendor_mtp"
    family: str | None = None
    num_modules: int = 1
    concat_order: str | None = None
    zero_first_embedding: bool | None = None
    recycle: str | None = None
    target_state: str = "normed"
    fc_bias: bool = False

    def __post_init__(self) -> None:
        super().__post_init__()
        if self.family is not None and self.family not in MTP_FAMILIES:
            raise ConfigError(f"unknown MTP family {self.family!r}; registered: {MTP_FAMILIES.names()}")
        if self.num_modules != 1:
            raise ConfigError(f"num_modules={self.num_modules}: this engine drafts with one MTP module")
        if self.concat_order is not None and self.concat_order not in CONCAT_ORDERS:
            raise ConfigError(f"concat_order must be one of {CONCAT_ORDERS}")
        if self.recycle is not None and self.recycle not in RECYCLE:
            raise ConfigError(f"recycle must be one of {RECYCLE}")
        if self.target_state not in ("normed", "raw"):
            raise ConfigError("target_state must be 'normed' or 'raw'")

    def resolve_family(self, model_type: str) -> str:
        return self.family or family_for(model_type) or DEFAULT_FAMILY

    def layout(self, model_type: str) -> MTPLayout:
        base = MTP_FAMILIES.get(self.resolve_family(model_type)).layout
        return MTPLayout(self.concat_order or base.concat_order,
                         base.zero_first_embedding if self.zero_first_embedding is None else self.zero_first_embedding,
                         self.recycle or base.recycle)


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
        # the module's own final norm (DeepSeek-V3's shared_head.norm), a copy of the model's to start from
        self.norm = nn.Parameter(model.norm.detach().to(**kw).clone())
        self.family = config.resolve_family(model.config.model_type)
        self.layout = config.layout(model.config.model_type)

    def drafter(self) -> MTPDrafter:
        return MTPDrafter(self)

    def mix(self, emb: torch.Tensor, state: torch.Tensor, positions: torch.Tensor | None) -> torch.Tensor:
        """``fc`` of the normed embedding and state in the layout's order (``positions``: zero the embedding at
        position 0 when the layout says so)."""
        if self.layout.zero_first_embedding and positions is not None:
            emb = emb * (positions != 0).to(emb.dtype)[..., None]
        e, _ = ops.rmsnorm(emb, self.enorm, self.eps)
        h, _ = ops.rmsnorm(state, self.hnorm, self.eps)
        pair = [e, h] if self.layout.concat_order == "emb_hidden" else [h, e]
        return ops.linear(torch.cat(pair, -1), self.fc, self.fc_bias)

    def target_state(self, feature: torch.Tensor) -> torch.Tensor:
        """The first draft step's state from the target's top-layer feature (the residual stream before the norm)."""
        if self.config.target_state == "raw":
            return feature
        model = self.model
        return ops.rmsnorm(feature, model.norm.to(feature.dtype), model.config.rms_norm_eps)[0]

    def vendor_state(self, num_layers: int | None = None) -> dict[str, torch.Tensor]:
        """This module under the family's checkpoint names (``num_layers``: the target's, by default)."""
        c = self.model.config
        layer = self.layer
        return state_to_vendor([self.export_state()], self.family, num_layers or c.num_layers,
                               (layer.heads, layer.kv_heads, layer.head_dim))


class MTPDrafter(EagleDrafter):
    def fuse(self, aux: dict[int, torch.Tensor]) -> torch.Tensor:
        return self.t.target_state(aux[self.capture_layers[0]].to(self.t.fc.dtype))

    def _step(self, tokens: torch.Tensor, states: torch.Tensor, batch: StepBatch):
        t = self.t
        emb = t.model.embed_tokens(tokens).to(t.fc.dtype)
        x = t.mix(emb, states.to(t.fc.dtype), batch.positions)
        xn, _ = ops.rmsnorm(x, t.input_norm, t.eps)
        mlp, a = t.layer.run(xn, x, self.cache, batch)
        normed, raw = ops.rmsnorm(mlp, t.norm.to(a.dtype), t.eps, a)
        logits = ops.linear(normed, t.model.head_weight).float()
        return logits, (normed if t.layout.recycle == "normed" else raw)


def mtp_torch(tech: VendorMTPTechnique, emb: torch.Tensor, state: torch.Tensor, positions: torch.Tensor
              ) -> tuple[torch.Tensor, torch.Tensor]:
    """The module in plain PyTorch (autograd): ``(normed, raw)`` outputs for embeddings and states ``[B, S, H]``."""
    from ...ops.reference import rmsnorm
    from ..eagle import draft_layer_torch

    if tech.layout.zero_first_embedding:
        emb = emb * (positions != 0).to(emb.dtype)[..., None]
    e, h = rmsnorm(emb, tech.enorm, tech.eps)[0], rmsnorm(state, tech.hnorm, tech.eps)[0]
    x = F.linear(torch.cat([e, h] if tech.layout.concat_order == "emb_hidden" else [h, e], -1), tech.fc, tech.fc_bias)
    raw = draft_layer_torch(tech.layer, rmsnorm(x, tech.input_norm, tech.eps)[0], x)
    return rmsnorm(raw, tech.norm, tech.eps)[0], raw


@OBJECTIVES.register("mtp_feature")
class MTPFeatureLoss(EagleFeatureLoss):
    """Teacher-forced MTP objective: cross-entropy of the module's readout against the target's greedy token two
    positions ahead, plus ``reg_weight`` times the smooth-L1 distance of the recycled state to the target's state
    at the next position (both in the layout's representation)."""

    name = "mtp_feature"

    def __init__(self, model, reg_weight: float = 1.0) -> None:
        if "vendor_mtp" not in model.techniques:
            raise ConfigError("mtp_feature needs an attached vendor_mtp technique")
        self.model = model
        self.tech = model.techniques["vendor_mtp"]
        self.reg_weight = reg_weight

    def loss(self, tokens: torch.Tensor):
        from ...ops.reference import rmsnorm
        from ...train.objective import teacher_pass

        tech, target = self.tech, self.model.model
        key = target.config.num_layers
        aux, labels = teacher_pass(self.model, tokens, (key,))
        raw = aux[key].detach().to(tech.fc.dtype)
        normed = rmsnorm(raw, target.norm.to(raw.dtype), target.config.rms_norm_eps)[0]
        first = normed if tech.config.target_state == "normed" else raw
        recycled = normed if tech.layout.recycle == "normed" else raw
        positions = torch.arange(1, tokens.shape[1], device=tokens.device)[None].expand(tokens.shape[0], -1)
        emb = target.embed_tokens(tokens[:, 1:]).to(tech.fc.dtype)
        out_normed, out_raw = mtp_torch(tech, emb, first[:, :-1], positions)
        pred = out_normed if tech.layout.recycle == "normed" else out_raw
        reg = F.smooth_l1_loss(pred.float(), recycled[:, 1:].float())
        logits = F.linear(out_normed, target.head_weight.to(out_normed.dtype)).float()
        ce = F.cross_entropy(logits.reshape(-1, logits.shape[-1]), labels[:, 1:].reshape(-1))
        loss = ce + self.reg_weight * reg
        return loss, {"loss": float(loss.detach()), "reg": float(reg.detach()), "ce": float(ce.detach())}
