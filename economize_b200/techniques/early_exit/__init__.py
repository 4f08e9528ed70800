"""Early-exit self-drafting (``early_exit``): the draft is the target's first ``exit_layer`` blocks read out by the
target's final norm and LM head (LayerSkip, Elhoushi et al. 2024; economize ``techniques/early_exit``, whose
optional LoRA/full readout adaptation is trained with the ``layerskip`` objective). The exit's KV cache is the
drafter's own, so verification never reuses draft keys."""

from __future__ import annotations

from dataclasses import dataclass
from typing import ClassVar

import torch
from torch import nn

from ...core.technique import TechniqueConfig, register_technique
from ...errors import ConfigError
from ...ops.lora import LoRAWeight
from ...ops.quant import install
from .._self_draft import SelfDraftTechnique

__all__ = ["EarlyExitConfig", "EarlyExitTechnique"]


@dataclass(frozen=True)
class EarlyExitConfig(TechniqueConfig):
    """``exit_layer``: number of leading blocks the draft runs (``None``: half the depth); ``adaptation``: the exit's
    readout, ``"none"`` (the target's final norm and head), ``"lora"`` (a low-rank update of the head, ``lora_rank``
    / ``lora_alpha``) or ``"full"`` (trainable copies of the final norm and head); trained by ``layerskip``."""

    technique: ClassVar[str] = "early_exit"
    exit_layer: int | None = None
    adaptation: str = "none"
    lora_rank: int = 16
    lora_alpha: float = 16.0

    def __post_init__(self) -> None:
        if self.exit_layer is not None and self.exit_layer < 1:
            raise ConfigError("exit_layer must be >= 1")
        if self.adaptation not in ("none", "lora", "full"):
            raise ConfigError(f"adaptation must be 'none', 'lora' or 'full', got {self.adaptation!r}")
        if self.lora_rank < 1:
            raise ConfigError("lora_rank must be positive")

    def validate(self, model) -> None:
        if self.exit_layer is not None and self.exit_layer >= model.config.num_layers:
            raise ConfigError(f"exit_layer {self.exit_layer} must be below the model's {model.config.num_layers} "
                              "layers")


@register_technique
class EarlyExitTechnique(SelfDraftTechnique):
    """With an adaptation, the readout parameters are the technique's state (``norm`` and ``head`` for ``"full"``,
    ``head_lora.a`` / ``head_lora.b`` for ``"lora"``)."""

    config_class = EarlyExitConfig
    objective_name = "layerskip"

    def __init__(self, config: EarlyExitConfig, model) -> None:
        super().__init__(config, model)
        if config.adaptation == "full":
            head = model.head_weight
            self.norm = nn.Parameter(model.norm.detach().clone())
            self.head = nn.Parameter(head.detach().clone() if isinstance(head, torch.Tensor) else head.dequantize())
        elif config.adaptation == "lora":
            self.head_lora = LoRAWeight(model.head_weight, config.lora_rank, config.lora_alpha)

    def lora_targets(self) -> dict:
        """The low-rank adapters by Hugging Face module name (``adaptation="lora"``: the readout ``lm_head``)."""
        return {"lm_head": self.head_lora} if self.config.adaptation == "lora" else {}

    def view_layers(self) -> list[int]:
        k = self.config.exit_layer or max(1, self.model.config.num_layers // 2)
        return list(range(k))

    def attach(self) -> None:
        super().attach()
        view = self.view
        if self.config.adaptation == "full":
            view.norm = self.norm
            view.lm_head = self.head
        elif self.config.adaptation == "lora":
            install(view, "lm_head", self.head_lora)


def _layerskip():
    import torch.nn.functional as F

    from ...runtime.cache import StepBatch
    from ...train.objective import OBJECTIVES, Objective, OptimDefaults, teacher_pass

    @OBJECTIVES.register("layerskip")
    class LayerSkipObjective(Objective):
        """Cross-entropy of the early exit's readout against the target's greedy next token (LayerSkip's early-exit
        loss); the exit's blocks are the target's own and stay frozen, only the readout adaptation trains."""

        name = "layerskip"
        defaults = OptimDefaults(lr=1e-3, warmup_steps=0)

        def __init__(self, model) -> None:
            super().__init__(model)
            tech = model.techniques["early_exit"] if "early_exit" in model.techniques else None
            if tech is None or tech.config.adaptation == "none":
                raise ConfigError("layerskip trains the readout of an early_exit technique with adaptation='lora' "
                                  "or 'full'")
            self.tech = tech

        def parameters(self):
            return [p for p in self.tech.parameters() if p.requires_grad]

        def loss(self, tokens: torch.Tensor):
            from ...ops.reference import rmsnorm

            tech = self.tech
            view = tech.view
            b, s = tokens.shape
            _, labels = teacher_pass(self.model, tokens, ())
            with torch.no_grad():
                cache = view.new_cache(b, ((s + 127) // 128) * 128)
                lengths = torch.full((b,), s, dtype=torch.int32, device=tokens.device)
                _, aux = view.forward_step(tokens, StepBatch.prefill(lengths, s), cache, capture=(-2,))
                h = aux[-2].float()
            eps = view.config.rms_norm_eps
            if tech.config.adaptation == "full":
                logits = F.linear(rmsnorm(h, tech.norm.float(), eps)[0], tech.head.float())
            else:
                normed = rmsnorm(h, view.norm.float(), eps)[0]
                base = tech.head_lora.base
                base = base if isinstance(base, torch.Tensor) else base.dequantize(torch.float32)
                logits = F.linear(normed, base.float()) + tech.head_lora.delta(normed)
            ce = F.cross_entropy(logits[:, :-1].reshape(-1, logits.shape[-1]), labels[:, :-1].reshape(-1))
            with torch.no_grad():
                acc = float((logits[:, :-1].argmax(-1) == labels[:, :-1]).float().mean())
            return ce, {"loss": float(ce.detach()), "acc": acc}

    return LayerSkipObjective


LayerSkipObjective = _layerskip()
