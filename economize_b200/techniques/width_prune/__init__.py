"""Width pruning of the MLP (``width_prune``; FLAP, An et al. 2024; economize ``techniques/width_prune``).

Every FFN channel ``c`` of a layer is scored by ``E[a_c^2] * ||W_down[:, c]||^2`` over calibration tokens (the
second moment of the SwiGLU activation feeding ``w_down`` times the squared norm of the column it multiplies: the
expected output energy the channel contributes, FLAP's fluctuation metric taken around zero); the lowest-scoring
``ratio`` of channels is removed (rows of gate/up, columns of down), with the channel count rounded to a multiple of
64 for the GEMM tiles. FLAP's bias compensation needs a bias on ``w_down``, which Llama MLPs do not have, so the
channels are dropped without it. Refuses tensor-parallel models, like the reference
(``width_prune/config.py:192``).

``recovery_rank > 0`` adds LLM-Pruner's recovery stage (economize ``width_prune/recovery.py:25``): a LoRA update
(rank ``recovery_rank``, ``alpha = recovery_alpha``) of every pruned layer's projections that is always applied (the
pruned model is the base, there is no exact path to protect); ``train.fit(model, tokens)`` trains it with the
``recovery_ce`` objective (next-token cross-entropy of the pruned model), and the adapters are listed by
:meth:`WidthPruneTechnique.lora_targets` for PEFT export.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import ClassVar

import torch
from torch import nn

from ...core.technique import Capability, Family, Technique, TechniqueConfig, register_technique
from ...errors import ConfigError
from ..quant.methods import collect

__all__ = ["WidthPruneConfig", "WidthPruneTechnique"]


@dataclass(frozen=True)
class WidthPruneConfig(TechniqueConfig):
    technique: ClassVar[str] = "width_prune"
    ratio: float = 0.2
    layers: tuple[int, ...] = ()
    recovery_rank: int = 0
    recovery_alpha: float = 16.0

    def __post_init__(self) -> None:
        if not 0.0 < self.ratio < 1.0:
            raise ConfigError("ratio must lie in (0, 1)")
        if self.recovery_rank < 0:
            raise ConfigError("recovery_rank must be >= 0")
        object.__setattr__(self, "layers", tuple(int(i) for i in self.layers))

    def validate(self, model) -> None:
        if model.tp is not None and model.tp.size > 1:
            raise ConfigError("width_prune refuses tensor-parallel models")
        if model.config.is_moe:
            raise ConfigError("width_prune supports dense MLPs")


@register_technique
class WidthPruneTechnique(Technique):
    config_class = WidthPruneConfig
    capabilities = Capability.WEIGHTS
    family = Family.PRUNING
    lossless = False

    objective_name = "recovery_ce"
    #: engine projections with a recovery adapter, and the Hugging Face module names they fuse
    RECOVERY = {"wqkv": ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj"), "wo": ("self_attn.o_proj",),
                "w_gate_up": ("mlp.gate_proj", "mlp.up_proj"), "w_down": ("mlp.down_proj",)}

    def __init__(self, config: WidthPruneConfig, model) -> None:
        super().__init__(config, model)
        self._calibration = None
        self.kept: dict[int, torch.Tensor] = {}
        self.recovery = nn.ModuleDict()  # "layer/projection" -> LoRAWeight

    def calibrate(self, calibration) -> None:
        self._calibration = calibration

    @torch.no_grad()
    def attach(self) -> None:
        cfg: WidthPruneConfig = self.config
        m = self.model
        layers = [i - 1 for i in cfg.layers] if cfg.layers else list(range(m.config.num_layers))
        if not self.kept:
            cal = self._calibration
            if cal is None:
                raise ConfigError("width_prune needs calibration tokens")
            batches = [cal if cal.dim() == 2 else cal[None]] if isinstance(cal, torch.Tensor) else list(cal)
            stats = collect(m, batches, {i: ["w_down"] for i in layers}, hessian=True, keep_rows=0)
            for i in layers:
                st = stats[(i, "w_down")]
                fluct = torch.diagonal(st.h) / max(st.n, 1)  # E[a_c^2]
                w_down = m.layers[i].w_down.float()
                score = fluct * (w_down ** 2).sum(0)
                f = score.numel()
                keep_n = max(64, int(round(f * (1 - cfg.ratio) / 64)) * 64)
                self.kept[i] = score.topk(min(keep_n, f)).indices.sort().values
        for i, idx in self.kept.items():
            layer = m.layers[i]
            f = layer.w_down.shape[1]
            idx = idx.to(layer.w_down.device)
            gate, up = layer.w_gate_up.data[:f], layer.w_gate_up.data[f:]
            layer.w_gate_up = nn.Parameter(torch.cat([gate[idx], up[idx]], 0).contiguous())
            layer.w_down = nn.Parameter(layer.w_down.data[:, idx].contiguous())
        if cfg.recovery_rank > 0:
            self._install_recovery()

    def _install_recovery(self) -> None:
        """Wrap every pruned layer's projections in always-on LoRA updates (the technique owns them)."""
        from ...ops.lora import LoRAWeight

        cfg: WidthPruneConfig = self.config
        for i in sorted(self.kept):
            layer = self.model.layers[i]
            for name in self.RECOVERY:
                key = f"{i}/{name}"
                base = getattr(layer, name)
                if key not in self.recovery:
                    self.recovery[key] = LoRAWeight(base, cfg.recovery_rank, cfg.recovery_alpha, seed=i)
                lora = self.recovery[key]
                saved = getattr(self, "_loaded_recovery", {})
                name_a = f"recovery.{key.replace('/', '.')}.a"
                if name_a in saved:  # a checkpoint's trained adapter
                    with torch.no_grad():
                        lora.a.copy_(saved[name_a])
                        lora.b.copy_(saved[name_a[:-1] + "b"])
                lora._base[0] = base if not isinstance(base, LoRAWeight) else base.base
                if name in layer._parameters:
                    del layer._parameters[name]
                setattr(layer, name, lora)

    def lora_targets(self) -> dict:
        """The recovery adapters by the Hugging Face module names of the maps they update."""
        out = {}
        for key, lora in self.recovery.items():
            i, name = key.split("/")
            for hf in self.RECOVERY[name]:
                out[f"model.layers.{i}.{hf}"] = lora
        return out

    def technique_state(self) -> dict[str, torch.Tensor]:
        out = {f"kept.{i}": idx for i, idx in self.kept.items()}
        for key, lora in self.recovery.items():
            out[f"recovery.{key.replace('/', '.')}.a"] = lora.a.detach()
            out[f"recovery.{key.replace('/', '.')}.b"] = lora.b.detach()
        return out

    def load_technique_state(self, state: dict[str, torch.Tensor]) -> None:
        self.kept = {int(k.split(".")[1]): v.long() for k, v in state.items() if k.startswith("kept.")}
        self._loaded_recovery = {k: v for k, v in state.items() if k.startswith("recovery.")}

