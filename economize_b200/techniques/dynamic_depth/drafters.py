"""The dynamic-depth methods that decode through the drafting cycle (economize
``techniques/dynamic_depth/{free,dmtd,hidden_transfer}.py``).

* ``free`` (Bae et al. 2023): the first ``exit_layer`` layers with the shared head are the shallow model; a chain
  stops at the first token whose confidence (top-1 minus top-2 probability) is below ``threshold``, and that token
  goes to the exact pass (the synchronized parallel pass over the stacked shallow tokens). Every earlier draft is
  kept (``accept_all``: lossy).
* ``dmtd`` (Luo et al. 2025): cycles of ``cycle_length`` tokens; the first runs every layer (the exact pass, which
  also refills the early layers' K/V of the tokens that skipped them), the others run only the last
  ``decoding_layers`` layers on their token embedding (a layer view). Every draft is kept (lossy).
* ``hidden_transfer`` (Wu et al. 2024): after an exact pass ending at ``n``, step ``i`` maps the state of ``n`` after
  layer ``t_i`` through ``W_i`` to a pseudo state of position ``n + i``, runs layers ``t_i + 1 .. L`` on it against
  the target's own cache and drafts token ``n + i + 1`` from the LM head. The target verifies (lossless).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import ClassVar

import torch
import torch.nn.functional as F
from torch import nn

from ...core.technique import Capability, Family, Technique, TechniqueConfig, register_technique
from ...decoding.config import DecodeConfig
from ...errors import ConfigError
from ...runtime.cache import StepBatch
from ...train.objective import OBJECTIVES, Objective, OptimDefaults, torch_block
from ...validation import check_choice, check_positive, check_unit_interval
from .._self_draft import SelfDraftTechnique

__all__ = ["DmtdConfig", "DmtdTechnique", "FreeConfig", "FreeTechnique", "HiddenTransferConfig",
           "HiddenTransferTechnique"]


# ---- FREE ------------------------------------------------------------------------------------------------------
@dataclass(frozen=True)
class FreeConfig(TechniqueConfig):
    """``exit_layer``: shallow depth (``None``: a quarter of the layers); ``threshold``: the confidence ``lambda``;
    ``max_exits``: most consecutive shallow tokens per cycle; ``head``: ``"shared"`` (the model's head);
    ``posterior`` / ``adaptation``: accepted for configuration compatibility (``adaptation`` must be ``"frozen"``:
    the shallow model is the deep model's first layers)."""

    technique: ClassVar[str] = "free"
    exit_layer: int | None = None
    head: str = "shared"
    threshold: float = 0.9
    posterior: float = 0.4
    max_exits: int = 31
    adaptation: str = "frozen"

    def __post_init__(self) -> None:
        check_unit_interval("threshold", self.threshold, closed_high=True)
        check_positive("max_exits", self.max_exits)
        check_choice("head", self.head, ("shared",))
        check_choice("adaptation", self.adaptation, ("frozen",))
        if self.exit_layer is not None and self.exit_layer < 1:
            raise ConfigError("exit_layer must be >= 1")

    def validate(self, model) -> None:
        if self.exit_layer is not None and self.exit_layer >= model.config.num_layers:
            raise ConfigError("exit_layer must be below the number of layers")


@register_technique
class FreeTechnique(SelfDraftTechnique):
    config_class = FreeConfig
    lossless = False

    def view_layers(self) -> list[int]:
        return list(range(self.config.exit_layer or max(1, self.model.config.num_layers // 4)))

    def drafter(self):
        d = super().drafter()
        d.confidence_measure = "gap"
        d.stop_inclusive = True
        return d

    def decode_config(self, max_exits: int | None = None) -> DecodeConfig:
        """Decoding options of FREE: chains of up to ``max_exits`` shallow tokens, every kept draft accepted."""
        n = max_exits or self.config.max_exits
        return DecodeConfig(cycle_length=n + 1, lossless=False, min_confidence=self.config.threshold,
                            draft_policy="confidence")

    def default_decoding(self) -> DecodeConfig:
        # a captured cycle runs all its draft steps, so the default chain is shorter than the paper's bound
        return self.decode_config(min(self.config.max_exits, 7))


# ---- DMTD ------------------------------------------------------------------------------------------------------
@dataclass(frozen=True)
class DmtdConfig(TechniqueConfig):
    """``decoding_layers``: the late layers ``L_d`` that draft; ``cycle_length``: ``tau``; ``predictor``:
    ``"embedding"`` (the token embedding is the late layers' input state)."""

    technique: ClassVar[str] = "dmtd"
    decoding_layers: int = 8
    cycle_length: int = 3
    adaptation: str = "full"
    predictor: str = "embedding"

    def __post_init__(self) -> None:
        check_positive("decoding_layers", self.decoding_layers)
        if self.cycle_length < 2:
            raise ConfigError("cycle_length (tau) must be at least 2")
        check_choice("predictor", self.predictor, ("embedding",))
        check_choice("adaptation", self.adaptation, ("full", "frozen"))

    def validate(self, model) -> None:
        if self.decoding_layers >= model.config.num_layers:
            raise ConfigError("decoding_layers must be below the number of layers")


@register_technique
class DmtdTechnique(SelfDraftTechnique):
    config_class = DmtdConfig
    lossless = False

    def view_layers(self) -> list[int]:
        n = self.model.config.num_layers
        return list(range(n - self.config.decoding_layers, n))

    def default_decoding(self) -> DecodeConfig:
        return DecodeConfig(cycle_length=self.config.cycle_length, lossless=False)

    def layers_per_token(self) -> float:
        """The paper's PLT ``(L + (tau - 1) L_d) / (tau L)``."""
        n, tau, ld = self.model.config.num_layers, self.config.cycle_length, self.config.decoding_layers
        return (n + (tau - 1) * ld) / (tau * n)


# ---- Hidden Transfer -------------------------------------------------------------------------------------------
@dataclass(frozen=True)
class HiddenTransferConfig(TechniqueConfig):
    """``transfer_layers``: the 1-indexed layers ``t_i`` after which step ``i`` transfers (``None``: from
    ``transfer_fractions`` of the depth); ``param_dtype``: ``"float32"`` or ``"model"``."""

    technique: ClassVar[str] = "hidden_transfer"
    transfer_layers: tuple[int, ...] | None = None
    transfer_fractions: tuple[float, ...] = (0.625, 0.75, 0.875)
    train_context: str = "teacher"
    param_dtype: str = "float32"

    def __post_init__(self) -> None:
        if self.transfer_layers is not None:
            object.__setattr__(self, "transfer_layers", tuple(int(t) for t in self.transfer_layers))
            if not self.transfer_layers or list(self.transfer_layers) != sorted(set(self.transfer_layers)):
                raise ConfigError("transfer_layers must be increasing")
        object.__setattr__(self, "transfer_fractions", tuple(self.transfer_fractions))
        if not self.transfer_fractions or any(not 0 < f < 1 for f in self.transfer_fractions):
            raise ConfigError("transfer_fractions must lie in (0, 1)")
        check_choice("train_context", self.train_context, ("teacher",))
        check_choice("param_dtype", self.param_dtype, ("float32", "model"))

    def layers_for(self, num_layers: int) -> tuple[int, ...]:
        if self.transfer_layers is not None:
            return self.transfer_layers
        out = sorted({min(num_layers - 1, max(1, round(f * num_layers))) for f in self.transfer_fractions})
        return tuple(out)

    def validate(self, model) -> None:
        if any(not 1 <= t < model.config.num_layers for t in self.layers_for(model.config.num_layers)):
            raise ConfigError("transfer layers must lie in 1 .. num_layers - 1")


class HiddenTransferDrafter:
    """Runs the transfer steps at observe time (against the target's cache) and hands the drafted distributions
    to the engine's chain or tree steps."""

    def __init__(self, tech: HiddenTransferTechnique) -> None:
        self.tech = tech
        self.layers = tech.transfer_layers
        self.capture_layers = self.layers
        h = tech.model.config.hidden_size
        self.carry_size = len(self.layers) * h
        self.cache = None
        self.stash: torch.Tensor | None = None
        self._step = 0

    def begin(self, batch: int, capacity: int) -> None:
        v = self.tech.model.config.vocab_size
        k = len(self.layers)
        if self.stash is None or self.stash.shape[0] != batch:
            self.stash = torch.zeros(batch, k, v, dtype=torch.float32, device=self.tech.model.device)

    def bind_target_cache(self, cache) -> None:
        self.cache = cache

    def draft_depth(self, decode: DecodeConfig) -> int:
        return max(1, decode.cycle_length - 1)

    def draft_nodes(self, decode: DecodeConfig) -> int:
        return self.draft_depth(decode)

    def fuse(self, aux: dict[int, torch.Tensor]) -> torch.Tensor:
        return torch.cat([aux[t] for t in self.layers], -1)

    def observe(self, tokens, sources, kv_len, n_valid, root):
        model, tech = self.tech.model, self.tech
        batch = tokens.shape[0]
        dev = tokens.device
        rows = torch.arange(batch, device=dev)
        h = model.config.hidden_size
        state = sources[rows, root.long()]  # [B, k H]: the root token's states after every transfer layer
        slot = (kv_len + root).to(torch.int32)  # the bonus token's position: the first pseudo state's
        dummy = torch.zeros(batch, 1, dtype=torch.long, device=dev)
        one = torch.ones(batch, dtype=torch.int32, device=dev)
        for i, t in enumerate(self.layers):
            src = state[:, i * h:(i + 1) * h]
            pseudo = tech.maps[i](src.to(tech.maps[i].weight.dtype)).to(model.dtype)
            pos = slot + i
            hidden, _ = model.forward_step(dummy, StepBatch(pos, one, pos[:, None].contiguous()), self.cache,
                                           layers=range(t, model.config.num_layers), hidden=pseudo[:, None])
            self.stash[:, i].copy_(model.logits(hidden[:, 0]).float())
        self._step = 0
        return self.stash[:, 0], torch.zeros(batch, h, dtype=model.dtype, device=dev)

    def tree_step(self, tokens, states, positions, kv_base, n_forwarded, q_offset, mask):
        self._step = min(self._step + 1, self.stash.shape[1] - 1)
        w = tokens.shape[1]
        return self.stash[:, self._step][:, None].expand(-1, w, -1), states

    def to_target(self, ids: torch.Tensor) -> torch.Tensor:
        return ids


@register_technique
class HiddenTransferTechnique(Technique):
    config_class = HiddenTransferConfig
    capabilities = Capability.DRAFTER
    family = Family.DRAFTER
    lossless = True
    objective_name = "hidden_transfer_kl"

    def __init__(self, config: HiddenTransferConfig, model) -> None:
        super().__init__(config, model)
        h = model.config.hidden_size
        self.transfer_layers = config.layers_for(model.config.num_layers)
        dtype = torch.float32 if config.param_dtype == "float32" else model.dtype
        maps = []
        for _ in self.transfer_layers:
            m = nn.Linear(h, h, bias=False)
            with torch.no_grad():
                m.weight.copy_(torch.eye(h))
            maps.append(m)
        self.maps = nn.ModuleList(maps).to(device=model.device, dtype=dtype)

    def drafter(self):
        return HiddenTransferDrafter(self)

    def default_decoding(self) -> DecodeConfig:
        return DecodeConfig(cycle_length=len(self.transfer_layers) + 1)


def _float_layer(layer):
    names = ("attn_norm", "wqkv", "bqkv", "wo", "q_norm", "k_norm", "mlp_norm", "w_gate_up", "w_down")
    return type("L", (), {n: (getattr(layer, n).float() if isinstance(getattr(layer, n), torch.Tensor)
                              else getattr(layer, n)) for n in names})


@OBJECTIVES.register("hidden_transfer_kl")
class HiddenTransferDistill(Objective):
    """``sum_i KL(P_{q+i} || P~_{i, q})``: the distribution drafted by step ``i`` from position ``q`` against the
    model's distribution at ``q + i``; the pseudo states run the upper layers as one causal sequence."""

    name = "hidden_transfer_kl"
    defaults = OptimDefaults(lr=1e-3, warmup_steps=0, grad_clip=1.0)

    def __init__(self, model) -> None:
        super().__init__(model)
        if "hidden_transfer" not in model.techniques:
            raise ConfigError("hidden_transfer_kl needs an attached hidden_transfer technique")
        self.tech = model.techniques["hidden_transfer"]

    def parameters(self):
        return list(self.tech.maps.parameters())

    def loss(self, tokens: torch.Tensor):
        from ...ops.reference import rmsnorm

        tech = self.tech
        model = tech.model
        cfg = model.config
        b, s = tokens.shape
        with torch.no_grad():
            cache = model.new_cache(b, ((s + 127) // 128) * 128)
            lengths = torch.full((b,), s, dtype=torch.int32, device=tokens.device)
            hidden, aux = model.forward_step(tokens, StepBatch.prefill(lengths, s), cache,
                                             capture=tech.transfer_layers)
            teacher = torch.log_softmax(model.logits(hidden).float(), -1)
        cos, sin = model.rope_tables(s)
        total, metrics = 0.0, {}
        for i, t in enumerate(tech.transfer_layers, start=1):
            if s <= i:
                continue
            x = tech.maps[i - 1](aux[t].detach().to(tech.maps[i - 1].weight.dtype)).float()
            for j in range(t, cfg.num_layers):
                x = torch_block(_float_layer(model.layers[j]), x, cfg, cos, sin)
            logp = torch.log_softmax(F.linear(rmsnorm(x, model.norm.float(), cfg.rms_norm_eps)[0],
                                              model.head_weight.float()), -1)
            kl = F.kl_div(logp[:, : s - i], teacher[:, i:], log_target=True, reduction="batchmean") / (s - i)
            total = total + kl
            metrics[f"kl{i}"] = float(kl.detach())
        loss = total / len(tech.transfer_layers)
        metrics["loss"] = float(loss.detach())
        return loss, metrics
