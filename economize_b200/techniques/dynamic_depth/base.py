"""Machinery of the dynamic-depth techniques (economize ``techniques/dynamic_depth/base.py``).

A :class:`DepthPolicy` is installed as ``model.depth_policy``. In every exact pass of the phases it acts in, the
model hands it each gated layer's input stream ``x`` and output stream ``out`` (``[B, T, H]``) and continues with
what :meth:`DepthPolicy.combine` returns: ``out`` for tokens that run the layer, ``x`` (or a technique-specific
state, e.g. FlexiDepth's adapter) for tokens that skip it. Skipped tokens keep the K/V the layer computed from their
state, which is the K/V convention of every technique here.

The engine runs a pass as one fixed-shape computation (a CUDA graph replay), so a skipped token's layer is computed
and its result discarded: the outputs are exactly those of the method, and the saving is counted (:class:`DepthMeter`
on the device, no host synchronisation) rather than realised (:meth:`DepthTechnique.simulation` says so).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import ClassVar

import torch
import torch.nn.functional as F
from torch import nn

from ...core.technique import Capability, Family, Simulation, Technique, TechniqueConfig
from ...errors import ConfigError
from ...runtime.phase import current_phase

__all__ = ["GENERATION_PHASES", "DepthMeter", "DepthPolicy", "DepthTechnique", "LayeredDepthConfig", "ScalarScore",
           "top_fraction", "unit_rms"]

#: The phases a policy acts in when the prompt runs every layer (``skip_prompt=False``).
GENERATION_PHASES = ("decode", "refresh", None)


def unit_rms(x: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    xf = x.float()
    return xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)


def top_fraction(scores: torch.Tensor, valid: torch.Tensor, fraction: float) -> torch.Tensor:
    """Per row, the ``ceil(fraction * n_valid)`` valid tokens with the highest scores (``[B, T]`` bool)."""
    s = scores.float().masked_fill(~valid, -math.inf)
    k = torch.ceil(valid.sum(1).float() * fraction).long().clamp_min(1)  # [B]
    order = torch.sort(s, dim=1, descending=True, stable=True).indices
    rank = torch.empty_like(order).scatter_(1, order, torch.arange(s.shape[1], device=s.device).expand_as(order))
    return (rank < k[:, None]) & valid


class ScalarScore(nn.Module):
    """A per-token linear score ``w . rms(x) + b`` (``input="rms"``) or ``w . x + b`` (``"raw"``), fp32."""

    def __init__(self, hidden: int, bias: float, std: float, input: str = "rms") -> None:
        super().__init__()
        self.input = input
        self.weight = nn.Parameter(torch.randn(hidden) * std if std > 0 else torch.zeros(hidden))
        self.bias = nn.Parameter(torch.tensor(float(bias)))

    def logit(self, x: torch.Tensor) -> torch.Tensor:
        src = unit_rms(x) if self.input == "rms" else x.float()
        return src @ self.weight.float() + self.bias.float()


class DepthMeter:
    """Per-layer counts of the tokens that entered and that ran each gated layer, accumulated on the device."""

    def __init__(self, num_layers: int, device) -> None:
        self.entered = torch.zeros(num_layers, dtype=torch.int64, device=device)
        self.ran = torch.zeros(num_layers, dtype=torch.int64, device=device)

    def record(self, index: int, valid: torch.Tensor, run: torch.Tensor) -> None:
        self.entered[index] += valid.sum()
        self.ran[index] += (run & valid).sum()

    def reset(self) -> None:
        self.entered.zero_()
        self.ran.zero_()

    def summary(self) -> dict[str, object]:
        entered, ran = self.entered.cpu(), self.ran.cpu()
        total = int(entered.sum())
        return {"layer_tokens_entered": total, "layer_tokens_ran": int(ran.sum()),
                "layer_tokens_skipped": total - int(ran.sum()),
                "run_fraction": float(ran.sum()) / total if total else 1.0,
                "per_layer_run_fraction": [float(r) / e if e else 1.0 for r, e in zip(ran.tolist(),
                                                                                      entered.tolist())]}


class DepthPolicy:
    """Base policy: subclasses implement :meth:`choose` (``[B, T]`` bool, which tokens run layer ``index``) and may
    override :meth:`apply` (the new stream from ``x``, ``out`` and the run mask). ``training`` makes every gated
    layer differentiable (soft gates, every token runs) for the objectives."""

    def __init__(self, technique: DepthTechnique, layers: list[int], phases: tuple) -> None:
        self.technique = technique
        self.layers = set(layers)
        self.phases = phases
        self.training = False
        self.meter = DepthMeter(technique.model.config.num_layers, technique.model.device)
        self.valid: torch.Tensor | None = None
        self.positions: torch.Tensor | None = None
        self.prompt_len: dict[int, torch.Tensor] = {}  # per batch size: a stable buffer (read by captured graphs)
        self.batch_size = 0
        self.gate_log: dict[int, torch.Tensor] = {}  # training: per layer scores (for regularizers)

    def acts(self, batch) -> bool:
        if self.training:
            return True
        if batch.is_prefill or current_phase() == "prefill":  # the last prompt chunk leaves the full length
            self._record_prompt(batch)
        return current_phase() in self.phases or (current_phase() == "prefill" and "prefill" in self.phases)

    def _record_prompt(self, batch) -> None:
        b = batch.n_new.shape[0]
        buf = self.prompt_len.get(b)
        if buf is None:
            buf = self.prompt_len[b] = torch.zeros(b, dtype=torch.int64, device=batch.n_new.device)
        buf.copy_((batch.kv_len + batch.n_new).long())

    def gates(self, index: int) -> bool:
        return index in self.layers

    def begin_pass(self, batch, h: torch.Tensor) -> None:
        bsz, width = h.shape[0], h.shape[1]
        cols = torch.arange(width, device=h.device)
        self.valid = cols[None] < batch.n_new.long()[:, None]
        self.positions = batch.positions.long() if batch.positions is not None else \
            (batch.kv_len.long()[:, None] + cols[None])
        self.batch_size = bsz
        self.gate_log = {}

    def generated(self) -> torch.Tensor:
        """``[B, T]`` generated position of every token (0 = the first token after the prompt)."""
        buf = self.prompt_len.get(self.batch_size)
        base = buf[:, None] if buf is not None else torch.zeros_like(self.positions[:, :1])
        return (self.positions - base).clamp_min(0)

    def choose(self, index: int, x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        raise NotImplementedError

    def apply(self, index: int, x: torch.Tensor, out: torch.Tensor, run: torch.Tensor) -> torch.Tensor:
        return torch.where(run[..., None], out, x)

    def combine(self, index: int, x: torch.Tensor, out: torch.Tensor, batch) -> torch.Tensor:
        run = self.choose(index, x, out)
        if not self.training:
            self.meter.record(index, self.valid, run)
        return self.apply(index, x, out, run).to(x.dtype)


@dataclass(frozen=True)
class LayeredDepthConfig(TechniqueConfig):
    """``layers``: 1-indexed gated layers (empty: the technique's default); ``skip_prompt``: act on the prompt too."""

    technique: ClassVar[str] = ""
    layers: tuple[int, ...] = ()
    skip_prompt: bool = False

    def __post_init__(self) -> None:
        object.__setattr__(self, "layers", tuple(self.layers))
        if any(i < 1 for i in self.layers):
            raise ConfigError(f"layers are 1-indexed, got {self.layers}")

    def validate(self, model) -> None:
        n = model.config.num_layers
        if any(i > n for i in self.layers):
            raise ConfigError(f"layers must be layers of the model's {n}, got {self.layers}")

    def default_layers(self, num_layers: int) -> tuple[int, ...]:
        return tuple(range(1, num_layers + 1))

    def layer_set(self, num_layers: int) -> list[int]:
        return [i - 1 for i in (self.layers or self.default_layers(num_layers))]

    def phases(self) -> tuple:
        return GENERATION_PHASES + (("prefill",) if self.skip_prompt else ())


class DepthTechnique(Technique):
    """Installs its policy as ``model.depth_policy``; :meth:`cost_summary` reports the counted layer applications."""

    capabilities = Capability.DEPTH
    family = Family.DEPTH
    lossless = False

    def __init__(self, config, model) -> None:
        super().__init__(config, model)
        self.layer_ids = config.layer_set(model.config.num_layers) if hasattr(config, "layer_set") else \
            list(range(model.config.num_layers))
        self.policy: DepthPolicy | None = None

    def make_policy(self) -> DepthPolicy:
        raise NotImplementedError

    def attach(self) -> None:
        if self.model.depth_policy is not None and self.model.depth_policy is not self.policy:
            raise ConfigError(f"{self.name}: the model already has a dynamic-depth policy")
        self.policy = self.make_policy()
        self.model.depth_policy = self.policy

    def detach(self) -> None:
        if self.model.depth_policy is self.policy:
            self.model.depth_policy = None

    def depth_stats(self) -> dict[str, object]:
        return self.policy.meter.summary() if self.policy is not None else {}

    def cost_summary(self, result=None) -> dict[str, object]:
        out = dict(result.cost_summary()) if result is not None and hasattr(result, "cost_summary") else {}
        out.update(self.depth_stats())
        return out

    def simulation(self) -> Simulation | None:
        return Simulation("layer compute", "a batched pass computes every gated layer and discards the skipped "
                                           "tokens' results; the skipped applications are counted")

    def conflicts(self, other: Technique) -> str | None:
        if other.family == Family.DEPTH and other is not self:
            return f"{self.name} and {other.name} both decide the depth of the exact passes"
        return super().conflicts(other)
