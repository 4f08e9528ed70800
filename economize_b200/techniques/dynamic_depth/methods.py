"""The exact-path dynamic-depth techniques: GateSkip, Mixture-of-Depths, FlexiDepth, SkipDecode, LoRA-Drop and CALM
(economize ``techniques/dynamic_depth/{gateskip,mod,flexidepth,skipdecode,loradrop,calm}.py``).

* ``gateskip`` (Laitenberger et al. 2025, layer-level variant): gate ``g = sigmoid(w . rms(x) + b)`` per layer; a
  token runs when ``g >= threshold`` (or is among the ``budget`` fraction with the highest gates of its row) and
  leaves as ``x + g (layer(x) - x)``, otherwise as ``x``.
* ``mod`` (Raposo et al. 2024): router ``r = w . x + b`` on every second layer; a token runs when ``r > threshold``
  and leaves as ``x + r (layer(x) - x)``.
* ``flexidepth`` (Luo et al. 2025, layer-level variant): ``g = sigmoid(router(x))``; a token with ``g > threshold``
  leaves as ``x + g (layer(x) - x)``, any other as ``x + (1 - g) adapter(rms(x))`` (a narrow SwiGLU).
* ``skipdecode`` (Del Corro et al. 2023): the ``t``-th generated token runs ``active(t)`` layers (a linear decline
  from ``max_layers`` to ``min_layers``), skipping the lowest (``"bottom"``) or highest (``"top"``) ones; one budget
  per step for the batch (``batch_uniform``).
* ``loradrop`` (Rajabzadeh et al. 2026): droppable layers run in full for every ``period``-th generated token (the
  anchor); between anchors a token leaves as ``h_l(anchor) + B A x * alpha / rank``.
* ``calm`` (Schuster et al. 2022): a token exits after the first layer ``>= min_layer`` whose confidence
  (``softmax`` top-1 minus top-2 of the head, ``state`` saturation, or a trained ``classifier``) exceeds the
  threshold ``0.9 lambda + 0.1 exp(-tau t / N)``; later layers keep its state.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import ClassVar

import torch
import torch.nn.functional as F
from torch import nn

from ...core.technique import register_technique
from ...errors import ConfigError
from ...validation import check_choice, check_non_negative, check_positive, check_unit_interval
from .base import DepthPolicy, DepthTechnique, LayeredDepthConfig, ScalarScore, top_fraction, unit_rms

__all__ = ["CONFIDENCE_MEASURES", "CalmConfig", "CalmTechnique", "FlexiDepthConfig", "FlexiDepthTechnique",
           "GATESKIP_RULES", "GateSkipConfig", "GateSkipTechnique", "LoRADropConfig", "LoRADropTechnique",
           "MoDConfig", "MoDTechnique", "SkipDecodeConfig", "SkipDecodeTechnique"]

GATESKIP_RULES = ("threshold", "budget")
CONFIDENCE_MEASURES = ("softmax", "state", "classifier")
FLEXI_ROUTERS = ("paper", "bottleneck")


# ---- GateSkip --------------------------------------------------------------------------------------------------
@dataclass(frozen=True)
class GateSkipConfig(LayeredDepthConfig):
    technique: ClassVar[str] = "gateskip"
    rule: str = "threshold"
    threshold: float = 0.5
    budget: float = 1.0
    gate_bias: float = 5.0
    gate_init_std: float = 0.0

    def __post_init__(self) -> None:
        super().__post_init__()
        check_choice("rule", self.rule, GATESKIP_RULES)
        check_unit_interval("threshold", self.threshold, closed_low=True, closed_high=True)
        check_unit_interval("budget", self.budget, closed_high=True)
        check_non_negative("gate_init_std", self.gate_init_std)


class _ScoredPolicy(DepthPolicy):
    def score(self, index: int, x: torch.Tensor) -> torch.Tensor:
        raise NotImplementedError

    def choose(self, index, x, out):
        s = self.score(index, x)
        self._score = s
        if self.training:
            self.gate_log[index] = s
            return torch.ones_like(self.valid)
        return self.select(index, s)


class GateSkipPolicy(_ScoredPolicy):
    def score(self, index, x):
        return torch.sigmoid(self.technique.gates[str(index)].logit(x))

    def select(self, index, g):
        cfg = self.technique.config
        if cfg.rule == "budget":
            return top_fraction(g, self.valid, cfg.budget)
        return g >= cfg.threshold

    def apply(self, index, x, out, run):
        g = self._score[..., None]
        ran = x.float() + g * (out.float() - x.float())
        return torch.where(run[..., None], ran, x.float())


@register_technique
class GateSkipTechnique(DepthTechnique):
    config_class = GateSkipConfig
    objective_name = "gateskip"

    def __init__(self, config: GateSkipConfig, model) -> None:
        super().__init__(config, model)
        h = model.config.hidden_size
        self.gates = nn.ModuleDict({str(i): ScalarScore(h, config.gate_bias, config.gate_init_std, "rms")
                                    for i in self.layer_ids}).to(model.device)

    def make_policy(self):
        return GateSkipPolicy(self, self.layer_ids, self.config.phases())


# ---- Mixture-of-Depths -----------------------------------------------------------------------------------------
@dataclass(frozen=True)
class MoDConfig(LayeredDepthConfig):
    technique: ClassVar[str] = "mod"
    capacity: float = 0.125
    router_bias: float = 1.0
    router_init_std: float = 0.0
    router_input: str = "raw"
    kv: str = "fill"
    threshold: float = 0.0

    def __post_init__(self) -> None:
        super().__post_init__()
        check_unit_interval("capacity", self.capacity, closed_high=True)
        check_choice("router_input", self.router_input, ("raw", "rms"))
        if self.kv != "fill":
            raise ConfigError("mod kv='routed' (no K/V for routed-around tokens) needs a routed-K/V attention; "
                              "this engine fills the K/V of every token (kv='fill')")

    def default_layers(self, num_layers: int) -> tuple[int, ...]:
        return tuple(range(2, num_layers + 1, 2))


class MoDPolicy(_ScoredPolicy):
    def score(self, index, x):
        return self.technique.routers[str(index)].logit(x)

    def select(self, index, r):
        return r > self.technique.config.threshold

    def apply(self, index, x, out, run):
        if self.training:  # per-sequence top-k capacity in training (the paper's rule)
            run = top_fraction(self._score.detach(), self.valid, self.technique.config.capacity)
            self.gate_log[(index, "topk")] = run
        r = self._score[..., None]
        ran = x.float() + r * (out.float() - x.float())
        return torch.where(run[..., None], ran, x.float())


@register_technique
class MoDTechnique(DepthTechnique):
    config_class = MoDConfig
    objective_name = "mod"

    def __init__(self, config: MoDConfig, model) -> None:
        super().__init__(config, model)
        h = model.config.hidden_size
        self.routers = nn.ModuleDict({str(i): ScalarScore(h, config.router_bias, config.router_init_std,
                                                          config.router_input) for i in self.layer_ids}).to(model.device)

    def make_policy(self):
        return MoDPolicy(self, self.layer_ids, self.config.phases())


# ---- FlexiDepth ------------------------------------------------------------------------------------------------
@dataclass(frozen=True)
class FlexiDepthConfig(LayeredDepthConfig):
    technique: ClassVar[str] = "flexidepth"
    threshold: float = 0.5
    router: str = "paper"
    router_reduction: int = 16
    adapter_reduction: int = 16
    router_bias: float = 5.0

    def __post_init__(self) -> None:
        super().__post_init__()
        check_unit_interval("threshold", self.threshold)
        check_choice("router", self.router, FLEXI_ROUTERS)
        check_positive("router_reduction", self.router_reduction)
        check_positive("adapter_reduction", self.adapter_reduction)

    def default_layers(self, num_layers: int) -> tuple[int, ...]:
        return tuple(range(num_layers // 2 + 1, num_layers + 1))


class _RMSNorm(nn.Module):
    def __init__(self, width: int) -> None:
        super().__init__()
        self.weight = nn.Parameter(torch.ones(width))

    def forward(self, x):
        return unit_rms(x) * self.weight.float()


class FlexiRouter(nn.Module):
    """``"paper"``: ``head(dec(tanh(norm(enc(n(x))))))``; ``"bottleneck"``: ``out(silu(down(n(x))))``. Returns logits."""

    def __init__(self, hidden: int, reduction: int, bias: float, kind: str) -> None:
        super().__init__()
        w = max(1, hidden // reduction)
        self.kind = kind
        self.input_norm = _RMSNorm(hidden)
        if kind == "paper":
            self.enc = nn.Linear(hidden, w, bias=False)
            self.norm = _RMSNorm(w)
            self.dec = nn.Linear(w, w, bias=False)
            self.head = nn.Linear(w, 1)
            out = self.head
        else:
            self.down = nn.Linear(hidden, w)
            self.out = nn.Linear(w, 1)
            out = self.out
        with torch.no_grad():
            out.weight.zero_()
            out.bias.fill_(bias)

    def forward(self, x):
        n = self.input_norm(x)
        if self.kind == "paper":
            return self.head(self.dec(torch.tanh(self.norm(self.enc(n)))))[..., 0]
        return self.out(F.silu(self.down(n)))[..., 0]


class SwiGLUAdapter(nn.Module):
    def __init__(self, hidden: int, width: int) -> None:
        super().__init__()
        self.norm = _RMSNorm(hidden)
        self.gate_proj = nn.Linear(hidden, width, bias=False)
        self.up_proj = nn.Linear(hidden, width, bias=False)
        self.down_proj = nn.Linear(width, hidden, bias=False)
        nn.init.zeros_(self.down_proj.weight)

    def forward(self, x):
        n = self.norm(x)
        return self.down_proj(F.silu(self.gate_proj(n)) * self.up_proj(n))


class FlexiDepthPolicy(_ScoredPolicy):
    def score(self, index, x):
        return torch.sigmoid(self.technique.routers[str(index)](x.float()))

    def select(self, index, g):
        return g > self.technique.config.threshold

    def apply(self, index, x, out, run):
        g = self._score[..., None]
        xf = x.float()
        ran = xf + g * (out.float() - xf)
        skipped = xf + (1 - g) * self.technique.adapters[str(index)](xf)
        if self.training:  # hard routing by the threshold; both branches carry the router's gradient
            run = g[..., 0] > self.technique.config.threshold
        return torch.where(run[..., None], ran, skipped)


@register_technique
class FlexiDepthTechnique(DepthTechnique):
    config_class = FlexiDepthConfig
    objective_name = "flexidepth"

    def __init__(self, config: FlexiDepthConfig, model) -> None:
        super().__init__(config, model)
        c = model.config
        h = c.hidden_size
        self.routers = nn.ModuleDict({str(i): FlexiRouter(h, config.router_reduction, config.router_bias,
                                                          config.router) for i in self.layer_ids}).to(model.device)
        self.adapters = nn.ModuleDict({str(i): SwiGLUAdapter(h, max(1, c.intermediate_size // config.adapter_reduction))
                                       for i in self.layer_ids}).to(model.device)

    def make_policy(self):
        return FlexiDepthPolicy(self, self.layer_ids, self.config.phases())


# ---- SkipDecode ------------------------------------------------------------------------------------------------
@dataclass(frozen=True)
class SkipDecodeConfig(LayeredDepthConfig):
    technique: ClassVar[str] = "skipdecode"
    max_layers: int = 0
    min_layers: int = 0
    warmup: int = 0
    decay: int = 256
    skip: str = "bottom"
    batch_uniform: bool = True
    fill_kv: bool = False

    def __post_init__(self) -> None:
        super().__post_init__()
        for name in ("max_layers", "min_layers", "warmup"):
            check_non_negative(name, getattr(self, name))
        check_positive("decay", self.decay)
        check_choice("skip", self.skip, ("bottom", "top"))
        if self.max_layers and self.min_layers and self.min_layers > self.max_layers:
            raise ConfigError("min_layers exceeds max_layers")

    def validate(self, model) -> None:
        super().validate(model)
        n = model.config.num_layers
        if self.max_layers > n or self.min_layers > n:
            raise ConfigError(f"layer budgets must not exceed the model's {n} layers")

    def active(self, generated: torch.Tensor, num_layers: int) -> torch.Tensor:
        """Layers the token at generated position ``generated`` runs."""
        hi = self.max_layers or num_layers
        lo = self.min_layers or num_layers
        t = (generated.float() - self.warmup).clamp_min(0) / self.decay
        return torch.ceil(hi - (hi - lo) * t.clamp(max=1.0)).long()


class SkipDecodePolicy(DepthPolicy):
    def begin_pass(self, batch, h):
        super().begin_pass(batch, h)
        cfg, n = self.technique.config, self.technique.model.config.num_layers
        active = cfg.active(self.generated(), n)  # [B, T]
        if cfg.batch_uniform:  # one budget per column: the largest over the valid rows
            col = active.masked_fill(~self.valid, 0).amax(0, keepdim=True)
            active = col.expand_as(active)
        self._active = active

    def choose(self, index, x, out):
        n = self.technique.model.config.num_layers
        if self.technique.config.skip == "bottom":
            return index >= n - self._active
        return index < self._active


@register_technique
class SkipDecodeTechnique(DepthTechnique):
    config_class = SkipDecodeConfig

    def make_policy(self):
        return SkipDecodePolicy(self, self.layer_ids, self.config.phases())


# ---- LoRA-Drop -------------------------------------------------------------------------------------------------
@dataclass(frozen=True)
class LoRADropConfig(LayeredDepthConfig):
    technique: ClassVar[str] = "loradrop"
    period: int = 2
    rank: int = 16
    alpha: float = 16.0

    def __post_init__(self) -> None:
        super().__post_init__()
        check_positive("period", self.period)
        check_positive("rank", self.rank)
        check_positive("alpha", self.alpha)

    def default_layers(self, num_layers: int) -> tuple[int, ...]:
        return tuple(range(4, num_layers))  # all but the first three and the last (1-indexed)


class LoRAUpdate(nn.Module):
    """``B A x * alpha / rank`` (``B`` starts at zero)."""

    def __init__(self, hidden: int, rank: int, alpha: float) -> None:
        super().__init__()
        self.a = nn.Parameter(torch.randn(rank, hidden) / math.sqrt(hidden))
        self.b = nn.Parameter(torch.zeros(hidden, rank))
        self.scale = alpha / rank

    def forward(self, x):
        return (x.float() @ self.a.float().t()) @ self.b.float().t() * self.scale


class LoRADropPolicy(DepthPolicy):
    def __init__(self, technique, layers, phases) -> None:
        super().__init__(technique, layers, phases)
        self.slot = {i: j for j, i in enumerate(sorted(layers))}
        self.anchors: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}  # per batch size: states, positions

    def _buffers(self, bsz: int, like: torch.Tensor):
        buf = self.anchors.get(bsz)
        if buf is None:
            n = len(self.slot)
            buf = (torch.zeros(bsz, n, like.shape[-1], dtype=like.dtype, device=like.device),
                   torch.full((bsz, n), -1, dtype=torch.long, device=like.device))
            self.anchors[bsz] = buf
        return buf

    def begin_pass(self, batch, h):
        super().begin_pass(batch, h)
        self._full = (self.generated() % self.technique.config.period == 0) & self.valid
        if self.training:
            self._full = torch.zeros_like(self._full)

    def choose(self, index, x, out):
        return self._full

    def apply(self, index, x, out, run):
        lora = self.technique.updates[str(index)](x)
        if self.training:  # the update learns to imitate the layer from the token's own input
            self.gate_log[index] = (lora, out.float() - x.float())
            return x.float() + lora
        states, pos = self._buffers(x.shape[0], x)
        j = self.slot[index]
        width = x.shape[1]
        cols = torch.arange(width, device=x.device).expand(x.shape[0], width)
        # latest full column <= t in this pass, else the stored anchor (valid when it precedes the pass)
        last_full = torch.where(run, cols, torch.full_like(cols, -1)).cummax(1).values
        stored_ok = pos[:, j] < self.positions[:, 0]
        in_pass = last_full.clamp_min(0)
        anchor_pass = out.float().gather(1, in_pass[..., None].expand(-1, -1, out.shape[-1]))
        anchor = torch.where((last_full >= 0)[..., None], anchor_pass,
                             torch.where(stored_ok[:, None, None], states[:, j][:, None].float(), x.float()))
        dropped = anchor + lora
        new = torch.where(run[..., None], out.float(), dropped)
        # keep this pass's last full token as the row's anchor
        has = run.any(1)
        last_col = torch.where(run, cols, torch.full_like(cols, -1)).amax(1).clamp_min(0)
        rows = torch.arange(x.shape[0], device=x.device)
        states[:, j] = torch.where(has[:, None], out[rows, last_col], states[:, j])
        pos[:, j] = torch.where(has, self.positions[rows, last_col], pos[:, j])
        return new


@register_technique
class LoRADropTechnique(DepthTechnique):
    config_class = LoRADropConfig
    objective_name = "loradrop"

    def __init__(self, config: LoRADropConfig, model) -> None:
        super().__init__(config, model)
        h = model.config.hidden_size
        with torch.random.fork_rng(devices=[]):
            torch.manual_seed(0)
            self.updates = nn.ModuleDict({str(i): LoRAUpdate(h, config.rank, config.alpha)
                                          for i in self.layer_ids}).to(model.device)

    def make_policy(self):
        return LoRADropPolicy(self, self.layer_ids, self.config.phases())


def redundant_layers(model, batches, count: int) -> list[int]:
    """The ``count`` layers (1-indexed) whose input and output are most alike (mean cosine similarity) on
    ``batches``: the natural droppable set."""
    from .._self_draft import block_influence

    influence = block_influence(model, batches)  # 1 - cos
    return sorted(int(i) + 1 for i in influence.argsort()[:count])


# ---- CALM ------------------------------------------------------------------------------------------------------
@dataclass(frozen=True)
class CalmConfig(LayeredDepthConfig):
    technique: ClassVar[str] = "calm"
    confidence: str = "softmax"
    threshold: float = 0.9
    min_layer: int = 1
    decay_temperature: float = 0.0
    decay_horizon: int = 256

    def __post_init__(self) -> None:
        super().__post_init__()
        check_choice("confidence", self.confidence, CONFIDENCE_MEASURES)
        check_unit_interval("threshold", self.threshold, closed_high=True)
        check_positive("min_layer", self.min_layer)
        check_non_negative("decay_temperature", self.decay_temperature)
        check_positive("decay_horizon", self.decay_horizon)

    def validate(self, model) -> None:
        super().validate(model)
        if self.min_layer >= model.config.num_layers:
            raise ConfigError(f"min_layer must be below the number of layers ({model.config.num_layers})")

    def threshold_at(self, generated: torch.Tensor) -> torch.Tensor:
        if self.decay_temperature == 0:
            return torch.full(generated.shape, self.threshold, device=generated.device)
        decay = torch.exp(-self.decay_temperature * generated.float().clamp_min(0) / self.decay_horizon)
        return (0.9 * self.threshold + 0.1 * decay).clamp(0.0, 1.0)


class CalmPolicy(DepthPolicy):
    def begin_pass(self, batch, h):
        super().begin_pass(batch, h)
        self.exited = torch.zeros_like(self.valid)
        self._thr = self.technique.config.threshold_at(self.generated())

    def choose(self, index, x, out):
        return ~self.exited

    def apply(self, index, x, out, run):
        new = torch.where(run[..., None], out, x)
        cfg = self.technique.config
        n = self.technique.model.config.num_layers
        if cfg.min_layer - 1 <= index < n - 1:
            conf = self.technique.confidence(index, x, new)
            self.exited = self.exited | ((conf > self._thr) & self.valid)
        return new


class ExitClassifier(ScalarScore):
    """``sigmoid(w . rms(h) + b)``, one classifier shared by all exit layers (starts at 0.5)."""

    def __init__(self, hidden: int) -> None:
        super().__init__(hidden, 0.0, 0.0, "rms")


@register_technique
class CalmTechnique(DepthTechnique):
    config_class = CalmConfig
    objective_name = "calm"

    def __init__(self, config: CalmConfig, model) -> None:
        super().__init__(config, model)
        self.layer_ids = list(range(model.config.num_layers))
        self.classifier = ExitClassifier(model.config.hidden_size).to(model.device) \
            if config.confidence == "classifier" else None

    def confidence(self, index: int, x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        kind = self.config.confidence
        if kind == "state":
            return F.cosine_similarity(out.float(), x.float(), dim=-1).clamp(-1.0, 1.0)
        if kind == "classifier":
            return torch.sigmoid(self.classifier.logit(out))
        from ... import ops

        model = self.model
        h = ops.rmsnorm(out.to(model.dtype), model.norm, model.config.rms_norm_eps)[0]
        probs = F.softmax(model.logits(h).float(), dim=-1)
        top = probs.topk(2, dim=-1).values
        return top[..., 0] - top[..., 1]

    def make_policy(self):
        return CalmPolicy(self, self.layer_ids, self.config.phases())
