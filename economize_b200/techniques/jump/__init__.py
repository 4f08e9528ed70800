"""Cross-layer jump drafting (``jump``; economize ``techniques/jump``). Between two exact passes each draft token
skips the target's layers ``1 .. m`` (and ``r + 1 .. L``): a predictor maps the previous token's state after layer
``u`` and the new token's embedding to the new token's state after layer ``m``, and only the target's layers
``m + 1 .. r`` run, against the target's own cache (the committed K/V of those layers are exact; the drafts write
theirs into the scratch slots past the committed length, which the verification pass overwrites). The exit reads
through the final norm and LM head. The target verifies (lossless).

The objective ``jump_rollout`` fits the predictor by teacher forcing: from the target's own states after layer
``u`` at ``t`` and the embedding of token ``t + 1`` to the state after layer ``m`` at ``t + 1`` (normalised squared
error); economize's open-loop rollouts, source mixers and RL pieces are not built.
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
from ...train.objective import OBJECTIVES, Objective, OptimDefaults
from ...validation import check_choice, check_positive

__all__ = ["JumpConfig", "JumpDrafter", "JumpPredictor", "JumpTechnique"]


@dataclass(frozen=True)
class JumpConfig(TechniqueConfig):
    """``target_layer`` ``m`` and ``source_layer`` ``u`` (1-indexed, ``m <= u``); ``exit_layer`` ``r`` (``None``:
    the last layer); ``predictor``: ``"mlp"``; ``width``: the predictor's inner width multiple of the hidden size;
    ``source_layers``: several sources in ``m .. r`` combined by ``mixer`` (``"concat"``, ``"linear"``,
    ``"attention"``) instead of the one ``source_layer``."""

    technique: ClassVar[str] = "jump"
    target_layer: int | None = None
    source_layer: int | None = None
    exit_layer: int | None = None
    predictor: str = "mlp"
    width: float = 1.0
    param_dtype: str = "float32"
    source_layers: tuple[int, ...] = ()
    mixer: str = "concat"

    def __post_init__(self) -> None:
        check_choice("predictor", self.predictor, ("mlp",))
        check_choice("mixer", self.mixer, MIXERS)
        object.__setattr__(self, "source_layers", tuple(sorted({int(u) for u in self.source_layers})))
        check_positive("width", self.width)
        check_choice("param_dtype", self.param_dtype, ("float32", "model"))

    def resolved(self, num_layers: int) -> tuple[int, int, int]:
        m = self.target_layer or max(1, num_layers // 3)
        u = self.source_layer or max(m, (num_layers * 9) // 16)
        r = self.exit_layer or num_layers
        return m, u, r

    def sources(self, num_layers: int) -> tuple[int, ...]:
        """The source layers (``source_layers``, else the one ``source_layer``)."""
        return self.source_layers or (self.resolved(num_layers)[1],)

    def validate(self, model) -> None:
        n = model.config.num_layers
        m, u, r = self.resolved(n)
        if not 1 <= m <= u <= r <= n or m >= r:
            raise ConfigError(f"jump needs 1 <= target_layer <= source_layer <= exit_layer <= {n} and "
                              f"target_layer < exit_layer, got {(m, u, r)}")
        if any(not m <= v <= r for v in self.sources(n)):
            raise ConfigError(f"source_layers must lie in target_layer .. exit_layer ({m} .. {r}): the drafter's "
                              f"partial pass produces only those states, got {self.sources(n)}")


#: source mixers (several source layers -> one predictor source; economize ``techniques/jump/mixer.py``):
#: ``concat``: a linear map of the concatenated states (starts as the last source); ``linear``: a learned convex
#: combination of the states (starts on the last); ``attention``: per-token softmax weights from a learned query
#: against the RMS-normalized states.
MIXERS = ("concat", "linear", "attention")


class SourceMixer(nn.Module):
    def __init__(self, kind: str, n: int, hidden: int) -> None:
        super().__init__()
        self.kind, self.n = kind, n
        if kind == "concat" and n > 1:
            self.proj = nn.Linear(n * hidden, hidden, bias=False)
            with torch.no_grad():
                self.proj.weight.zero_()
                self.proj.weight[:, (n - 1) * hidden:].copy_(torch.eye(hidden))
        elif kind == "linear":
            init = torch.full((n,), -8.0)
            init[-1] = 8.0
            self.logits = nn.Parameter(init)
        elif kind == "attention":
            self.query = nn.Parameter(torch.zeros(hidden))

    def forward(self, states: torch.Tensor) -> torch.Tensor:
        """``states [..., n, H]`` (ascending layers) -> ``[..., H]``."""
        if self.n == 1:
            return states[..., 0, :]
        x = states.float()
        if self.kind == "concat":
            return self.proj(x.flatten(-2).to(self.proj.weight.dtype))
        if self.kind == "linear":
            w = torch.softmax(self.logits.float(), 0)
        else:
            normed = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6)
            w = torch.softmax((normed * self.query.float()).sum(-1), -1)[..., None]
            return (w * x).sum(-2)
        return (w[:, None] * x).sum(-2)


class JumpPredictor(nn.Module):
    """``e + W2 silu(W1 [s_u; e])``: starts as the embedding itself."""

    def __init__(self, hidden: int, width: int) -> None:
        super().__init__()
        self.w1 = nn.Linear(2 * hidden, width)
        self.w2 = nn.Linear(width, hidden)
        nn.init.zeros_(self.w2.weight)
        nn.init.zeros_(self.w2.bias)

    def forward(self, source: torch.Tensor, emb: torch.Tensor) -> torch.Tensor:
        dt = self.w1.weight.dtype
        e = emb.to(dt)
        return e + self.w2(F.silu(self.w1(torch.cat([source.to(dt), e], -1))))


class JumpDrafter:
    def __init__(self, tech: JumpTechnique) -> None:
        self.tech = tech
        self.m, self.u, self.r = tech.layers
        self.capture_layers = tech.sources
        self.carry_size = tech.model.config.hidden_size
        self.cache = None

    def begin(self, batch: int, capacity: int) -> None:
        pass

    def bind_target_cache(self, cache) -> None:
        self.cache = cache

    def fuse(self, aux):
        return self.tech.mix(aux).to(self.tech.model.dtype)

    def _run(self, tokens, states, batch: StepBatch):
        tech = self.tech
        model = tech.model
        h_m = tech.predictor(states, model.embed_tokens(tokens.clamp_min(0))).to(model.dtype)
        cap = tuple(-2 if v == self.r else v for v in tech.sources)  # the last run layer's output is -2
        out, aux = model.forward_step(tokens.clamp_min(0), batch, self.cache, capture=cap,
                                      layers=range(self.m, self.r), hidden=h_m)
        nxt = tech.mix(aux, cap).to(model.dtype)
        return model.logits(out).float(), nxt

    def observe(self, tokens, sources, kv_len, n_valid, root):
        b = tokens.shape[0]
        rows = torch.arange(b, device=tokens.device)
        r = root.long()
        slot = (kv_len + root).to(torch.int32)
        one = torch.ones(b, dtype=torch.int32, device=tokens.device)
        logits, nxt = self._run(tokens[rows, r][:, None], sources[rows, r][:, None],
                                StepBatch(slot, one, slot[:, None].contiguous()))
        return logits[:, 0], nxt[:, 0]

    def tree_step(self, tokens, states, positions, kv_base, n_forwarded, q_offset, mask):
        batch = tokens.shape[0]
        n_new = torch.full((batch,), n_forwarded, dtype=torch.int32, device=tokens.device)
        return self._run(tokens, states, StepBatch(kv_base.to(torch.int32), n_new, positions.to(torch.int32), mask,
                                                   q_offset))

    def to_target(self, ids):
        return ids


@register_technique
class JumpTechnique(Technique):
    config_class = JumpConfig
    capabilities = Capability.DRAFTER
    family = Family.DRAFTER
    lossless = True
    objective_name = "jump_rollout"

    def __init__(self, config: JumpConfig, model) -> None:
        super().__init__(config, model)
        h = model.config.hidden_size
        self.layers = config.resolved(model.config.num_layers)
        dtype = torch.float32 if config.param_dtype == "float32" else model.dtype
        self.predictor = JumpPredictor(h, max(8, int(config.width * h))).to(device=model.device, dtype=dtype)
        self.sources = config.sources(model.config.num_layers)
        self.mixer = SourceMixer(config.mixer, len(self.sources), h).to(device=model.device, dtype=dtype)

    def mix(self, aux: dict[int, torch.Tensor], keys: tuple[int, ...] | None = None) -> torch.Tensor:
        """The predictor's source from captured states ``aux`` (``keys``: their capture indices, default the
        source layers)."""
        keys = keys or self.sources
        return self.mixer(torch.stack([aux[k] for k in keys], -2))

    def drafter(self):
        return JumpDrafter(self)

    def default_decoding(self) -> DecodeConfig:
        return DecodeConfig(cycle_length=5)


@OBJECTIVES.register("jump_rollout")
class JumpRollout(Objective):
    """``horizon=1``: normalised squared error between the predicted and the target's state after layer ``m`` at
    ``t + 1``, from the target's own sources (teacher forcing). ``horizon > 1``: open-loop rollouts
    (:func:`~.rollout.rollout_steps`): step ``j`` of the rollout from every start ``p`` predicts position ``p + j``
    from the states the drafter itself produced at step ``j - 1``; each step's loss is the state error against the
    target's state after layer ``m`` at ``p + j`` plus ``ce_weight`` times the cross-entropy of the step's logits
    against the target's greedy token after ``p + j``, and step ``j`` weighs ``decay**(j - 1)``."""

    name = "jump_rollout"
    defaults = OptimDefaults(lr=1e-3, warmup_steps=0)

    def __init__(self, model, horizon: int = 1, ce_weight: float = 1.0, decay: float = 0.8) -> None:
        super().__init__(model)
        if "jump" not in model.techniques:
            raise ConfigError("jump_rollout needs an attached jump technique")
        check_positive("horizon", horizon)
        if ce_weight < 0 or not 0 < decay <= 1:
            raise ConfigError(f"jump_rollout needs ce_weight >= 0 and 0 < decay <= 1, got {ce_weight}, {decay}")
        self.tech = model.techniques["jump"]
        self.horizon, self.ce_weight, self.decay = int(horizon), float(ce_weight), float(decay)

    def parameters(self):
        return list(self.tech.predictor.parameters()) + list(self.tech.mixer.parameters())

    def loss(self, tokens: torch.Tensor):
        tech = self.tech
        model = tech.model
        m, _, r = tech.layers
        b, s = tokens.shape
        capture = (m, *tech.sources) if self.horizon == 1 else tuple(sorted({*range(m, r + 1), *tech.sources}))
        with torch.no_grad():
            cache = model.new_cache(b, ((s + 127) // 128) * 128)
            lengths = torch.full((b,), s, dtype=torch.int32, device=tokens.device)
            final, aux = model.forward_step(tokens, StepBatch.prefill(lengths, s), cache, capture=capture)
            emb = model.embed_tokens(tokens)
        if self.horizon == 1:
            pred = tech.predictor(tech.mix(aux)[:, :-1].float(), emb[:, 1:].float())
            target = aux[m][:, 1:].float()
            err = (pred.float() - target).pow(2).sum(-1) / target.pow(2).sum(-1).clamp_min(1e-6)
            loss = err.mean()
            return loss, {"loss": float(loss.detach())}
        from ...ops import reference
        from ...train.objective import dense_linear
        from .rollout import rollout_steps

        with torch.no_grad():
            labels = model.logits(final).argmax(-1)  # the target's greedy token after every position
        starts, steps = rollout_steps(tech, tokens, aux, self.horizon)
        total, weight, stats = 0.0, 0.0, {}
        for j, (h_m, h_r) in enumerate(steps, start=1):
            pos = starts + j
            target = aux[m][:, pos].float()
            err = ((h_m.float() - target).pow(2).sum(-1) / target.pow(2).sum(-1).clamp_min(1e-6)).mean()
            step_loss = err
            if self.ce_weight:
                x = reference.rmsnorm(h_r, model.norm, model.config.rms_norm_eps)[0]
                logits = dense_linear(x, model.head_weight, None).float() / model.config.logits_scaling
                ce = F.cross_entropy(logits.reshape(-1, logits.shape[-1]), labels[:, pos].reshape(-1))
                step_loss = step_loss + self.ce_weight * ce
                stats[f"ce_{j}"] = float(ce.detach())
            w = self.decay ** (j - 1)
            total = total + w * step_loss
            weight += w
            stats[f"state_{j}"] = float(err.detach())
        loss = total / weight
        stats["loss"] = float(loss.detach())
        return loss, stats
