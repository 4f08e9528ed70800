"""Gated-MLP channel sparsity: CATS (``cats``; Lee et al., "CATS: Contextually-Aware Thresholding for Sparsity in
Large Language Models", COLM 2024) and Deja Vu (``dejavu``; Liu et al., "Deja Vu: Contextual Sparsity for Efficient
LLMs at Inference Time", ICML 2023), economize ``techniques/mlp_sparsity``.

Both skip FFN channels of ``down(silu(gate(x)) * up(x))`` per token:

* CATS keeps channel ``c`` when ``|silu(gate(x))_c| > t``, with ``t`` the ``sparsity`` quantile of those
  magnitudes on calibration text; the gate stays dense.
* Deja Vu keeps the ``1 - sparsity`` fraction of channels with the largest scores of a per-layer low-rank
  predictor ``Linear(d, rank) -> Linear(rank, ffn)`` (no bias, no nonlinearity), fitted on labels = the top
  channels of ``|silu(gate(x)) * up(x)|`` and trainable with the objective ``dejavu``. ``predictor_input``
  ``"lookahead"`` reads the layer's attention input instead of the MLP input (the paper's asynchronous predictor).

Decoding steps (at most 16 rows) run ``glu_rows`` (only the up, or gate and up, rows of kept channels are read)
and a column-sparse down projection over the exact zeros of its input (``colsparse_linear`` on the transposed
down weight), both in ``csrc/act_sparse.cu``.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import ClassVar

import torch
import torch.nn.functional as F
from torch import nn

from ...core.technique import Capability, Family, Simulation, Technique, TechniqueConfig, register_technique
from ...errors import ConfigError
from ...ops.act_sparse import (PhasePolicy, TransposedWeight, cats_mlp, kept_channels, kept_mlp, magnitude_quantile,
                               second_half_mask, tokens_per_sequence, topk_mask)
from ...ops.quant import install
from ...runtime.cache import StepBatch
from ...runtime.phase import current_phase
from ...validation import check_choice, check_non_negative, check_positive, check_unit_interval
from ..sparsity import MagnitudeSamples

__all__ = ["MLP_SPARSITY_BACKENDS", "PREDICTOR_DTYPES", "PREDICTOR_INPUTS", "CatsConfig", "CatsTechnique",
           "DejaVuConfig", "DejaVuTechnique", "dejavu_labels", "fit_predictor"]

MLP_SPARSITY_BACKENDS = ("auto", "cuda", "dense")
PREDICTOR_INPUTS = ("mlp", "lookahead")
PREDICTOR_DTYPES = ("float32", "bfloat16", "float16")


@dataclass(frozen=True)
class MlpSparsityConfig(TechniqueConfig):
    """Fields shared by ``cats`` and ``dejavu``.

    Args:
        sparsity: Fraction of FFN channels skipped per token.
        prefill: Phase policy as for TEAL (:class:`~economize_b200.ops.act_sparse.PhasePolicy`, a mapping of its
            fields, or the mode string of the exact passes).
        backend: ``"auto"`` (CUDA kernels; ConfigError where they cannot serve a layer), ``"cuda"`` (kernels with
            the masked dense MLP where they cannot) or ``"dense"`` (masked dense MLP: a simulation).
        layers: 1-indexed layers; empty means all.
        mlp, gate, up, down, act: Attribute names of economize's Hugging Face adapters; the engine's layers have one
            fused ``[gate; up]`` weight and SiLU, so these are accepted for configuration compatibility only.
    """

    technique: ClassVar[str] = ""
    sparsity: float = 0.5
    prefill: object = "dense"
    backend: str = "auto"
    layers: tuple[int, ...] = ()
    mlp: str = "mlp"
    gate: str = "gate_proj"
    up: str = "up_proj"
    down: str = "down_proj"
    act: str = "act_fn"

    def __post_init__(self) -> None:
        check_unit_interval("sparsity", self.sparsity, closed_low=True)
        if self.backend == "triton":
            raise ConfigError("backend 'triton' is economize's Triton kernel; this build's kernels are CUDA: use "
                              "backend='auto' or 'cuda'")
        check_choice("backend", self.backend, MLP_SPARSITY_BACKENDS)
        policy = PhasePolicy.coerce(self.prefill)
        if not isinstance(self.prefill, str):
            object.__setattr__(self, "prefill", policy)
        object.__setattr__(self, "layers", tuple(self.layers))

    @property
    def policy(self) -> PhasePolicy:
        return PhasePolicy.coerce(self.prefill)

    def to_dict(self):
        data = super().to_dict()
        if not isinstance(self.prefill, str):
            data["prefill"] = self.policy.to_dict()
        return data

    def validate(self, model) -> None:
        n = model.config.num_layers
        if any(not 1 <= i <= n for i in self.layers):
            raise ConfigError(f"layers must be 1-indexed layers of the model's {n}, got {self.layers}")
        if model.config.is_moe:
            raise ConfigError(f"{self.technique} sparsifies dense gated MLPs; the model's MLPs are mixtures of experts")


@dataclass(frozen=True)
class CatsConfig(MlpSparsityConfig):
    """CATS (see the module docstring). ``max_samples``: magnitudes kept per layer for the threshold;
    ``offload``: keep them on the CPU."""

    technique: ClassVar[str] = "cats"
    max_samples: int = 1 << 20
    offload: bool = False

    def __post_init__(self) -> None:
        super().__post_init__()
        check_positive("max_samples", self.max_samples)


@dataclass(frozen=True)
class DejaVuConfig(MlpSparsityConfig):
    """Deja Vu (see the module docstring).

    Args:
        rank: Inner width of each predictor.
        predictor_input: ``"mlp"`` or ``"lookahead"``.
        lookahead_norm: Accepted for configuration compatibility (the lookahead source is the attention input).
        predictor_dtype: Storage dtype of the predictors.
        fit_steps: Adam steps per layer of the attach-time fit (0: none).
        fit_lr, fit_batch: Learning rate and tokens per step of that fit.
        max_tokens: Calibration tokens kept per layer for the fit.
        seed: Seed of the predictor initialisation and the token subsample.
        offload: Keep the fit's activations on the CPU.
    """

    technique: ClassVar[str] = "dejavu"
    rank: int = 1000
    predictor_input: str = "mlp"
    lookahead_norm: str = "input_layernorm"
    predictor_dtype: str = "float32"
    fit_steps: int = 200
    fit_lr: float = 1e-3
    fit_batch: int = 1024
    max_tokens: int = 65536
    seed: int = 0
    offload: bool = False

    def __post_init__(self) -> None:
        super().__post_init__()
        check_positive("rank", self.rank)
        check_choice("predictor_input", self.predictor_input, PREDICTOR_INPUTS)
        check_choice("predictor_dtype", self.predictor_dtype, PREDICTOR_DTYPES)
        check_non_negative("fit_steps", self.fit_steps)
        check_positive("fit_lr", self.fit_lr)
        check_positive("fit_batch", self.fit_batch)
        check_positive("max_tokens", self.max_tokens)


def _batches(cal) -> list[torch.Tensor]:
    if cal is None:
        return []
    out = [cal] if isinstance(cal, torch.Tensor) else list(cal)
    return [b[None] if b.dim() == 1 else b for b in out]


def _eligible(w) -> str | None:
    if not isinstance(w, torch.Tensor) or w.dim() != 2:
        return f"a {type(w).__name__} weight"
    if not w.is_cuda:
        return f"a weight on {w.device.type}"
    if w.dtype != torch.bfloat16:
        return f"a {str(w.dtype).removeprefix('torch.')} weight"
    return None


class _MlpSparsityBase(Technique):
    """Installs a per-layer MLP rule (``layer.mlp_rule``) and, with the kernels, the transposed down weights."""

    capabilities = Capability.ACTIVATIONS
    family = Family.SPARSITY
    lossless = False

    def __init__(self, config, model) -> None:
        super().__init__(config, model)
        n = model.config.num_layers
        self.layer_ids = [i - 1 for i in config.layers] if config.layers else list(range(n))
        self._calibration = None
        self._installed: list[tuple[nn.Module, object, bool]] = []
        self.masked: list[int] = []

    def calibrate(self, calibration) -> None:
        self._calibration = calibration

    def _rule(self, li: int, kernel: bool):
        raise NotImplementedError

    def install(self) -> None:
        self.detach()
        cfg = self.config
        self.masked = []
        for li, i in enumerate(self.layer_ids):
            layer = self.model.layers[i]
            if layer.down_hadamard:
                self.detach()
                raise ConfigError(f"{self.name}: layer {i + 1}'s down projection reads an online-rotated input "
                                  "(rotate with online=()) and the sparse MLP kernels compute it unrotated")
            reason = _eligible(layer.w_gate_up) or _eligible(layer.w_down)
            if cfg.backend == "auto" and reason is not None:
                self.detach()
                raise ConfigError(f"{self.name} backend 'auto': layer {i + 1} has {reason}; use backend='dense' "
                                  "to simulate the saving")
            kernel = cfg.backend != "dense" and reason is None
            if cfg.backend == "cuda" and not kernel:
                self.masked.append(i + 1)
            down = layer.w_down
            was_param = isinstance(down, nn.Parameter)
            if kernel:
                install(layer, "w_down", TransposedWeight(down))
            layer.mlp_rule = self._rule(li, kernel)
            self._installed.append((layer, down if kernel else None, was_param))

    def detach(self) -> None:
        for layer, down, was_param in reversed(self._installed):
            layer.mlp_rule = None
            if down is not None:
                w = layer.w_down.restore()
                install(layer, "w_down", nn.Parameter(w, requires_grad=False) if was_param else w)
        self._installed = []

    def simulation(self) -> Simulation | None:
        if self.config.backend == "dense":
            return Simulation("FFN weight reads", "backend='dense' masks channels of the dense MLP")
        if self.masked:
            return Simulation("FFN weight reads", f"layers {self.masked[:8]} run the masked dense MLP")
        return None


@register_technique
class CatsTechnique(_MlpSparsityBase):
    """CATS: the thresholds are the buffer ``thresholds`` (one per selected layer), saved with the technique."""

    config_class = CatsConfig

    def __init__(self, config: CatsConfig, model) -> None:
        super().__init__(config, model)
        self.register_buffer("thresholds", torch.full((len(self.layer_ids),), math.nan, device=model.device))

    @property
    def calibrated(self) -> bool:
        return bool(torch.isfinite(self.thresholds).all())

    @torch.no_grad()
    def _calibrate(self) -> None:
        model, cfg = self.model, self.config
        batches = _batches(self._calibration)
        if not batches:
            raise ConfigError("cats needs calibration tokens (apply(..., calibration=ids)) or a saved state")
        samples = {i: MagnitudeSamples(cfg.max_samples, i, cfg.offload) for i in self.layer_ids}

        def observer(layer: int, name: str, x: torch.Tensor) -> None:
            if name == "w_gate_up" and layer in samples:
                w = model.layers[layer].w_gate_up
                f = w.shape[0] // 2
                samples[layer].update(F.silu(F.linear(x, w[:f])))

        model.observer = observer
        try:
            for tokens in batches:
                tokens = tokens.to(model.device)
                b, s = tokens.shape
                cache = model.new_cache(b, ((s + 127) // 128) * 128)
                lengths = torch.full((b,), s, dtype=torch.int32, device=model.device)
                model.forward_step(tokens, StepBatch.prefill(lengths, s), cache)
        finally:
            model.observer = None
        for li, i in enumerate(self.layer_ids):
            self.thresholds[li] = magnitude_quantile(samples[i].sorted(), cfg.sparsity)

    def attach(self) -> None:
        self.detach()
        if not self.calibrated:
            self._calibrate()
        self.install()

    def _rule(self, li: int, kernel: bool):
        policy = self.config.policy
        threshold = self.thresholds[li:li + 1].reshape(())  # a view: a state load updates it in place

        def rule(model, layer, x, index):
            mode = policy.mode(current_phase(), tokens_per_sequence(x))
            if mode == "dense":
                return None
            return cats_mlp(layer.w_gate_up, layer.w_down, x, threshold, mode, kernel)

        return rule

    def threshold_map(self) -> dict[int, float]:
        return {i + 1: float(t) for i, t in zip(self.layer_ids, self.thresholds.tolist())}


@torch.no_grad()
def dejavu_labels(w_gate_up: torch.Tensor, x: torch.Tensor, k: int, chunk: int = 4096) -> torch.Tensor:
    """The ``k`` channels with the largest ``|silu(gate(x)) * up(x)|`` per token (boolean ``[..., ffn]``), computed
    ``chunk`` tokens at a time."""
    flat = x.reshape(-1, x.shape[-1])
    out = []
    for part in flat.split(chunk):
        g, u = F.linear(part, w_gate_up.to(part.dtype)).chunk(2, -1)
        out.append(topk_mask((F.silu(g) * u).abs().float(), k))
    return torch.cat(out).reshape(*x.shape[:-1], -1)


def fit_predictor(predictor: nn.Module, sources: torch.Tensor, labels: torch.Tensor, *, steps: int, lr: float,
                  batch: int, seed: int) -> float:
    """Adam on the binary cross-entropy of the predictor's scores against ``labels [n, ffn]`` (fp32 training,
    stored back in the predictor's dtype); returns the last loss."""
    dtype = next(predictor.parameters()).dtype
    predictor.float()
    opt = torch.optim.Adam(predictor.parameters(), lr=lr)
    gen = torch.Generator().manual_seed(seed)
    n, last = sources.shape[0], math.nan
    with torch.enable_grad():
        for _ in range(steps):
            idx = torch.randint(n, (min(batch, n),), generator=gen).to(sources.device)
            scores = predictor(sources[idx].float())
            loss = F.binary_cross_entropy_with_logits(scores, labels[idx].to(scores.dtype))
            opt.zero_grad(set_to_none=True)
            loss.backward()
            opt.step()
            last = float(loss.detach())
    predictor.to(dtype)
    return last


@register_technique
class DejaVuTechnique(_MlpSparsityBase):
    """Deja Vu: ``predictors[str(layer)]`` (1-indexed layer) and the buffer ``fitted`` are the technique's state."""

    config_class = DejaVuConfig
    objective_name = "dejavu"

    def __init__(self, config: DejaVuConfig, model) -> None:
        super().__init__(config, model)
        c = model.config
        self.k = kept_channels(c.intermediate_size, config.sparsity)
        dtype = getattr(torch, config.predictor_dtype)
        preds = nn.ModuleDict()
        with torch.random.fork_rng(devices=[]):
            torch.manual_seed(config.seed)
            for i in self.layer_ids:
                preds[str(i + 1)] = nn.Sequential(nn.Linear(c.hidden_size, config.rank, bias=False),
                                                  nn.Linear(config.rank, c.intermediate_size, bias=False)
                                                  ).to(device=model.device, dtype=dtype)
        self.predictors = preds
        self.register_buffer("fitted", torch.zeros((), dtype=torch.bool, device=model.device))
        self._lookahead: dict[int, torch.Tensor] = {}

    def predict(self, index: int, source: torch.Tensor) -> torch.Tensor:
        p = self.predictors[str(index + 1)]
        return p(source.to(p[0].weight.dtype))

    @torch.no_grad()
    def _collect(self, batches: list[torch.Tensor]) -> dict[int, tuple[torch.Tensor, torch.Tensor]]:
        """Per layer: (predictor sources, MLP inputs) of the calibration tokens, at most ``max_tokens`` of each."""
        model, cfg = self.model, self.config
        src: dict[int, list[torch.Tensor]] = {i: [] for i in self.layer_ids}
        mlp_in: dict[int, list[torch.Tensor]] = {i: [] for i in self.layer_ids}

        def keep(t: torch.Tensor) -> torch.Tensor:
            t = t.reshape(-1, t.shape[-1])
            return t.cpu() if cfg.offload else t

        def observer(layer: int, name: str, x: torch.Tensor) -> None:
            if layer not in src:
                return
            if name == "wqkv" and cfg.predictor_input == "lookahead":
                src[layer].append(keep(x))
            if name == "w_gate_up":
                mlp_in[layer].append(keep(x))
                if cfg.predictor_input == "mlp":
                    src[layer].append(keep(x))

        model.observer = observer
        try:
            for tokens in batches:
                tokens = tokens.to(model.device)
                b, s = tokens.shape
                cache = model.new_cache(b, ((s + 127) // 128) * 128)
                lengths = torch.full((b,), s, dtype=torch.int32, device=model.device)
                model.forward_step(tokens, StepBatch.prefill(lengths, s), cache)
        finally:
            model.observer = None
        gen = torch.Generator().manual_seed(cfg.seed)
        out = {}
        for i in self.layer_ids:
            a, m = torch.cat(src[i]), torch.cat(mlp_in[i])
            if a.shape[0] > cfg.max_tokens:
                sel = torch.randperm(a.shape[0], generator=gen)[: cfg.max_tokens].to(a.device)
                a, m = a[sel], m[sel]
            out[i] = (a, m)
        return out

    def _fit(self) -> None:
        cfg = self.config
        batches = _batches(self._calibration)
        if cfg.fit_steps == 0 or not batches:
            return
        dev = self.model.device
        for i, (a, m) in self._collect(batches).items():
            labels = dejavu_labels(self.model.layers[i].w_gate_up, m.to(dev), self.k)
            fit_predictor(self.predictors[str(i + 1)], a.to(dev), labels, steps=cfg.fit_steps, lr=cfg.fit_lr,
                          batch=cfg.fit_batch, seed=cfg.seed + i)
        self.fitted.fill_(True)

    def attach(self) -> None:
        self.detach()
        if not bool(self.fitted):
            self._fit()
        self.install()

    def install(self) -> None:
        super().install()
        if self.config.predictor_input == "lookahead":
            for i in self.layer_ids:
                self.model.layers[i].attn_input_hook = self._store_lookahead(i)

    def detach(self) -> None:
        for i in self.layer_ids:
            if getattr(self.model.layers[i], "attn_input_hook", None) is not None:
                self.model.layers[i].attn_input_hook = None
        super().detach()

    def _store_lookahead(self, index: int):
        def hook(x: torch.Tensor) -> None:
            self._lookahead[index] = x

        return hook

    def _rule(self, li: int, kernel: bool):
        policy = self.config.policy
        index = self.layer_ids[li]
        lookahead = self.config.predictor_input == "lookahead"

        def rule(model, layer, x, _index):
            mode = policy.mode(current_phase(), tokens_per_sequence(x))
            if mode == "dense":
                return None
            source = self._lookahead.get(index, x) if lookahead else x
            keep = topk_mask(self.predict(index, source), self.k)
            if mode == "second_half":
                keep = second_half_mask(keep)
            return kept_mlp(layer.w_gate_up, layer.w_down, x, keep, kernel)

        return rule


def _objective():
    from ...train.objective import OBJECTIVES, Objective, OptimDefaults

    @OBJECTIVES.register("dejavu")
    class DejaVuObjective(Objective):
        """Binary cross-entropy of every Deja Vu predictor against the channels the dense MLP would keep for the
        batch's tokens (the labels of :func:`dejavu_labels`)."""

        name = "dejavu"
        defaults = OptimDefaults(lr=1e-3, warmup_steps=0, grad_clip=None)

        def __init__(self, model) -> None:
            super().__init__(model)
            if "dejavu" not in model.techniques:
                raise ConfigError("the dejavu objective needs an attached dejavu technique")
            self.tech = model.techniques["dejavu"]

        def parameters(self) -> list[torch.nn.Parameter]:
            return [p for p in self.tech.predictors.parameters()]

        def loss(self, tokens: torch.Tensor) -> tuple[torch.Tensor, dict[str, float]]:
            tech = self.tech
            layers = tech.model.layers
            rules = {i: getattr(layers[i], "mlp_rule", None) for i in tech.layer_ids}
            for i in rules:  # labels and sources come from the dense MLPs
                layers[i].mlp_rule = None
            try:
                data = tech._collect([tokens])
            finally:
                for i, r in rules.items():
                    layers[i].mlp_rule = r
            total, metrics = 0.0, {}
            for i, (a, m) in data.items():
                labels = dejavu_labels(layers[i].w_gate_up, m, tech.k)
                p = tech.predictors[str(i + 1)]
                scores = p(a.to(p[0].weight.dtype)).float()
                total = total + F.binary_cross_entropy_with_logits(scores, labels.float())
            loss = total / max(len(data), 1)
            metrics["loss"] = float(loss.detach())
            return loss, metrics

    return DejaVuObjective


DejaVuObjective = _objective()
