"""TEAL: training-free magnitude activation sparsity on the inputs of every linear map (``teal``; economize
``techniques/sparsity``, Liu et al., "Training-Free Activation Sparsity in Large Language Models", ICLR 2025).

Each map's input entries with ``|x| <= t`` are zeroed; the threshold ``t`` of a map is the quantile of the dense
model's input magnitudes on calibration text at the map's sparsity level, and the levels come from TEAL's greedy
search (each layer reaches the target parameter-weighted sparsity with the lowest layer-output error) or are
uniform. Decoding steps run ``colsparse_linear`` (``csrc/act_sparse.cu``): the weights are stored transposed and
only the weight rows of kept inputs are read, so a step reads about ``1 - sparsity`` of the weight bytes.

The engine's fused projections share one input per group, so they share one level here: ``wqkv`` (q, k, v) and
``w_gate_up`` (gate, up); TEAL's search over the separate maps of a Hugging Face layer gives them equal thresholds
at equal levels anyway, since their inputs are the same.
"""

from __future__ import annotations

import fnmatch
import math
from dataclasses import dataclass, field
from typing import ClassVar

import torch
from torch import nn

from ...core.technique import Capability, Family, Simulation, Technique, TechniqueConfig, register_technique
from ...errors import ConfigError
from ...ops.act_sparse import (PhasePolicy, TealWeight, greedy_allocation, greedy_error, magnitude_quantile,
                               uniform_allocation)
from ...ops.quant import install
from ...runtime.cache import StepBatch
from ...validation import check_choice, check_non_negative, check_positive, check_unit_interval

__all__ = ["MAPS", "TEAL_ALLOCATIONS", "TEAL_BACKENDS", "MagnitudeSamples", "TealConfig", "TealTechnique",
           "kernel_ineligibility"]

TEAL_ALLOCATIONS = ("greedy", "uniform")
#: ``auto``: the CUDA kernel on every map (ConfigError where it cannot serve one); ``cuda``: the kernel with the
#: masked dense product on maps it cannot serve; ``dense``: the masked dense product everywhere (simulated saving).
TEAL_BACKENDS = ("auto", "cuda", "dense")
#: The engine's projections and the Hugging Face maps each one fuses.
MAPS = {"wqkv": ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj"), "wo": ("self_attn.o_proj",),
        "w_gate_up": ("mlp.gate_proj", "mlp.up_proj"), "w_down": ("mlp.down_proj",)}


def _selected(name: str, targets: tuple[str, ...], exclude: tuple[str, ...]) -> bool:
    names = (name, *MAPS[name], *(n.split(".")[-1] for n in MAPS[name]))

    def hit(pats):
        return any(fnmatch.fnmatchcase(n, p) for n in names for p in pats)

    return hit(targets) and not hit(exclude)


def kernel_ineligibility(weight) -> str | None:
    """Why ``colsparse_linear`` cannot serve ``weight``, or ``None``."""
    if not isinstance(weight, torch.Tensor) or weight.dim() != 2:
        return f"a {type(weight).__name__} weight (quantized or packed)"
    if not weight.is_cuda:
        return f"a weight on {weight.device.type}"
    if weight.dtype != torch.bfloat16:
        return f"a {str(weight.dtype).removeprefix('torch.')} weight (the kernel takes bfloat16)"
    if weight.shape[0] % 8:
        return "an output width that is not a multiple of 8"
    return None


@dataclass(frozen=True)
class TealConfig(TechniqueConfig):
    """Magnitude activation sparsity on the inputs of a decoder layer's linear maps (TEAL).

    Args:
        sparsity: Target layer-level sparsity (parameter-weighted mean fraction of zeroed inputs).
        allocation: ``"greedy"`` (TEAL's block-wise greedy search) or ``"uniform"``.
        greedy_step: Base step of the greedy search (a map with ``hidden_size**2`` parameters moves by this much).
        greedy_fraction: Trailing fraction of positions on which the greedy search measures the layer error.
        greedy_batches: Calibration batches the greedy search evaluates (0: all).
        prefill: A :class:`~economize_b200.ops.act_sparse.PhasePolicy` (or its fields as a mapping), or the mode of
            the exact passes and multi-token calls outside decoding (``"dense"``, ``"second_half"``, ``"all"``).
        backend: ``"auto"``, ``"cuda"`` or ``"dense"`` (:data:`TEAL_BACKENDS`).
        targets: Globs over map names (``"self_attn.*"``, ``"mlp.down_proj"``, ``"q_proj"`` or ``"wqkv"``).
        exclude: Globs removed from ``targets``.
        layers: 1-indexed layers to sparsify; empty means all.
        max_samples: Magnitudes kept per map for the threshold quantiles.
        offload: Keep calibration samples on the CPU.
        seed: Seed of the magnitude subsample.
    """

    technique: ClassVar[str] = "teal"
    sparsity: float = 0.4
    allocation: str = "greedy"
    greedy_step: float = 0.05
    greedy_fraction: float = 0.25
    greedy_batches: int = 0
    prefill: object = "dense"
    backend: str = "auto"
    targets: tuple[str, ...] = ("*",)
    exclude: tuple[str, ...] = ()
    layers: tuple[int, ...] = ()
    max_samples: int = 1 << 20
    offload: bool = False
    seed: int = 0

    def __post_init__(self) -> None:
        check_unit_interval("sparsity", self.sparsity, closed_low=True)
        check_choice("allocation", self.allocation, TEAL_ALLOCATIONS)
        check_unit_interval("greedy_step", self.greedy_step, closed_high=True)
        check_unit_interval("greedy_fraction", self.greedy_fraction, closed_high=True)
        check_non_negative("greedy_batches", self.greedy_batches)
        if self.backend in ("triton", "triton_autotune"):
            raise ConfigError(f"backend {self.backend!r} is the Triton kernel of economize; this build's sparse "
                              "GEMV is CUDA: use backend='auto' or 'cuda'")
        check_choice("backend", self.backend, TEAL_BACKENDS)
        policy = PhasePolicy.coerce(self.prefill)
        if not isinstance(self.prefill, str):
            object.__setattr__(self, "prefill", policy)
        object.__setattr__(self, "targets", tuple(self.targets))
        object.__setattr__(self, "exclude", tuple(self.exclude))
        object.__setattr__(self, "layers", tuple(self.layers))
        check_positive("max_samples", self.max_samples)

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


class MagnitudeSamples:
    """A bounded random subsample of the magnitudes of every tensor it sees."""

    def __init__(self, max_samples: int, seed: int, offload: bool) -> None:
        self.max_samples = max_samples
        self.offload = offload
        self.gen = torch.Generator().manual_seed(seed)
        self.parts: list[torch.Tensor] = []
        self.count = 0

    def update(self, x: torch.Tensor) -> None:
        v = x.detach().abs().float().flatten()
        if self.offload:
            v = v.cpu()
        self.parts.append(v)
        self.count += v.numel()
        if self.count > 2 * self.max_samples:
            self._shrink()

    def _shrink(self) -> None:
        v = torch.cat(self.parts)
        keep = torch.randperm(v.numel(), generator=self.gen)[: self.max_samples].to(v.device)
        self.parts, self.count = [v[keep]], self.max_samples

    def sorted(self) -> torch.Tensor:
        if self.count > self.max_samples:
            self._shrink()
        return torch.cat(self.parts).sort().values if self.parts else torch.zeros(0)


def _batches(cal) -> list[torch.Tensor]:
    if cal is None:
        return []
    out = [cal] if isinstance(cal, torch.Tensor) else list(cal)
    return [b[None] if b.dim() == 1 else b for b in out]


@torch.no_grad()
def run_layer(model, index: int, hidden: torch.Tensor) -> torch.Tensor:
    """The residual stream after block ``index`` for the input stream ``hidden [B, S, H]`` (a causal prefill)."""
    b, s, _ = hidden.shape
    cache = model.new_cache(b, ((s + 127) // 128) * 128)
    lengths = torch.full((b,), s, dtype=torch.int32, device=hidden.device)
    tokens = torch.zeros(b, s, dtype=torch.long, device=hidden.device)
    _, aux = model.forward_step(tokens, StepBatch.prefill(lengths, s), cache, capture=(-2,),
                                layers=range(index, index + 1), hidden=hidden)
    return aux[-2]


@register_technique
class TealTechnique(Technique):
    """TEAL (see :class:`TealConfig`). State: ``thresholds [layers, 4]`` and ``levels [layers, 4]`` (one column per
    engine projection, NaN where a map is not sparsified), so a loaded technique skips calibration."""

    config_class = TealConfig
    capabilities = Capability.ACTIVATIONS
    family = Family.SPARSITY
    lossless = False

    def __init__(self, config: TealConfig, model) -> None:
        super().__init__(config, model)
        n = model.config.num_layers
        self.layer_ids = [i - 1 for i in config.layers] if config.layers else list(range(n))
        self.map_names = [m for m in MAPS if _selected(m, config.targets, config.exclude)]
        if not self.map_names:
            raise ConfigError("teal: targets select no linear map")
        dev = model.device
        self.register_buffer("thresholds", torch.full((len(self.layer_ids), len(MAPS)), math.nan, device=dev))
        self.register_buffer("levels", torch.full((len(self.layer_ids), len(MAPS)), math.nan, device=dev))
        self._calibration = None
        self._installed: list[tuple[nn.Module, str, object, bool]] = []
        self.masked: list[str] = []  # maps the kernel could not serve (backend "cuda")
        self.greedy_paths: dict[int, list] = {}

    def calibrate(self, calibration) -> None:
        self._calibration = calibration

    @property
    def calibrated(self) -> bool:
        cols = [list(MAPS).index(m) for m in self.map_names]
        return bool(torch.isfinite(self.thresholds[:, cols]).all())

    def _maps_of(self, layer) -> list[str]:
        out = []
        for m in self.map_names:
            w = getattr(layer, m)
            if getattr(w, "dim", lambda: 2)() == 3:  # expert weights of a MoE block: not a linear map here
                continue
            out.append(m)
        return out

    # ---- calibration --------------------------------------------------------------------------------------------
    @torch.no_grad()
    def _calibrate(self) -> None:
        model, cfg = self.model, self.config
        batches = _batches(self._calibration)
        if not batches:
            raise ConfigError("teal needs calibration tokens (apply(..., calibration=ids)) or a saved state")
        wanted = {i: self._maps_of(model.layers[i]) for i in self.layer_ids}
        samples = {(i, m): MagnitudeSamples(cfg.max_samples, cfg.seed + 7 * i + j, cfg.offload)
                   for i, maps in wanted.items() for j, m in enumerate(maps)}

        def observer(layer: int, name: str, x: torch.Tensor) -> None:
            s = samples.get((layer, name))
            if s is not None:
                s.update(x)

        greedy = cfg.allocation == "greedy" and cfg.sparsity > 0
        n_eval = len(batches) if cfg.greedy_batches == 0 else min(cfg.greedy_batches, len(batches))
        inputs: dict[int, list[torch.Tensor]] = {i: [] for i in self.layer_ids}
        model.observer = observer
        try:
            for bi, tokens in enumerate(batches):
                tokens = tokens.to(model.device)
                b, s = tokens.shape
                cache = model.new_cache(b, ((s + 127) // 128) * 128)
                lengths = torch.full((b,), s, dtype=torch.int32, device=model.device)
                capture = tuple(self.layer_ids) if greedy and bi < n_eval else ()
                _, aux = model.forward_step(tokens, StepBatch.prefill(lengths, s), cache, capture=capture)
                for i in capture:
                    inputs[i].append(aux[i].cpu() if cfg.offload else aux[i])
        finally:
            model.observer = None
        sorted_mags = {k: v.sorted() for k, v in samples.items()}
        names = list(MAPS)
        hidden = model.config.hidden_size
        for li, i in enumerate(self.layer_ids):
            layer = model.layers[i]
            maps = wanted[i]
            sizes = {m: int(getattr(layer, m).shape[0]) * int(getattr(layer, m).shape[1]) for m in maps}
            if greedy:
                levels, path = self._greedy(i, maps, sizes, sorted_mags, inputs[i], hidden * hidden)
                self.greedy_paths[i] = path
            else:
                levels = uniform_allocation(sizes, cfg.sparsity)
            for m in maps:
                j = names.index(m)
                self.levels[li, j] = levels[m]
                self.thresholds[li, j] = magnitude_quantile(sorted_mags[(i, m)], levels[m])

    def _greedy(self, index: int, maps: list[str], sizes: dict[str, int], mags, inputs: list[torch.Tensor],
                unit: int):
        model, cfg = self.model, self.config
        layer = model.layers[index]
        dev = model.device
        refs = [run_layer(model, index, h.to(dev)) for h in inputs]
        everywhere = PhasePolicy("all", "all", "all", "all", "all")
        originals = {m: getattr(layer, m) for m in maps}
        wrappers = {m: TealWeight(originals[m], 0.0, everywhere, kernel=False) for m in maps}
        for m, w in wrappers.items():
            install(layer, m, w)
        try:
            def error(levels) -> float:
                for m, w in wrappers.items():
                    w.threshold.fill_(magnitude_quantile(mags[(index, m)], levels[m]))
                errs = [greedy_error(ref, run_layer(model, index, h.to(dev)), cfg.greedy_fraction)
                        for ref, h in zip(refs, inputs)]
                return sum(errs) / max(len(errs), 1)

            return greedy_allocation(error, sizes, cfg.sparsity, step=cfg.greedy_step, unit=unit)
        finally:
            for m, w in originals.items():
                install(layer, m, w)

    # ---- install ------------------------------------------------------------------------------------------------
    def attach(self) -> None:
        self.detach()
        if not self.calibrated:
            self._calibrate()
        self.install()

    def install(self) -> None:
        self.detach()
        cfg, model = self.config, self.model
        policy = cfg.policy
        names = list(MAPS)
        self.masked = []
        for li, i in enumerate(self.layer_ids):
            layer = model.layers[i]
            for m in self._maps_of(layer):
                w = getattr(layer, m)
                reason = kernel_ineligibility(w)
                if cfg.backend == "auto" and reason is not None:
                    self.detach()
                    raise ConfigError(f"teal backend 'auto': layer {i + 1} {m} is {reason}; use backend='dense' "
                                      "to simulate the saving")
                kernel = cfg.backend != "dense" and reason is None
                if cfg.backend == "cuda" and not kernel:
                    self.masked.append(f"{i + 1}:{m}")
                thr = float(self.thresholds[li, names.index(m)])
                wrapped = TealWeight(w, thr, policy, kernel)
                was_param = isinstance(w, nn.Parameter)
                install(layer, m, wrapped)
                self._installed.append((layer, m, wrapped, was_param))

    def detach(self) -> None:
        for layer, m, wrapped, was_param in reversed(self._installed):
            w = wrapped.restore()
            install(layer, m, nn.Parameter(w, requires_grad=False) if was_param else w)
        self._installed = []

    def refresh_thresholds(self) -> None:
        """Hand the current thresholds to the installed maps (after a state load)."""
        names = list(MAPS)
        index = {i: li for li, i in enumerate(self.layer_ids)}
        for layer, m, wrapped, _ in self._installed:
            i = next(k for k in self.layer_ids if self.model.layers[k] is layer)
            wrapped.threshold.fill_(float(self.thresholds[index[i], names.index(m)]))

    def load_technique_state(self, state: dict[str, torch.Tensor]) -> None:
        super().load_technique_state(state)
        self.refresh_thresholds()

    def simulation(self) -> Simulation | None:
        if self.config.backend == "dense":
            return Simulation("weight reads", "backend='dense' masks the inputs of the dense products")
        if self.masked:
            return Simulation("weight reads", f"maps the kernel cannot serve run the masked dense product: "
                                              f"{', '.join(self.masked[:6])}")
        return None

    @property
    def summary(self) -> dict[str, object]:
        cols = [list(MAPS).index(m) for m in self.map_names]
        lv = self.levels[:, cols]
        return {"target": self.config.sparsity, "layers": len(self.layer_ids), "maps": self.map_names,
                "mean_level": float(lv[torch.isfinite(lv)].mean()) if torch.isfinite(lv).any() else math.nan,
                "installed": bool(self._installed)}
