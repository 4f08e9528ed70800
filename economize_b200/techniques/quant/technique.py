"""``quant`` and ``draft_quant`` techniques: replace projections by packed :class:`~economize_b200.ops.quant.QWeight`
weights that the tcgen05 weight-only GEMM reads (economize ``techniques/quant/technique.py:30-120``).

The quantized weights (and, after AWQ, the re-scaled norm and producer weights) are the technique's state, so a
saved model reloads without recalibrating.
"""

from __future__ import annotations

import fnmatch
from typing import Any

import torch
from torch import nn

from ...core.technique import Capability, Family, Technique, register_technique
from ...errors import ConfigError
from ...ops.fp8 import FP8BlockWeight
from ...ops.quant import CODES_PER_BYTE, FP4_GROUP, QWeight, install
from . import methods
from .config import PROJECTIONS, DraftQuantConfig, QuantConfig

__all__ = ["DraftQuantTechnique", "QuantTechnique"]


def _selected(names: tuple[str, ...], targets: tuple[str, ...], exclude: tuple[str, ...]) -> bool:
    def match(pats):
        return any(fnmatch.fnmatchcase(n, p) for n in names for p in pats)

    return match(targets) and not (exclude and all(any(fnmatch.fnmatchcase(n, p) for p in exclude) for n in names))


def _key(layer: int, name: str) -> str:
    return f"{layer}:{name}"


class _QuantBase(Technique):
    capabilities = Capability.WEIGHTS
    family = Family.QUANTIZATION

    def __init__(self, config, model) -> None:
        super().__init__(config, model)
        self.weights = nn.ModuleDict()
        self.replaced: dict[str, torch.Tensor] = {}  # full-precision weights other than projections (AWQ folding)

    def technique_state(self) -> dict[str, torch.Tensor]:
        out = {}
        for key, qw in self.weights.items():
            for buf in ("codes", "qweight", "scales", "zeros"):
                t = getattr(qw, buf, None)
                if t is not None:
                    out[f"weights.{key}.{buf}"] = t.detach()
        for key, t in self.replaced.items():
            out[f"replaced.{key}"] = t.detach()
        return out

    def load_technique_state(self, state: dict[str, torch.Tensor]) -> None:
        cfg = self.config
        found: dict[str, dict[str, torch.Tensor]] = {}
        for name, t in state.items():
            if name.startswith("weights."):
                key, buf = name[len("weights."):].rsplit(".", 1)
                found.setdefault(key, {})[buf] = t
            elif name.startswith("replaced."):
                self.replaced[name[len("replaced."):]] = t
            else:
                raise ConfigError(f"{self.name}: unexpected tensor {name}")
        self.weights = nn.ModuleDict()
        for key, bufs in found.items():
            if "codes" in bufs:
                self.weights[key] = FP8BlockWeight(bufs["codes"], bufs["scales"], self._dtype())
                continue
            k_in = bufs["qweight"].shape[1] * CODES_PER_BYTE.get(cfg.format, 1)
            group = FP4_GROUP.get(cfg.format) or cfg.group_size or k_in
            self.weights[key] = QWeight(bufs["qweight"], bufs["scales"], bufs.get("zeros"), cfg.format, group,
                                        self._dtype())

    def _dtype(self) -> torch.dtype:
        return self.model.dtype

    def nbytes(self) -> int:
        return sum(q.nbytes() for q in self.weights.values())


@register_technique
class QuantTechnique(_QuantBase):
    """Weight-only quantization of the target (RTN, GPTQ or AWQ; int4 / int8 / fp8)."""

    config_class = QuantConfig
    lossless = False

    def __init__(self, config: QuantConfig, model) -> None:
        super().__init__(config, model)
        self._calibration: Any = None

    def calibrate(self, calibration: Any) -> None:
        self._calibration = calibration

    def _targets(self) -> dict[int, list[str]]:
        """Projections to quantize; those whose input width the group size (or the kernel's 64-wide K tile) does
        not divide are skipped and listed in ``self.skipped``."""
        cfg: QuantConfig = self.config
        layers = [i - 1 for i in cfg.layers] if cfg.layers else range(self.model.config.num_layers)
        out = {}
        self.skipped: list[str] = []
        for i in layers:
            names = []
            for n, hf in PROJECTIONS.items():
                if not _selected(hf, cfg.targets, cfg.exclude):
                    continue
                w = getattr(self.model.layers[i], n)
                if w.dim() != 2:  # stacked MoE experts
                    self.skipped.append(f"layers.{i}.{n}")
                    continue
                k = w.shape[1]
                block = cfg.format == "fp8_block"
                if (block and (k % 128 or w.shape[0] % 128)) or \
                        (not block and (k % 64 or (cfg.group_size and k % cfg.group_size))):
                    self.skipped.append(f"layers.{i}.{n}")
                    continue
                names.append(n)
            if names:
                out[i] = names
        return out

    def _batches(self) -> list[torch.Tensor]:
        cal = self._calibration
        if cal is None:
            raise ConfigError(f"method={self.config.method!r} needs calibration tokens: apply(..., calibration=ids)")
        if isinstance(cal, torch.Tensor):
            return [cal if cal.dim() == 2 else cal[None]]
        return [torch.as_tensor(c) for c in cal]

    @torch.no_grad()
    def _quantize(self) -> None:
        cfg: QuantConfig = self.config
        model = self.model
        wanted = self._targets()
        stats = None
        if cfg.needs_calibration:
            stats = methods.collect(model, self._batches(), wanted, hessian=cfg.method == "gptq",
                                    keep_rows=cfg.calibration_tokens)
        if cfg.method in ("awq", "smoothquant"):
            self._awq_fold(wanted, stats)
        for i, names in wanted.items():
            layer = model.layers[i]
            for name in names:
                w = getattr(layer, name).detach()
                if cfg.format == "fp8_block":
                    self.weights[_key(i, name)] = FP8BlockWeight.from_weight(w)
                    continue
                if cfg.method == "gptq":
                    qw = methods.gptq(w, stats[(i, name)].hessian, cfg.format, cfg.group_size, cfg.symmetric,
                                      cfg.blocksize, cfg.percdamp, cfg.act_order)
                elif cfg.method == "awq" and cfg.awq_clip:
                    g = cfg.group_size or w.shape[1]
                    x = stats[(i, name)].sample * self._awq_scale.get((i, name), 1.0)
                    ratio = methods.awq_clip(w, x, cfg.format, g, cfg.symmetric, cfg.awq_grid)
                    qw = methods.rtn(w, cfg.format, g, cfg.symmetric, ratio)
                elif cfg.method == "hqq":
                    qw = methods.hqq(w, cfg.format, cfg.group_size, cfg.symmetric, cfg.hqq_iters, cfg.hqq_p)
                else:
                    qw = methods.rtn(w, cfg.format, cfg.group_size, cfg.symmetric)
                self.weights[_key(i, name)] = qw

    @torch.no_grad()
    def _awq_fold(self, wanted: dict[int, list[str]], stats) -> None:
        """Search and fold AWQ scales: x/s goes into the producer of x (a norm weight or projection rows)."""
        cfg: QuantConfig = self.config
        c = self.model.config
        self._awq_scale: dict[tuple[int, str], torch.Tensor] = {}
        for i, names in wanted.items():
            layer = self.model.layers[i]
            g = cfg.group_size
            for name in names:
                if name == "wo" and c.num_heads != c.num_kv_heads:
                    continue  # query heads share value heads: no per-channel producer to fold into
                if cfg.method == "smoothquant" and name not in ("wqkv", "w_gate_up"):
                    continue  # SmoothQuant smooths the inputs that a norm produces (QKV and the first FFN map)
                w = getattr(layer, name)
                if cfg.method == "smoothquant":
                    s = methods.smooth_scales([w.detach()], stats[(i, name)], cfg.smooth_alpha)
                else:
                    s = methods.awq_search([w.detach()], stats[(i, name)], cfg.format, g or w.shape[1],
                                           cfg.symmetric, cfg.awq_grid)
                w.mul_(s.to(w.dtype)[None, :])
                if name == "wqkv":
                    layer.attn_norm.div_(s.to(layer.attn_norm.dtype))
                    self.replaced[f"{i}:attn_norm"] = layer.attn_norm.detach().clone()
                elif name == "w_gate_up":
                    layer.mlp_norm.div_(s.to(layer.mlp_norm.dtype))
                    self.replaced[f"{i}:mlp_norm"] = layer.mlp_norm.detach().clone()
                elif name == "w_down":
                    f = w.shape[1]
                    if isinstance(layer.w_gate_up, QWeight):
                        raise ConfigError("AWQ needs the full-precision up projection to fold the down scales")
                    layer.w_gate_up[f:].div_(s.to(w.dtype)[:, None])
                    self.replaced[f"{i}:w_gate_up"] = layer.w_gate_up.detach().clone()
                elif name == "wo":
                    v0 = c.q_size + c.kv_size
                    layer.wqkv[v0:].div_(s.to(w.dtype)[:, None])
                    self.replaced[f"{i}:wqkv"] = layer.wqkv.detach().clone()
                self._awq_scale[(i, name)] = (1.0 / s)[None, :]

    def inplace_targets(self) -> list[torch.Tensor]:
        """AWQ and SmoothQuant fold their scales into the projections and norms of the quantized layers in place."""
        if self.weights or self.config.method not in ("awq", "smoothquant"):
            return []
        layers = [i - 1 for i in self.config.layers] if self.config.layers else range(self.model.config.num_layers)
        out = []
        for i in layers:
            layer = self.model.layers[i]
            out += [t for t in (layer.attn_norm, layer.mlp_norm, layer.wqkv, layer.wo, layer.w_gate_up, layer.w_down)
                    if isinstance(t, torch.Tensor)]
        return out

    def attach(self) -> None:
        if not self.weights:
            self._quantize()
        model = self.model
        for key, t in self.replaced.items():  # AWQ-folded full-precision tensors (before the projections)
            i, name = key.split(":")
            p = getattr(model.layers[int(i)], name)
            if isinstance(p, torch.Tensor):
                p.data.copy_(t.to(p.device, p.dtype))
        for key, qw in self.weights.items():
            i, name = key.split(":")
            layer = model.layers[int(i)]
            if self.config.backend == "fake":
                install(layer, name, nn.Parameter(qw.dequantize().to(model.device), requires_grad=False))
            else:
                install(layer, name, qw.to(model.device))


@register_technique
class DraftQuantTechnique(_QuantBase):
    """Round-to-nearest quantization of the drafter's projections (lossless: the target verifies every token)."""

    config_class = DraftQuantConfig
    family = Family.DRAFT_COMPRESSION  # quantizes a different model than ``quant``: the two combine
    lossless = True

    def conflicts(self, other) -> str | None:
        return None

    def _drafter_technique(self):
        return self._drafter

    def bind(self, drafter_technique) -> None:
        self._drafter = drafter_technique

    def attach(self) -> None:
        """Quantization of the drafter happens when the drafting technique attaches (it attaches after weights)."""

    @torch.no_grad()
    def after_drafter(self, technique: nn.Module) -> None:
        cfg: DraftQuantConfig = self.config
        while hasattr(technique, "wrapped_drafter"):  # a hybrid's fallback
            technique = technique.wrapped_drafter
        if not self.weights:
            for name, p in list(technique.named_parameters()):
                if p.dim() != 2 or not _selected((name,), cfg.targets, cfg.exclude):
                    continue
                k = p.shape[1]
                g = cfg.group_size if cfg.group_size and k % cfg.group_size == 0 else None
                if (g or k) % 64 or k % 64 or p.shape[0] % 8:
                    continue
                self.weights[name.replace(".", "/")] = methods.rtn(p.detach(), cfg.format, g or k, cfg.symmetric)
        for key, qw in self.weights.items():
            path = key.split("/")
            owner = technique
            for part in path[:-1]:
                owner = getattr(owner, part)
            if cfg.backend == "fake":
                install(owner, path[-1], nn.Parameter(qw.dequantize().to(technique_device(technique)),
                                                      requires_grad=False))
            else:
                install(owner, path[-1], qw.to(technique_device(technique)))


def technique_device(module: nn.Module) -> torch.device:
    for t in list(module.parameters()) + list(module.buffers()):
        return t.device
    return torch.device("cpu")
