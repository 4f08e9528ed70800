"""LittleBit (``littlebit``; Lee et al., NeurIPS 2025; economize ``techniques/littlebit``): binary low-rank weight
factorization below one bit per weight.

Every selected projection becomes ``P`` paths (two with residual compensation) of
``diag(h) sign(U) diag(l) sign(V) diag(g)`` (:class:`~economize_b200.ops.littlebit.LittleBitWeight`), initialised
by Dual-SVID: the truncated SVD ``W ~ U' V'`` with ``sqrt(sigma)`` split between the factors, their signs kept and
the magnitudes fitted by rank-one products ``|U'| ~ h l_u^T``, ``|V'| ~ l_v g^T``, ``l = l_u l_v``; the residual path
repeats it on ``W - W_1``. The rank follows the bit budget ``bpw`` (signs ``r (out + in)`` and 16-bit scales
``16 (out + in + r)`` per path). Not built: the SmoothSign quantization-aware training.
"""

from __future__ import annotations

import fnmatch
from dataclasses import dataclass
from typing import ClassVar

import torch
from torch import nn

from ...core.technique import Capability, Family, Technique, TechniqueConfig, register_technique
from ...errors import ConfigError
from ...ops.littlebit import LittleBitWeight
from ...ops.quant import install
from ...validation import check_choice, check_positive

__all__ = ["LittleBitConfig", "LittleBitTechnique", "dual_svid", "rank_for_bpw", "rank_one"]

SCALE_BITS = 16
MAPS = {"wqkv": ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj"), "wo": ("self_attn.o_proj",),
        "w_gate_up": ("mlp.gate_proj", "mlp.up_proj"), "w_down": ("mlp.down_proj",)}


def rank_for_bpw(out_features: int, in_features: int, bpw: float, *, paths: int = 2, multiple: int = 1) -> int:
    """The largest rank within ``bpw`` bits per weight, rounded down to a multiple of ``multiple`` (0: none fits)."""
    if bpw <= 0:
        raise ConfigError(f"bpw must be positive, got {bpw}")
    budget = bpw * out_features * in_features - paths * SCALE_BITS * (out_features + in_features)
    rank = int(budget // (paths * (out_features + in_features + SCALE_BITS)))
    rank = min(rank, out_features, in_features)
    return max(0, rank // multiple * multiple)


def rank_one(m: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """The best rank-one fit ``m ~ a b^T`` of a non-negative matrix (leading singular pair, made non-negative)."""
    u, s, vh = torch.linalg.svd(m, full_matrices=False)
    a = u[:, 0].abs() * s[0].sqrt()
    b = vh[0].abs() * s[0].sqrt()
    return a, b


def dual_svid(weight: torch.Tensor, rank: int):
    """One path ``(u [out, r], v [r, in], h [out], g [in], l [r])`` of Dual-SVID for ``weight`` (fp32)."""
    left, sigma, right = torch.linalg.svd(weight.detach().float(), full_matrices=False)
    root = sigma[:rank].sqrt()
    u = left[:, :rank] * root
    v = root[:, None] * right[:rank]
    h, l_u = rank_one(u.abs())
    l_v, g = rank_one(v.abs())
    return u, v, h, g, l_u * l_v


def _dense(u, v, h, g, l) -> torch.Tensor:
    return (h[:, None] * torch.sign(u) * l[None]) @ (torch.sign(v) * g[None])


def littlebit_factors(weight: torch.Tensor, rank: int, residual: bool):
    paths = [dual_svid(weight, rank)]
    if residual:
        paths.append(dual_svid(weight.float() - _dense(*paths[0]), rank))
    return [torch.stack([p[i] for p in paths]) for i in range(5)]


@dataclass(frozen=True)
class LittleBitConfig(TechniqueConfig):
    technique: ClassVar[str] = "littlebit"
    method: str = "dual_svid"
    bpw: float = 1.0
    residual: bool = True
    targets: tuple[str, ...] = ("*",)
    exclude: tuple[str, ...] = ()
    layers: tuple[int, ...] = ()
    rank_multiple: int = 32
    backend: str = "auto"
    qat_steps: int = 0
    qat_lr: float = 1e-3
    smooth_k: float = 100.0
    calibration_tokens: int = 512

    def __post_init__(self) -> None:
        check_choice("method", self.method, ("dual_svid",))
        check_positive("bpw", self.bpw)
        check_positive("rank_multiple", self.rank_multiple)
        if self.backend == "triton":
            raise ConfigError("backend 'triton' is economize's Triton kernel; this build's is CUDA: use 'auto'")
        check_choice("backend", self.backend, ("auto", "reference"))
        if self.qat_steps < 0 or self.qat_lr <= 0 or self.smooth_k <= 0 or self.calibration_tokens < 1:
            raise ConfigError("qat_steps must be >= 0 and qat_lr, smooth_k, calibration_tokens positive")
        object.__setattr__(self, "targets", tuple(self.targets))
        object.__setattr__(self, "exclude", tuple(self.exclude))
        object.__setattr__(self, "layers", tuple(self.layers))


def _selected(name: str, targets, exclude) -> bool:
    names = (name, *MAPS[name], *(n.split(".")[-1] for n in MAPS[name]))
    hit = lambda pats: any(fnmatch.fnmatchcase(n, p) for n in names for p in pats)  # noqa: E731
    return hit(targets) and not hit(exclude)


@register_technique
class LittleBitTechnique(Technique):
    """State: the packed factors of every replaced projection (``weights.<layer>:<name>.<buffer>``)."""

    config_class = LittleBitConfig
    capabilities = Capability.WEIGHTS
    family = Family.QUANTIZATION
    lossless = False

    def __init__(self, config: LittleBitConfig, model) -> None:
        super().__init__(config, model)
        if model.config.is_moe:
            raise ConfigError("littlebit supports dense models")
        n = model.config.num_layers
        self.layer_ids = [i - 1 for i in config.layers] if config.layers else list(range(n))
        self.weights = nn.ModuleDict()

    @torch.no_grad()
    def attach(self) -> None:
        cfg, m = self.config, self.model
        paths = 2 if cfg.residual else 1
        for i in self.layer_ids:
            layer = m.layers[i]
            for name in MAPS:
                if not _selected(name, cfg.targets, cfg.exclude):
                    continue
                key = f"{i}:{name}"
                if key not in self.weights:
                    w = getattr(layer, name)
                    if not isinstance(w, torch.Tensor):
                        raise ConfigError(f"littlebit replaces plain weights; layer {i + 1} {name} is a "
                                          f"{type(w).__name__}")
                    out_f, in_f = w.shape
                    r = rank_for_bpw(out_f, in_f, cfg.bpw, paths=paths, multiple=cfg.rank_multiple)
                    if r == 0:
                        raise ConfigError(f"bpw={cfg.bpw} leaves no rank for a {out_f} x {in_f} map")
                    self.weights[key] = LittleBitWeight(*littlebit_factors(w, r, cfg.residual), m.dtype)
                install(layer, name, self.weights[key])

    def _targets(self) -> dict[int, list[str]]:
        cfg = self.config
        return {i: [n for n in MAPS if _selected(n, cfg.targets, cfg.exclude)] for i in self.layer_ids}

    def calibrate(self, calibration) -> None:
        """With ``qat_steps > 0``: train every selected map's factors on calibration activations (SmoothSign
        straight-through signs, activation-aware output error; :mod:`.qat`) before the maps are replaced.
        ``qat_report`` keeps each map's relative output error before and after."""
        cfg = self.config
        if cfg.qat_steps == 0:
            return
        from ..quant.methods import collect
        from .qat import train_map

        tokens = calibration if isinstance(calibration, (list, tuple)) else [torch.as_tensor(calibration)]
        tokens = [t if t.dim() == 2 else t[None] for t in tokens]
        wanted = self._targets()
        stats = collect(self.model, tokens, wanted, False, cfg.calibration_tokens)
        paths = 2 if cfg.residual else 1
        self.qat_report: dict[str, tuple[float, float]] = {}
        for i, names in wanted.items():
            layer = self.model.layers[i]
            for name in names:
                w = getattr(layer, name)
                if not isinstance(w, torch.Tensor):
                    continue
                out_f, in_f = w.shape
                r = rank_for_bpw(out_f, in_f, cfg.bpw, paths=paths, multiple=cfg.rank_multiple)
                if r == 0:
                    continue
                init = littlebit_factors(w, r, cfg.residual)
                with torch.enable_grad():
                    factors, before, after = train_map(w, stats[(i, name)].sample, init, cfg.qat_steps, cfg.qat_lr,
                                                       cfg.smooth_k)
                self.weights[f"{i}:{name}"] = LittleBitWeight(*factors, self.model.dtype)
                self.qat_report[f"{i}:{name}"] = (before, after)

    def technique_state(self) -> dict[str, torch.Tensor]:
        out = {}
        for key, w in self.weights.items():
            for buf in ("u_bits", "v_bits", "h", "g", "l"):
                out[f"weights.{key}.{buf}"] = getattr(w, buf).detach()
        return out

    def load_technique_state(self, state: dict[str, torch.Tensor]) -> None:
        found: dict[str, dict[str, torch.Tensor]] = {}
        for name, t in state.items():
            if not name.startswith("weights."):
                raise ConfigError(f"littlebit: unexpected tensor {name}")
            key, buf = name[len("weights."):].rsplit(".", 1)
            found.setdefault(key, {})[buf] = t
        self.weights = nn.ModuleDict()
        for key, b in found.items():
            w = LittleBitWeight.__new__(LittleBitWeight)
            nn.Module.__init__(w)
            w.out_features, w.rank = b["u_bits"].shape[1], b["v_bits"].shape[1]
            w.in_features = b["g"].shape[1]
            w.compute_dtype = self.model.dtype
            for buf, t in b.items():
                w.register_buffer(buf, t.to(self.model.device))
            self.weights[key] = w

    def bits_per_weight(self) -> float:
        total = sum(w.out_features * w.in_features for w in self.weights.values())
        return sum(w.bits_per_weight() * w.out_features * w.in_features for w in self.weights.values()) / max(total, 1)
