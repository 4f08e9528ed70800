"""Low-rank factorization of projections (``lowrank``; economize ``techniques/lowrank``, ``FACTORIZERS``).

``W [N, K] ~ U V`` with ``U [N, r]``, ``V [r, K]``; a decode pass then streams ``r (N + K)`` instead of ``N K``
weights (two tcgen05 GEMMs). Factorizers: ``svd`` (truncated SVD of W) and ``svd_llm`` (SVD-LLM, Wang et al. 2024:
SVD of ``W S`` where ``S`` is the Cholesky factor of the calibration Gram matrix ``X^T X``, so truncation minimises
the output error instead of the weight error; ``V = (top rows) S^-1``).
"""

from __future__ import annotations

from collections.abc import Callable
from dataclasses import dataclass
from typing import ClassVar

import torch
from torch import nn

from ... import ops
from ...core.technique import Capability, Family, Technique, TechniqueConfig, register_technique
from ...errors import ConfigError
from ...ops.quant import install
from ...registry import Registry
from ..quant.config import PROJECTIONS
from ..quant.methods import collect
from ..quant.technique import _key, _selected

__all__ = ["FACTORIZERS", "LowRankConfig", "LowRankTechnique", "LowRankWeight"]

FACTORIZERS: Registry[Callable] = Registry("factorizer", "economize_b200.factorizers")


class LowRankWeight(nn.Module):
    """``W = U V`` as two projections."""

    def __init__(self, u: torch.Tensor, v: torch.Tensor) -> None:
        super().__init__()
        self.u = nn.Parameter(u.contiguous(), requires_grad=False)
        self.v = nn.Parameter(v.contiguous(), requires_grad=False)

    @property
    def shape(self) -> torch.Size:
        return torch.Size((self.u.shape[0], self.v.shape[1]))

    @property
    def dtype(self) -> torch.dtype:
        return self.u.dtype

    @property
    def device(self) -> torch.device:
        return self.u.device

    def linear(self, x: torch.Tensor) -> torch.Tensor:
        return ops.linear(ops.linear(x, self.v), self.u)

    def dequantize(self, dtype: torch.dtype | None = None) -> torch.Tensor:
        return (self.u.float() @ self.v.float()).to(dtype or self.u.dtype)


@FACTORIZERS.register("svd")
def svd(w: torch.Tensor, rank: int, gram: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    u, s, vh = torch.linalg.svd(w.float(), full_matrices=False)
    r = min(rank, s.numel())
    return (u[:, :r] * s[:r]).to(w.dtype), vh[:r].to(w.dtype)


@FACTORIZERS.register("svd_llm")
def svd_llm(w: torch.Tensor, rank: int, gram: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    if gram is None:
        raise ConfigError("svd_llm needs calibration statistics")
    k = gram.shape[0]
    g = gram.double() + 1e-2 * torch.mean(torch.diag(gram.double())) * torch.eye(k, device=gram.device,
                                                                                 dtype=torch.float64)
    s_chol = torch.linalg.cholesky(g)  # X^T X = S S^T
    u, sig, vh = torch.linalg.svd(w.double() @ s_chol, full_matrices=False)
    r = min(rank, sig.numel())
    v = torch.linalg.solve_triangular(s_chol, vh[:r], upper=False, left=False)  # vh S^-1
    return (u[:, :r] * sig[:r]).to(w.dtype), v.to(w.dtype)


@dataclass(frozen=True)
class LowRankConfig(TechniqueConfig):
    """``ratio``: kept parameter fraction per projection (rank = ratio * N K / (N + K)); ``method`` a registered
    factorizer; ``targets`` / ``exclude`` / ``layers`` as for ``quant``."""

    technique: ClassVar[str] = "lowrank"
    method: str = "svd_llm"
    ratio: float = 0.5
    targets: tuple[str, ...] = ("*",)
    exclude: tuple[str, ...] = ()
    layers: tuple[int, ...] = ()

    def __post_init__(self) -> None:
        FACTORIZERS.get(self.method)
        if not 0.0 < self.ratio < 1.0:
            raise ConfigError("ratio must lie in (0, 1)")
        object.__setattr__(self, "targets", tuple(self.targets))
        object.__setattr__(self, "exclude", tuple(self.exclude))
        object.__setattr__(self, "layers", tuple(int(i) for i in self.layers))


@register_technique
class LowRankTechnique(Technique):
    config_class = LowRankConfig
    capabilities = Capability.WEIGHTS
    family = Family.OTHER
    lossless = False

    def __init__(self, config: LowRankConfig, model) -> None:
        super().__init__(config, model)
        self._calibration = None
        self.factors = nn.ModuleDict()

    def calibrate(self, calibration) -> None:
        self._calibration = calibration

    @torch.no_grad()
    def attach(self) -> None:
        cfg: LowRankConfig = self.config
        model = self.model
        if not self.factors:
            layers = [i - 1 for i in cfg.layers] if cfg.layers else range(model.config.num_layers)
            wanted = {i: [n for n, hf in PROJECTIONS.items() if _selected(hf, cfg.targets, cfg.exclude)
                          and getattr(model.layers[i], n).dim() == 2] for i in layers}
            stats = None
            if cfg.method == "svd_llm":
                cal = self._calibration
                if cal is None:
                    raise ConfigError("lowrank method='svd_llm' needs calibration tokens")
                batches = [cal if cal.dim() == 2 else cal[None]] if isinstance(cal, torch.Tensor) else list(cal)
                stats = collect(model, batches, wanted, hessian=True, keep_rows=0)
            for i, names in wanted.items():
                for name in names:
                    w = getattr(model.layers[i], name).detach()
                    n, k = w.shape
                    rank = max(8, int(cfg.ratio * n * k / (n + k)) // 8 * 8)
                    gram = stats[(i, name)].h if stats is not None else None
                    u, v = FACTORIZERS.get(cfg.method)(w, rank, gram)
                    self.factors[_key(i, name)] = LowRankWeight(u, v)
        for key, f in self.factors.items():
            i, name = key.split(":")
            install(model.layers[int(i)], name, f)

    def load_technique_state(self, state: dict[str, torch.Tensor]) -> None:
        found: dict[str, dict[str, torch.Tensor]] = {}
        for name, t in state.items():
            _, key, part = name.split(".")
            found.setdefault(key, {})[part] = t
        for key, parts in found.items():
            self.factors[key] = LowRankWeight(parts["u"], parts["v"])
