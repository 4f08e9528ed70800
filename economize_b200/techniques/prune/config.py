"""Configurations of ``prune`` and ``depth_prune`` (economize field names, ``techniques/prune/config.py``)."""

from __future__ import annotations

from dataclasses import dataclass
from typing import ClassVar

from ...core.technique import TechniqueConfig
from ...errors import ConfigError
from ...validation import check_choice, check_positive

__all__ = ["DepthPruneConfig", "PruneConfig", "parse_sparsity"]


def parse_sparsity(value: float | str) -> tuple[float, tuple[int, int] | None]:
    """``(fraction removed, (n, m) or None)`` of ``0.5`` or ``"2:4"`` (keep n of every m)."""
    if isinstance(value, str):
        try:
            n, m = (int(v) for v in value.split(":"))
        except ValueError as e:
            raise ConfigError(f"sparsity must be a fraction or 'n:m', got {value!r}") from e
        if not 0 < n < m:
            raise ConfigError(f"N:M sparsity needs 0 < n < m, got {value!r}")
        return 1.0 - n / m, (n, m)
    v = float(value)
    if not 0.0 < v < 1.0:
        raise ConfigError(f"sparsity must lie in (0, 1), got {value}")
    return v, None


@dataclass(frozen=True)
class PruneConfig(TechniqueConfig):
    """Args:
        method: ``"magnitude"``, ``"wanda"`` (|W| x input norm; calibration) or ``"sparsegpt"`` (OBS masks with error
            feedback; calibration).
        sparsity: Fraction of weights removed per output row, or ``"n:m"`` (keep n of every m consecutive inputs).
        targets / exclude / layers: Which projections (Hugging Face name globs) of which 1-indexed layers.
        blocksize / percdamp: SparseGPT lazy block and Hessian damping.
        semi_structured: Store 2:4 weights compressed for the sparse GEMM (``None``: whenever the pattern is 2:4).
    """

    technique: ClassVar[str] = "prune"
    method: str = "wanda"
    sparsity: float | str = "2:4"
    targets: tuple[str, ...] = ("*",)
    exclude: tuple[str, ...] = ()
    layers: tuple[int, ...] = ()
    blocksize: int = 128
    percdamp: float = 0.01
    semi_structured: bool | None = None
    calibration_tokens: int = 512

    def __post_init__(self) -> None:
        check_choice("method", self.method, ("magnitude", "wanda", "sparsegpt"))
        parse_sparsity(self.sparsity)
        check_positive("blocksize", self.blocksize)
        object.__setattr__(self, "targets", tuple(self.targets))
        object.__setattr__(self, "exclude", tuple(self.exclude))
        object.__setattr__(self, "layers", tuple(int(i) for i in self.layers))
        if self.semi_structured and parse_sparsity(self.sparsity)[1] != (2, 4):
            raise ConfigError("semi_structured storage needs sparsity='2:4'")

    @property
    def needs_calibration(self) -> bool:
        return self.method != "magnitude"


@dataclass(frozen=True)
class DepthPruneConfig(TechniqueConfig):
    """Remove whole decoder blocks.

    Args:
        method: ``"shortgpt"`` (lowest block influence, one pass) or ``"sleb"`` (greedily remove the block whose removal
            raises the calibration NLL least, re-measured after each removal).
        num_blocks: Blocks to remove.
        keep_first / keep_last: Blocks at either end never removed (``None``: 1).
        layers: 1-indexed blocks to remove (filled with the chosen ones after attaching, so a checkpoint replays the
            same removal without calibration).
    """

    technique: ClassVar[str] = "depth_prune"
    method: str = "shortgpt"
    num_blocks: int = 1
    keep_first: int | None = None
    keep_last: int | None = None
    layers: tuple[int, ...] = ()

    def __post_init__(self) -> None:
        check_choice("method", self.method, ("shortgpt", "sleb"))
        check_positive("num_blocks", self.num_blocks)
        object.__setattr__(self, "layers", tuple(int(i) for i in self.layers))

    def validate(self, model) -> None:
        n = model.config.num_layers
        if self.num_blocks >= n:
            raise ConfigError(f"cannot remove {self.num_blocks} of {n} blocks")
