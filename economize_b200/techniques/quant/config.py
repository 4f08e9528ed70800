"""Configurations of weight quantization (``quant``) and drafter-only quantization (``draft_quant``).

Field names and defaults follow economize (``src/economize/techniques/quant/config.py:82-245``) for the options the
engine executes; the storage is always the packed layout of the tcgen05 weight-only GEMM, so ``backend`` accepts
``"auto"`` (that kernel on CUDA, the PyTorch reference on the CPU) and ``"fake"`` (dequantized bf16 weights: the
simulated reference economize also offers).
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import ClassVar

from ...core.technique import TechniqueConfig
from ...errors import ConfigError
from ...validation import check_choice, check_positive

__all__ = ["DraftQuantConfig", "QUANT_FORMATS", "QUANT_METHODS_NAMES", "QuantConfig"]

#: formats the packed kernel layout stores
QUANT_FORMATS = ("int2", "int3", "int4", "int8", "fp8", "fp8_block", "mxfp4", "nvfp4")
QUANT_METHODS_NAMES = ("rtn", "gptq", "awq", "hqq", "smoothquant")
#: engine projection names and the Hugging Face module names fused into them
PROJECTIONS = {"wqkv": ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj"), "wo": ("self_attn.o_proj",),
               "w_gate_up": ("mlp.gate_proj", "mlp.up_proj"), "w_down": ("mlp.down_proj",)}


def _check_common(config) -> None:
    check_choice("format", config.format, QUANT_FORMATS)
    check_choice("backend", config.backend, ("auto", "fake"))
    if config.group_size is not None:
        check_positive("group_size", config.group_size)
        if config.group_size % 64:
            raise ConfigError(f"group_size must be a multiple of 64 (the kernel's K tile), got {config.group_size}")
    if config.format == "fp8_block":
        return  # 128 x 128 weight blocks and 1 x 128 activation blocks are fixed by the format
    if config.format in ("int8", "fp8") and not config.symmetric:
        raise ConfigError(f"{config.format} weights are stored symmetric (no zero point): set symmetric=True")


@dataclass(frozen=True)
class QuantConfig(TechniqueConfig):
    """Weight-only quantization of the target's decoder projections.

    Args:
        format: ``"int4"`` (default, GPTQ/AWQ W4A16), ``"int3"`` / ``"int2"`` (W3A16 in the int4 layout, W2A16
            packed 16 per word), ``"mxfp4"`` / ``"nvfp4"`` (FP4 E2M1 weights with a scale per 32 / 16 columns;
            ``group_size`` and ``symmetric`` do not apply), ``"int8"`` (W8A16), ``"fp8"`` (e4m3 weights, bf16
            activations) or ``"fp8_block"`` (W8A8: e4m3 weights with 128 x 128 block scales and activations
            quantised per token and 128-wide block on the fly; ``group_size`` is ignored).
        method: ``"rtn"`` (round to nearest, no data), ``"hqq"`` (half-quadratic fit of the grid, no data),
            ``"smoothquant"`` (activation outliers migrated into the weights, then round to nearest: for W8A8 with
            ``format="fp8_block"``), ``"gptq"`` (Hessian-aware error feedback, needs
            calibration tokens) or ``"awq"`` (activation-aware scaling folded into the preceding norm, then round
            to nearest with clipping search; needs calibration tokens).
        group_size: Input columns per scale (``None``: one scale per output row).
        symmetric: Integer grids without a zero point (int4 then stores the zero point 8).
        backend: ``"auto"`` or ``"fake"``.
        targets: Projection globs over Hugging Face names (``"self_attn.*"``, ``"mlp.down_proj"``); a fused
            projection is quantized when any of its parts matches.
        exclude: Globs removed from ``targets``.
        layers: 1-indexed layers to quantize; empty means all.
        act_order: GPTQ: quantize columns by decreasing Hessian diagonal (groups fitted on contiguous columns).
        blocksize: GPTQ lazy-update block.
        percdamp: GPTQ relative Hessian damping.
        awq_grid: AWQ: number of scale exponents and clipping ratios searched.
        awq_clip: AWQ: search per-group clipping thresholds.
        calibration_tokens: Rows of activations kept per projection for AWQ's search.
        hqq_iters, hqq_p: HQQ: half-quadratic iterations and the ``l_p`` norm of its error model (``p < 1``).
        smooth_alpha: SmoothQuant's migration strength ``alpha``.
    """

    technique: ClassVar[str] = "quant"

    format: str = "int4"
    method: str = "rtn"
    group_size: int | None = 128
    symmetric: bool = False
    backend: str = "auto"
    targets: tuple[str, ...] = ("*",)
    exclude: tuple[str, ...] = ()
    layers: tuple[int, ...] = ()
    act_order: bool = False
    blocksize: int = 128
    percdamp: float = 0.01
    awq_grid: int = 20
    awq_clip: bool = True
    calibration_tokens: int = 512
    hqq_iters: int = 20
    hqq_p: float = 0.7
    smooth_alpha: float = 0.5

    def __post_init__(self) -> None:
        check_choice("method", self.method, QUANT_METHODS_NAMES)
        check_positive("blocksize", self.blocksize)
        check_positive("awq_grid", self.awq_grid)
        if not 0.0 <= self.percdamp <= 1.0:
            raise ConfigError(f"percdamp must lie in [0, 1], got {self.percdamp}")
        if any(int(i) < 1 for i in self.layers):
            raise ConfigError("layers are 1-indexed")
        if self.method in ("gptq", "awq", "hqq") and self.format in ("fp8", "fp8_block"):
            raise ConfigError(f"{self.method} fits integer grids; use method='rtn' for fp8")
        if self.method in ("hqq", "smoothquant") and self.format in ("mxfp4", "nvfp4"):
            raise ConfigError(f"{self.method} does not fit FP4 grids; use rtn, gptq or awq")
        check_positive("hqq_iters", self.hqq_iters)
        if not 0.0 < self.hqq_p <= 1.0 or not 0.0 <= self.smooth_alpha <= 1.0:
            raise ConfigError("hqq_p must lie in (0, 1] and smooth_alpha in [0, 1]")
        object.__setattr__(self, "targets", tuple(self.targets))
        object.__setattr__(self, "exclude", tuple(self.exclude))
        object.__setattr__(self, "layers", tuple(int(i) for i in self.layers))
        _check_common(self)

    @property
    def needs_calibration(self) -> bool:
        return self.method in ("gptq", "awq", "smoothquant")

    def validate(self, model) -> None:
        n = model.config.num_layers
        bad = [i for i in self.layers if i > n]
        if bad:
            raise ConfigError(f"layers {bad} exceed the model's {n} layers")
        if model.config.is_moe and self.format != "fp8_block":
            raise ConfigError("MoE models take format='fp8_block' (attention projections; experts stay bf16)")


@dataclass(frozen=True)
class DraftQuantConfig(TechniqueConfig):
    """Round-to-nearest quantization of the drafter's own projections only (the verified target is untouched, so
    decoding stays lossless; only the acceptance rate can change)."""

    technique: ClassVar[str] = "draft_quant"

    format: str = "int8"
    group_size: int | None = 128
    symmetric: bool = True
    backend: str = "auto"
    targets: tuple[str, ...] = ("*",)
    exclude: tuple[str, ...] = ("*lora*",)

    def __post_init__(self) -> None:
        object.__setattr__(self, "targets", tuple(self.targets))
        object.__setattr__(self, "exclude", tuple(self.exclude))
        _check_common(self)
