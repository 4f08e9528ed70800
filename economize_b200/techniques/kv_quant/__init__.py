"""KV-cache quantization: ``kivi`` / ``kivi_fused`` (2- or 4-bit KIVI chunks dequantised inside the attention
kernel) and ``kv_fp8`` / ``kv_fp8_fused`` (e4m3 codes with static per-head, per-layer or unit scales,
read directly by the tcgen05 attention kernel) (economize ``techniques/kv_quant/fp8.py:55-270`` and
``techniques/kv_fp8_fused``).

The cache stores ``e4m3(x / s)``; the attention kernel converts the codes to bf16 in shared memory and applies
``s_k`` to the scores and ``s_v`` to the output, so a decode pass reads half the cache bytes. Scales come from the
absolute maxima of a calibration prefill (``scale="head"``: one per layer and KV head, ``"tensor"``: one per layer,
``"none"``: 1.0) divided by 448, e4m3's largest finite value.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, ClassVar

import torch

from ...core.technique import Capability, Family, Technique, TechniqueConfig, register_technique
from ...errors import ConfigError
from ...validation import check_choice

__all__ = ["KIVIConfig", "KIVIFusedConfig", "KIVITechnique", "KVFp8Config", "KVFp8FusedConfig", "KVFp8Technique",
           "calibrate_kv_scales"]

E4M3_MAX = 448.0


@dataclass(frozen=True)
class KVFp8Config(TechniqueConfig):
    """fp8 KV cache.

    Args:
        format: ``"e4m3"`` (the only format the kernels read).
        scale: ``"head"`` (static per layer and KV head, from calibration), ``"tensor"`` (one per layer) or
            ``"none"`` (unit scales: values beyond +-448 saturate).
        margin: Headroom factor applied to calibrated maxima.
    """

    technique: ClassVar[str] = "kv_fp8"
    format: str = "e4m3"
    scale: str = "head"
    margin: float = 1.0

    def __post_init__(self) -> None:
        check_choice("format", self.format, ("e4m3",))
        check_choice("scale", self.scale, ("head", "tensor", "none"))
        if self.margin < 1.0:
            raise ConfigError("margin must be >= 1")


@dataclass(frozen=True)
class KVFp8FusedConfig(KVFp8Config):
    """Same storage under economize's name for the kernel-read fp8 views."""

    technique: ClassVar[str] = "kv_fp8_fused"


@torch.no_grad()
def calibrate_kv_scales(model, batches, mode: str = "head", margin: float = 1.0) -> tuple[torch.Tensor, torch.Tensor]:
    """Per (layer, KV head) scales ``max|x| * margin / 448`` of keys (after rotary) and values over a prefill of the
    calibration token batches ``[B, L]``."""
    from ...runtime.cache import KVCache, StepBatch

    c = model.config
    hkv = model.local["num_kv_heads"]
    amax = torch.zeros(2, c.num_layers, hkv, device=model.device)
    for tokens in batches:
        tokens = torch.as_tensor(tokens).to(model.device)
        if tokens.dim() == 1:
            tokens = tokens[None]
        b, length = tokens.shape
        cache = KVCache(c.num_layers, b, hkv, ((length + 127) // 128) * 128, c.head_dim, model.dtype, model.device)
        lengths = torch.full((b,), length, dtype=torch.int32, device=model.device)
        model.forward_step(tokens, StepBatch.prefill(lengths, length), cache)
        vals = cache.data[:, :, :, :, :length].float().abs().amax(dim=(2, 4, 5))  # [L, 2, Hkv]
        amax = torch.maximum(amax, vals.permute(1, 0, 2))
    if mode == "tensor":
        amax = amax.amax(-1, keepdim=True).expand_as(amax)
    scales = torch.where(amax > 0, amax * margin / E4M3_MAX, torch.ones_like(amax))
    return scales[0].contiguous(), scales[1].contiguous()


@register_technique
class KVFp8Technique(Technique):
    config_class = KVFp8Config
    capabilities = Capability.KV_CACHE
    family = Family.KV_COMPRESSION
    lossless = False

    def __init__(self, config: KVFp8Config, model) -> None:
        super().__init__(config, model)
        hkv = model.local["num_kv_heads"]
        ones = torch.ones(model.config.num_layers, hkv, dtype=torch.float32, device=model.device)
        self.register_buffer("k_scale", ones.clone())
        self.register_buffer("v_scale", ones.clone())
        self._calibration: Any = None
        self._calibrated = False

    def calibrate(self, calibration: Any) -> None:
        self._calibration = calibration

    def load_technique_state(self, state: dict[str, torch.Tensor]) -> None:
        super().load_technique_state(state)
        self._calibrated = True

    def attach(self) -> None:
        model = self.model
        if not self._calibrated and self.config.scale != "none":
            if self._calibration is None:
                raise ConfigError(f"kv_fp8 with scale={self.config.scale!r} needs calibration tokens "
                                  "(apply(..., calibration=ids)); use scale='none' for unit scales")
            cal = self._calibration
            batches = [cal] if isinstance(cal, torch.Tensor) else list(cal)
            k, v = calibrate_kv_scales(model, batches, self.config.scale, self.config.margin)
            self.k_scale.copy_(k)
            self.v_scale.copy_(v)
            self._calibrated = True
        model.kv_dtype = torch.float8_e4m3fn
        model.kv_scales = (self.k_scale, self.v_scale)

    def detach(self) -> None:
        self.model.kv_dtype = None
        self.model.kv_scales = None


@register_technique
class KVFp8FusedTechnique(KVFp8Technique):
    config_class = KVFp8FusedConfig


# ---- KIVI ------------------------------------------------------------------------------------------------------
@dataclass(frozen=True)
class KIVIConfig(TechniqueConfig):
    """KIVI-coded KV cache (Liu et al., 2024; economize ``kivi``/``kivi_fused``, ``kv_quant/packed.py``).

    Args:
        bits: 2 or 4.
        residual: Most recent committed tokens kept in bf16 (at least this many; coding happens in 128-key chunks).
    """

    technique: ClassVar[str] = "kivi"
    bits: int = 2
    residual: int = 128

    def __post_init__(self) -> None:
        check_choice("bits", self.bits, (2, 4))
        if self.residual < 0:
            raise ConfigError("residual must be >= 0")


@dataclass(frozen=True)
class KIVIFusedConfig(KIVIConfig):
    technique: ClassVar[str] = "kivi_fused"


@register_technique
class KIVITechnique(Technique):
    """Codes committed chunks after every commit (one kernel per cycle, inside the captured graph) and hands the
    attention kernel the coded chunks, which it dequantises in shared memory. The bf16 cache keeps every slot (the
    drafters and KV compaction address it by slot), so the saving is in the bytes attention reads."""

    config_class = KIVIConfig
    capabilities = Capability.KV_CACHE
    family = Family.KV_COMPRESSION
    lossless = False

    def __init__(self, config: KIVIConfig, model) -> None:
        super().__init__(config, model)
        self._store: dict[int, tuple[torch.Tensor, torch.Tensor]] = {}

    def attach(self) -> None:
        if self.model.kv_dtype is not None:
            raise ConfigError("kivi codes a bf16 cache; it cannot be combined with kv_fp8")
        if self.model.device.type == "cuda" and self.model.config.head_dim != 128:
            raise ConfigError(f"kivi's CUDA kernels code 128-dimensional heads, not {self.model.config.head_dim}")
        self.model.kv_quantizer = self

    def detach(self) -> None:
        self.model.kv_quantizer = None

    def storage(self, cache) -> tuple[torch.Tensor, torch.Tensor]:
        from ...ops.kivi import chunk_bytes

        key = id(cache.data)
        st = self._store.get(key)
        if getattr(cache, "paged", False):
            L, B, hkv, S, dim = cache.num_layers, cache.batch, cache.num_kv_heads, cache.capacity, cache.head_dim
        else:
            L, _, B, hkv, S, dim = cache.data.shape
        if st is None or st[0].shape[:4] != (L, B, hkv, S // 128):
            st = (torch.zeros(L, B, hkv, S // 128, chunk_bytes(self.config.bits, dim), dtype=torch.uint8,
                              device=cache.data.device),
                  torch.zeros(B, dtype=torch.int32, device=cache.data.device))
            self._store = {key: st}  # one live cache at a time
        return st

    def layer_args(self, layer: int, cache) -> dict:
        data, chunks = self.storage(cache)
        return {"kivi": data[layer], "kivi_chunks": chunks, "kivi_bits": self.config.bits}

    def reset(self, cache) -> None:
        self.storage(cache)[1].zero_()

    def after_commit(self, cache, kv_len: torch.Tensor, max_new: int = 1) -> None:
        from ... import ops

        data, chunks = self.storage(cache)
        ops.kivi_quantize(cache.data, data, kv_len.to(torch.int32), chunks, self.config.bits, self.config.residual,
                          max_new, pages=cache.tables)


@register_technique
class KIVIFusedTechnique(KIVITechnique):
    config_class = KIVIFusedConfig
