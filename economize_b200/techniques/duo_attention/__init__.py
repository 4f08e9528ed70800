"""DuoAttention (``duo_attention``; Xiao et al., 2024; economize ``techniques/duo_attention``): each KV head is a
*retrieval* head (full cache) or a *streaming* head (attention sinks + a recent window). The reference trains
per-head gates; here the heads are ranked on calibration tokens by how much of their attention mass already falls
on the sinks and the recent window (measured with the tensor-core score kernel), and the ``streaming_ratio``
most concentrated heads become streaming heads. Streaming heads hide their other prompt slots through the attention
kernel's per-head keep bitmap.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import ClassVar

import torch

from ... import ops
from ...core.technique import Capability, Family, Technique, TechniqueConfig, register_technique
from ...errors import ConfigError
from ...runtime.cache import KVCache, StepBatch
from ..kv_evict import keep_words

__all__ = ["DuoAttentionConfig", "DuoAttentionTechnique"]


@dataclass(frozen=True)
class DuoAttentionConfig(TechniqueConfig):
    technique: ClassVar[str] = "duo_attention"
    streaming_ratio: float = 0.5
    sink: int = 16
    window: int = 64

    def __post_init__(self) -> None:
        if not 0.0 <= self.streaming_ratio <= 1.0:
            raise ConfigError("streaming_ratio must lie in [0, 1]")


@register_technique
class DuoAttentionTechnique(Technique):
    config_class = DuoAttentionConfig
    capabilities = Capability.KV_CACHE
    family = Family.KV_COMPRESSION
    lossless = False

    def __init__(self, config: DuoAttentionConfig, model) -> None:
        super().__init__(config, model)
        self._calibration = None
        self.register_buffer("streaming", torch.zeros(model.config.num_layers, model.local["num_kv_heads"],
                                                       dtype=torch.bool, device=model.device))
        self._chosen = False
        self.keep: torch.Tensor | None = None

    def calibrate(self, calibration) -> None:
        self._calibration = calibration

    def load_technique_state(self, state) -> None:
        super().load_technique_state(state)
        self._chosen = True

    @torch.no_grad()
    def _choose(self) -> None:
        cfg: DuoAttentionConfig = self.config
        m = self.model
        cal = self._calibration
        if cal is None:
            raise ConfigError("duo_attention needs calibration tokens to classify its heads")
        tokens = (cal if isinstance(cal, torch.Tensor) else torch.as_tensor(cal[0])).to(m.device)
        tokens = tokens[None] if tokens.dim() == 1 else tokens
        b, length = tokens.shape
        c = m.config
        mass = torch.zeros(c.num_layers, m.local["num_kv_heads"], device=m.device)
        recorder = _MassRecorder(cfg, mass)
        prev, m.kv_evictor = m.kv_evictor, recorder
        try:
            cache = KVCache(c.num_layers, b, m.local["num_kv_heads"], ((length + 127) // 128) * 128, c.head_dim,
                            m.dtype, m.device)
            lengths = torch.full((b,), length, dtype=torch.int32, device=m.device)
            m.forward_step(tokens, StepBatch.prefill(lengths, length), cache)
        finally:
            m.kv_evictor = prev
        n_stream = int(round(cfg.streaming_ratio * mass.numel()))
        flat = torch.zeros(mass.numel(), dtype=torch.bool, device=m.device)
        if n_stream:
            flat[mass.flatten().topk(n_stream).indices] = True
        self.streaming.copy_(flat.reshape(mass.shape))
        self._chosen = True

    def attach(self) -> None:
        if not self._chosen:
            self._choose()
        self.model.kv_evictor = self

    def detach(self) -> None:
        self.model.kv_evictor = None

    def keep_for(self, layer, k_cache, q=None, batch=None):
        if self.keep is None or self.keep.shape[3] * 32 != k_cache.shape[2]:
            return None
        return self.keep[layer]

    @torch.no_grad()
    def observe_prefill(self, layer, q, k_cache, v_cache, batch) -> None:
        cfg: DuoAttentionConfig = self.config
        b, hkv, s = k_cache.shape[0], k_cache.shape[1], k_cache.shape[2]
        n = self.model.config.num_layers
        if self.keep is None or self.keep.shape[1:] != (b, hkv, s // 32):
            self.keep = torch.full((n, b, hkv, s // 32), -1, dtype=torch.int32, device=q.device)
        slots = torch.arange(s, device=q.device)
        lengths = batch.n_new
        local = (slots[None] < cfg.sink) | (slots[None] >= lengths[:, None] - cfg.window)  # [B, S]
        keep = local[:, None] | ~self.streaming[layer][None, :, None]
        self.keep[layer] = keep_words(keep)


class _MassRecorder:
    """Calibration hook: the fraction of each KV head's attention mass (last ``window`` queries) on sinks + recent."""

    def __init__(self, cfg: DuoAttentionConfig, mass: torch.Tensor) -> None:
        self.cfg, self.mass = cfg, mass

    def keep_for(self, layer, k_cache, q=None, batch=None):
        return None

    def observe_prefill(self, layer, q, k_cache, v_cache, batch) -> None:
        cfg = self.cfg
        b, length, heads, _ = q.shape
        hkv, s = k_cache.shape[1], k_cache.shape[2]
        w = min(cfg.window, length)
        qw = q[:, length - w:].contiguous()
        zero = torch.zeros_like(batch.kv_len)
        lse = torch.empty(b, w, heads, dtype=torch.float32, device=q.device)
        ops.attention(qw, k_cache, v_cache, zero, batch.n_new, None, q_offset=length - w, lse_out=lse)
        scores = torch.zeros(b, hkv, s, dtype=torch.float32, device=q.device)
        ops.attention_scores(qw, k_cache, zero, batch.n_new, None, lse, scores, q_offset=length - w)
        slots = torch.arange(s, device=q.device)
        local = (slots[None] < cfg.sink) | (slots[None] >= batch.n_new[:, None] - cfg.window)
        self.mass[layer] = (scores * local[:, None]).sum((0, 2)) / scores.sum((0, 2)).clamp_min(1e-9)
