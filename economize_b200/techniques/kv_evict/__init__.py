"""KV-cache eviction (``kv_evict``; economize ``techniques/kv_evict``, methods ``streaming``, ``h2o``,
``h2o_prefill``, ``snapkv``, ``pyramidkv`` at ``policies.py:165-343``).

During the prompt pass every layer scores its cached keys and keeps ``budget`` of them per KV head; later passes
do not see the evicted slots (the attention kernel ANDs a per-head keep bitmap into its visibility rule, so the
outputs are exactly those of attention over the kept keys). Scores come from the tensor cores: the layer's
observation queries are re-run through the attention kernel for their log-sum-exp, then ``attention_scores``
accumulates the normalised probability every key receives (the reference recomputes fp32 probabilities through a
``TorchFunctionMode`` tap, ``kv_evict/tap.py``).

* ``streaming`` (StreamingLLM): the first ``sink`` and the last ``budget - sink`` prompt tokens.
* ``h2o_prefill``: the heaviest hitters under the attention of every prompt query, plus the recent ``window``.
* ``h2o``: as ``h2o_prefill`` (generated tokens are never evicted in this engine: they stay visible).
* ``snapkv``: scores from the last ``window`` queries only, max-pooled over ``pool`` neighbouring slots.
* ``pyramidkv``: SnapKV with budgets that shrink linearly with depth (mean ``budget``, ratio ``pyramid_ratio``
  between the first and the last layer).

Evicted keys still occupy their slots (the cache is slot-addressed and shared with the drafters), so the saving is
in what attention reads as visible, not in memory.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import ClassVar

import torch
import torch.nn.functional as F

from ... import ops
from ...core.technique import Capability, Family, Technique, TechniqueConfig, register_technique
from ...errors import ConfigError
from ...validation import check_choice, check_positive

__all__ = ["KVEvictConfig", "KVEvictTechnique", "keep_words"]

METHODS = ("streaming", "h2o", "h2o_prefill", "snapkv", "pyramidkv")


@dataclass(frozen=True)
class KVEvictConfig(TechniqueConfig):
    technique: ClassVar[str] = "kv_evict"
    method: str = "snapkv"
    budget: int = 1024
    window: int = 32
    sink: int = 4
    pool: int = 7
    pyramid_ratio: float = 4.0

    def __post_init__(self) -> None:
        check_choice("method", self.method, METHODS)
        check_positive("budget", self.budget)
        check_positive("window", self.window)
        if self.pool < 1 or self.pool % 2 == 0:
            raise ConfigError("pool must be an odd positive size")
        if self.window > self.budget:
            raise ConfigError("window must not exceed budget")
        if self.pyramid_ratio < 1.0:
            raise ConfigError("pyramid_ratio must be >= 1")


def keep_words(keep: torch.Tensor) -> torch.Tensor:
    """Bool ``[..., S]`` (S a multiple of 32) -> int32 bit words ``[..., S / 32]`` (bit i of word w = slot 32 w + i)."""
    s = keep.shape[-1]
    bits = keep.reshape(*keep.shape[:-1], s // 32, 32).to(torch.int64)
    words = (bits << torch.arange(32, device=keep.device)).sum(-1)
    return torch.where(words >= 2 ** 31, words - 2 ** 32, words).to(torch.int32)


@register_technique
class KVEvictTechnique(Technique):
    config_class = KVEvictConfig
    capabilities = Capability.KV_CACHE
    family = Family.KV_COMPRESSION
    lossless = False

    def __init__(self, config: KVEvictConfig, model) -> None:
        super().__init__(config, model)
        self.keep: torch.Tensor | None = None  # [L, B, H_kv, S / 32] int32

    def attach(self) -> None:
        self.model.kv_evictor = self

    def detach(self) -> None:
        self.model.kv_evictor = None

    def layer_budget(self, layer: int) -> int:
        cfg: KVEvictConfig = self.config
        if cfg.method != "pyramidkv":
            return cfg.budget
        n = self.model.config.num_layers
        top = 2 * cfg.budget * cfg.pyramid_ratio / (1 + cfg.pyramid_ratio)  # linear from top to top / ratio
        low = top / cfg.pyramid_ratio
        return max(cfg.window, int(round(top - (top - low) * layer / max(n - 1, 1))))

    def keep_for(self, layer: int, k_cache: torch.Tensor, q=None, batch=None) -> torch.Tensor | None:
        if self.keep is None or self.keep.shape[1] != k_cache.shape[0] or self.keep.shape[3] * 32 != k_cache.shape[2]:
            return None
        return self.keep[layer]

    @torch.no_grad()
    def observe_prefill(self, layer: int, q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
                        batch) -> None:
        cfg: KVEvictConfig = self.config
        b, length, heads, dim = q.shape
        hkv, s = k_cache.shape[1], k_cache.shape[2]
        n = self.model.config.num_layers
        if self.keep is None or self.keep.shape[1:] != (b, hkv, s // 32) or layer == 0:
            if self.keep is None or self.keep.shape[1:] != (b, hkv, s // 32):
                self.keep = torch.full((n, b, hkv, s // 32), -1, dtype=torch.int32, device=q.device)
        lengths = batch.n_new
        slots = torch.arange(s, device=q.device)
        budget = self.layer_budget(layer)
        recent = (slots[None] >= (lengths[:, None] - cfg.window)) & (slots[None] < lengths[:, None])  # [B, S]
        if cfg.method == "streaming":  # attention sinks + the most recent (budget - sink) tokens
            tail = (slots[None] >= (lengths[:, None] - (budget - cfg.sink))) & (slots[None] < lengths[:, None])
            keep = (tail | (slots[None] < cfg.sink))[:, None].expand(b, hkv, s)
        else:
            w = length if cfg.method in ("h2o", "h2o_prefill") else min(cfg.window, length)
            qw = q[:, length - w:].contiguous()
            zero = torch.zeros_like(batch.kv_len)
            lse = torch.empty(b, w, heads, dtype=torch.float32, device=q.device)
            k_scale, v_scale = (None, None)
            if self.model.kv_scales is not None:
                k_scale, v_scale = self.model.kv_scales[0][layer], self.model.kv_scales[1][layer]
            if k_cache.dtype != q.dtype:
                raise ConfigError("kv_evict scores bf16 caches; apply it without kv_fp8")
            ops.attention(qw, k_cache, v_cache, zero, lengths, None, q_offset=length - w, lse_out=lse,
                          k_scale=k_scale, v_scale=v_scale)
            scores = torch.zeros(b, hkv, s, dtype=torch.float32, device=q.device)
            ops.attention_scores(qw, k_cache, zero, lengths, None, lse, scores, q_offset=length - w)
            if cfg.method in ("snapkv", "pyramidkv") and cfg.pool > 1:
                scores = F.max_pool1d(scores.reshape(b * hkv, 1, s), cfg.pool, 1, cfg.pool // 2).reshape(b, hkv, s)
            valid = slots[None] < lengths[:, None]  # [B, S]
            scores = scores.masked_fill(~valid[:, None], -1.0)
            scores = scores.masked_fill(recent[:, None], float("inf"))  # the recent window always stays
            k = min(budget, s)
            top = scores.topk(k, -1).indices
            keep = torch.zeros(b, hkv, s, dtype=torch.bool, device=q.device).scatter_(-1, top, True)
            keep &= valid[:, None]
        # prompts shorter than the budget keep everything
        short = (lengths <= budget)[:, None, None]
        keep = keep | (short & (slots[None, None] < lengths[:, None, None]))
        keep |= slots[None, None] >= lengths[:, None, None]  # slots after the prompt are never evicted
        self.keep[layer] = keep_words(keep)

    def kept_fraction(self, lengths: torch.Tensor) -> float:
        """Average fraction of prompt slots kept over layers, rows and heads."""
        if self.keep is None:
            return 1.0
        bits = ((self.keep.long()[..., None] >> torch.arange(32, device=self.keep.device)) & 1).reshape(
            *self.keep.shape[:3], -1)
        slots = torch.arange(bits.shape[-1], device=bits.device)
        prompt = slots[None] < lengths.to(bits.device)[:, None]  # [B, S]
        return float((bits.bool() & prompt[None, :, None]).sum() / (prompt.sum() * bits.shape[0] * bits.shape[2]))
