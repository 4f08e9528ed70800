"""Quest (``quest``; Tang et al., 2024; economize ``techniques/quest``): query-aware selection of KV pages. At the
prompt pass every ``page`` consecutive keys are summarised by their elementwise minimum and maximum; before each
later attention call the pass's queries (averaged over the pass and the GQA group) bound every page's best score
``sum_d max(q_d min_d, q_d max_d)`` and only the ``pages`` best prompt pages (plus the first and the most recent
page) stay visible, through the attention kernel's per-head keep bitmap. The selection is plain tensor algebra on
the device, so it runs inside captured cycles."""

from __future__ import annotations

from dataclasses import dataclass
from typing import ClassVar

import torch

from ...core.technique import Capability, Family, Technique, TechniqueConfig, register_technique
from ...errors import ConfigError
from ...validation import check_positive
from ..kv_evict import keep_words

__all__ = ["QuestConfig", "QuestTechnique"]


@dataclass(frozen=True)
class QuestConfig(TechniqueConfig):
    technique: ClassVar[str] = "quest"
    page: int = 16
    pages: int = 32

    def __post_init__(self) -> None:
        check_positive("page", self.page)
        check_positive("pages", self.pages)
        if 32 % self.page and self.page % 32:
            raise ConfigError("page must divide 32 or be a multiple of 32")


@register_technique
class QuestTechnique(Technique):
    config_class = QuestConfig
    capabilities = Capability.KV_CACHE
    family = Family.KV_COMPRESSION
    lossless = False

    def __init__(self, config: QuestConfig, model) -> None:
        super().__init__(config, model)
        self.kmin: list[torch.Tensor | None] = [None] * model.config.num_layers
        self.kmax: list[torch.Tensor | None] = [None] * model.config.num_layers
        self.prompt_len: torch.Tensor | None = None

    def attach(self) -> None:
        self.model.kv_evictor = self

    def detach(self) -> None:
        self.model.kv_evictor = None

    @torch.no_grad()
    def observe_prefill(self, layer, q, k_cache, v_cache, batch) -> None:
        b, hkv, s, d = k_cache.shape
        pages = s // self.config.page
        k = k_cache.float().reshape(b, hkv, pages, self.config.page, d)
        slots = torch.arange(s, device=q.device).reshape(pages, self.config.page)
        valid = (slots[None] < batch.n_new[:, None, None])[:, None, :, :, None]  # [B, 1, P, page, 1]
        self.kmin[layer] = torch.where(valid, k, torch.full_like(k, float("inf"))).amin(3)
        self.kmax[layer] = torch.where(valid, k, torch.full_like(k, float("-inf"))).amax(3)
        self.prompt_len = batch.n_new.clone()

    @torch.no_grad()
    def keep_for(self, layer, k_cache, q=None, batch=None):
        if q is None or batch is None or batch.is_prefill or self.kmin[layer] is None:
            return None
        kmin, kmax = self.kmin[layer], self.kmax[layer]
        b, hkv, s, _ = k_cache.shape
        if kmin.shape[2] * self.config.page != s:
            return None
        group = q.shape[2] // hkv
        qa = q.float().mean(1).reshape(b, hkv, group, -1).mean(2)  # [B, Hkv, D]
        bound = torch.maximum(qa[:, :, None] * kmin, qa[:, :, None] * kmax)
        score = torch.nan_to_num(bound, nan=0.0, posinf=0.0, neginf=0.0).sum(-1)  # [B, Hkv, P]
        pages = kmin.shape[2]
        page_start = torch.arange(pages, device=q.device) * self.config.page
        in_prompt = page_start[None] < self.prompt_len[:, None]  # [B, P]
        last = (self.prompt_len - 1).div(self.config.page, rounding_mode="floor")  # the most recent prompt page
        score = score.masked_fill(~in_prompt[:, None], float("-inf"))
        top = score.topk(min(self.config.pages, pages), -1).indices
        keep_p = torch.zeros(b, hkv, pages, dtype=torch.bool, device=q.device).scatter_(-1, top, True)
        keep_p[:, :, 0] = True
        keep_p.scatter_(-1, last.long()[:, None, None].expand(b, hkv, 1), True)
        keep = keep_p.repeat_interleave(self.config.page, -1)
        keep |= (torch.arange(s, device=q.device)[None] >= self.prompt_len[:, None])[:, None]  # generated tokens
        return keep_words(keep)
