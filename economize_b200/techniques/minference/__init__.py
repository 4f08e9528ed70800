"""MInference (``minference``; Jiang et al., NeurIPS 2024; economize ``techniques/minference``,
``attention/minference.py``): long prompts attend over a sparse pattern fitted to the prompt at prefill.

A prompt of at least ``min_queries`` tokens is prefilled in query chunks of ``chunk`` tokens. Every chunk attends
densely (causally) to itself and, among the earlier keys, only to the keys its pattern keeps; the pattern is written
into the attention kernel's per-KV-head keep bitmap, and the kernel skips every 128-key chunk the bitmap hides
entirely, which is where the prefill saves compute. Patterns (one for every head, the union over a GQA group):

* ``"a_shape"``: the first ``sinks`` keys and a local window of ``local`` keys before the chunk;
* ``"vertical_slash"``: the ``vertical`` key columns and the ``slash`` diagonals (offsets ``q - k``) that receive the
  most attention from the chunk's last 64 queries (estimated in fp32 from the cached keys), plus the first 30
  columns and the 100 diagonals nearest the main one; a diagonal keeps the keys it crosses for the chunk's queries;
* ``"block_sparse"``: the ``top_k`` blocks of 64 keys whose mean-pooled key has the largest product with the chunk's
  mean-pooled query.

A pattern holds for a whole chunk (the union over its queries), so it keeps at least the keys the per-query
pattern keeps. Decoding steps attend densely and the cache keeps every entry. Not built: per-head pattern files.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import ClassVar

import torch

from ... import ops
from ...core.technique import Capability, Family, Technique, TechniqueConfig, register_technique
from ...errors import ConfigError
from ...runtime.cache import StepBatch
from ...validation import check_choice, check_positive
from ..kv_evict import keep_words

__all__ = ["MInferenceConfig", "MInferencePrefill", "MInferenceTechnique", "PATTERNS"]

PATTERNS = ("vertical_slash", "block_sparse", "a_shape")


@dataclass(frozen=True)
class MInferenceConfig(TechniqueConfig):
    technique: ClassVar[str] = "minference"
    pattern: str = "vertical_slash"
    pattern_file: str | None = None
    vertical: int = 1000
    slash: int = 6096
    top_k: int = 100
    sinks: int = 128
    local: int = 3968
    dense_layers: int = 0
    layers: tuple[int, ...] = ()
    min_queries: int = 65
    ratio: float = 1.0
    chunk: int = 1024

    def __post_init__(self) -> None:
        check_choice("pattern", self.pattern, PATTERNS)
        if self.pattern_file is not None:
            raise ConfigError("minference pattern files (per-head patterns of an offline search) are not read by "
                              "this build; give pattern=")
        if self.vertical < 0 or self.slash < 1 or self.sinks < 0 or self.local < 1:
            raise ConfigError("minference needs vertical >= 0, slash >= 1, sinks >= 0 and local >= 1")
        check_positive("top_k", self.top_k)
        check_positive("min_queries", self.min_queries)
        check_positive("ratio", self.ratio)
        if self.chunk < 128 or self.chunk % 128:
            raise ConfigError("chunk must be a positive multiple of 128 (the attention kernel's key chunk)")
        object.__setattr__(self, "layers", tuple(self.layers))


class MInferencePrefill:
    """The model's sparse-prefill hook: :meth:`chunked_forward` runs a long prefill as query chunks and
    :meth:`keep_for` gives each chunk's keep bitmap."""

    def __init__(self, config: MInferenceConfig, model) -> None:
        self.config = config
        n = model.config.num_layers
        chosen = [i - 1 for i in config.layers] if config.layers else range(n)
        self.layers = {i for i in chosen if i >= config.dense_layers}
        self.active = False
        self.group = model.config.num_heads // model.config.num_kv_heads

    def covers(self, tokens: torch.Tensor, batch: StepBatch) -> bool:
        return batch.is_prefill and tokens.shape[1] >= max(self.config.min_queries, self.config.chunk + 1)

    def chunked_forward(self, model, tokens, batch: StepBatch, cache, capture):
        b, width = tokens.shape
        lengths = batch.n_new.long().to(tokens.device)
        outs, auxes = [], []
        self.active = True
        try:
            for start in range(0, width, self.config.chunk):
                end = min(width, start + self.config.chunk)
                kv = torch.full((b,), start, dtype=torch.int32, device=tokens.device)
                n = (lengths - start).clamp(0, end - start).to(torch.int32)
                pos = torch.arange(start, end, device=tokens.device, dtype=torch.int32).expand(b, end - start)
                h, a = model.forward_step(tokens[:, start:end], StepBatch(kv, n, pos.contiguous(), prompt=True), cache,
                                          capture)
                outs.append(h)
                auxes.append(a)
        finally:
            self.active = False
        return torch.cat(outs, 1), {k: torch.cat([a[k] for a in auxes], 1) for k in auxes[0]}

    # ---- patterns ------------------------------------------------------------------------------------------------
    @torch.no_grad()
    def keep_for(self, index: int, k_cache: torch.Tensor, q: torch.Tensor, batch: StepBatch):
        if index not in self.layers:
            return None
        c = self.config
        b, hkv, s, d = k_cache.shape
        base = int(batch.kv_len.max())  # the chunk's first position (the same for every row)
        if base == 0:
            return None  # the first chunk has no earlier keys
        t = q.shape[1]
        dev = k_cache.device
        pos = torch.arange(s, device=dev)
        keep = torch.zeros(b, hkv, s, dtype=torch.bool, device=dev)
        if c.pattern == "a_shape":
            keep |= (pos < c.sinks)[None, None]
            keep |= ((pos >= base - c.local) & (pos < base))[None, None]
        elif c.pattern == "vertical_slash":
            return self._vertical_slash(k_cache, q, base, t)
        else:
            keep |= self._block_sparse(k_cache, q, base)
        return keep_words(keep)

    def _scores(self, k_cache, q, base: int, last: int):
        """fp32 softmax of the chunk's last ``last`` queries over the keys ``< base + t`` (causal), per KV head:
        ``[B, Hkv, G * last, base + t]``."""
        b, hkv, s, d = k_cache.shape
        t = q.shape[1]
        qs = q[:, -last:].float()  # [B, L, H, D]
        g = self.group
        qs = qs.reshape(b, last, hkv, g, d).permute(0, 2, 3, 1, 4).reshape(b, hkv, g * last, d)
        keys = k_cache[:, :, : base + t].float()
        scores = qs @ keys.transpose(-1, -2) / d ** 0.5
        qpos = base + t - last + torch.arange(last, device=q.device)
        causal = torch.arange(base + t, device=q.device)[None] <= qpos[:, None]  # [L, S']
        scores = scores.masked_fill(~causal.repeat(g, 1)[None, None], -float("inf"))
        return torch.softmax(scores, -1), qpos

    def _vertical_slash(self, k_cache, q, base: int, t: int) -> torch.Tensor:
        c = self.config
        b, hkv, s, d = k_cache.shape
        dev = k_cache.device
        last = min(64, t)
        probs, qpos = self._scores(k_cache, q, base, last)  # [B, Hkv, G L, S']
        width = probs.shape[-1]
        nv = min(width, max(int(c.vertical * c.ratio), 30))
        vert = probs.sum(2)  # [B, Hkv, S']
        vert[..., :30] = float("inf")  # the first 30 columns always stay
        cols = vert.topk(nv, -1).indices
        # diagonals: offset o = q - k, summed over the estimating queries
        g = self.group
        off = (qpos.repeat(g)[:, None] - torch.arange(width, device=dev)[None])  # [G L, S']
        valid = off >= 0
        slash = torch.zeros(b, hkv, width, device=dev)
        slash.scatter_add_(2, off.clamp_min(0)[None, None].expand(b, hkv, -1, -1).reshape(b, hkv, -1),
                           (probs * valid[None, None]).reshape(b, hkv, -1))
        slash[..., :100] = float("inf")  # the 100 diagonals nearest the main one
        ns = min(width, max(int(c.slash * c.ratio), 50))
        offsets = slash.topk(ns, -1).indices  # [B, Hkv, ns]
        # columns and the keys [base - o, base + t - o) each diagonal crosses for the chunk's queries, as bit words
        # (a kernel on CUDA); only keys before the chunk are read through the pattern
        return ops.vs_keep(cols, offsets, base, t, base, s)

    def _block_sparse(self, k_cache, q, base: int) -> torch.Tensor:
        c = self.config
        b, hkv, s, d = k_cache.shape
        dev = k_cache.device
        nb = (base + 63) // 64
        keys = k_cache[:, :, : nb * 64].float().reshape(b, hkv, nb, 64, d)
        valid = (torch.arange(nb * 64, device=dev) < base).reshape(nb, 64)
        pooled_k = (keys * valid[None, None, :, :, None]).sum(3) / valid.sum(1).clamp_min(1)[None, None, :, None]
        g = self.group
        pooled_q = q.float().mean(1).reshape(b, hkv, g, d).mean(2)  # [B, Hkv, D]
        score = (pooled_k @ pooled_q[..., None])[..., 0]  # [B, Hkv, nb]
        top = score.topk(min(nb, c.top_k), -1).indices
        blocks = torch.zeros(b, hkv, nb, dtype=torch.bool, device=dev).scatter_(2, top, True)
        keep = torch.zeros(b, hkv, s, dtype=torch.bool, device=dev)
        keep[..., : nb * 64] = blocks.repeat_interleave(64, -1)
        return keep & (torch.arange(s, device=dev) < base)[None, None]


@register_technique
class MInferenceTechnique(Technique):
    config_class = MInferenceConfig
    capabilities = Capability.KV_CACHE
    family = Family.OTHER
    lossless = False

    def attach(self) -> None:
        self.model.prefill_sparsity = MInferencePrefill(self.config, self.model)

    def detach(self) -> None:
        self.model.prefill_sparsity = None
