"""Static layer skipping for self-speculative decoding (``layer_skip``): the draft is the target with a set of
layers skipped (Draft & Verify, Zhang et al. 2024; SWIFT, Xia et al. 2025). Economize: ``techniques/layer_skip``
with its ``SKIP_SEARCHES`` registry.

Skip sets come from ``skip`` (1-indexed layers) or a registered search over calibration tokens:

* ``"influence"``: skip the ``ratio`` of layers with the lowest ShortGPT block influence (1 - cos of the layer's
  input and output residual streams);
* ``"interleave"``: skip every other layer of the middle ``2 * ratio`` of the depth (no data needed);
* ``"greedy"``: add one layer at a time, each time the one whose removal keeps the final hidden states closest
  (cosine) to the full model's on the calibration tokens.
"""

from __future__ import annotations

from collections.abc import Callable
from dataclasses import dataclass
from typing import ClassVar

import torch

from ...core.technique import TechniqueConfig, register_technique
from ...errors import ConfigError
from ...registry import Registry
from ...runtime.cache import StepBatch
from .._self_draft import SelfDraftTechnique, block_influence, layer_view

__all__ = ["LayerSkipConfig", "LayerSkipTechnique", "SKIP_SEARCHES"]

SKIP_SEARCHES: Registry[Callable] = Registry("skip search", "economize_b200.skip_searches")


@dataclass(frozen=True)
class LayerSkipConfig(TechniqueConfig):
    technique: ClassVar[str] = "layer_skip"
    skip: tuple[int, ...] = ()
    search: str = "influence"
    ratio: float = 0.4
    keep_first: int = 1
    keep_last: int = 1

    def __post_init__(self) -> None:
        object.__setattr__(self, "skip", tuple(int(i) for i in self.skip))
        if not 0.0 < self.ratio < 1.0:
            raise ConfigError(f"ratio must lie in (0, 1), got {self.ratio}")
        if not self.skip:
            SKIP_SEARCHES.get(self.search)
        if any(i < 1 for i in self.skip):
            raise ConfigError("skip lists 1-indexed layers")

    def validate(self, model) -> None:
        n = model.config.num_layers
        if any(i > n for i in self.skip):
            raise ConfigError(f"skip {self.skip} exceeds the model's {n} layers")


def _candidates(n: int, cfg: LayerSkipConfig) -> list[int]:
    return list(range(cfg.keep_first, n - cfg.keep_last))


@SKIP_SEARCHES.register("interleave")
def interleave(model, cfg: LayerSkipConfig, batches) -> list[int]:
    n = model.config.num_layers
    want = max(1, int(round(cfg.ratio * n)))
    cand = _candidates(n, cfg)
    mid = len(cand) // 2
    span = cand[max(0, mid - want): mid + want]
    return span[::2][:want]


@SKIP_SEARCHES.register("influence")
def influence(model, cfg: LayerSkipConfig, batches) -> list[int]:
    n = model.config.num_layers
    want = max(1, int(round(cfg.ratio * n)))
    bi = block_influence(model, batches)
    cand = _candidates(n, cfg)
    return sorted(sorted(cand, key=lambda i: float(bi[i]))[:want])


@torch.no_grad()
def _final_states(model, batches):
    outs = []
    for tokens in batches:
        tokens = torch.as_tensor(tokens).to(model.device)
        tokens = tokens[None] if tokens.dim() == 1 else tokens
        b, length = tokens.shape
        cache = model.new_cache(b, ((length + 127) // 128) * 128)
        lengths = torch.full((b,), length, dtype=torch.int32, device=model.device)
        h, _ = model.forward_step(tokens, StepBatch.prefill(lengths, length), cache)
        outs.append(h.float().reshape(-1, h.shape[-1]))
    return torch.cat(outs)


@SKIP_SEARCHES.register("greedy")
def greedy(model, cfg: LayerSkipConfig, batches) -> list[int]:
    n = model.config.num_layers
    want = max(1, int(round(cfg.ratio * n)))
    ref = _final_states(model, batches)
    skipped: list[int] = []
    for _ in range(want):
        best, best_i = -2.0, None
        for i in _candidates(n, cfg):
            if i in skipped:
                continue
            keep = [j for j in range(n) if j not in skipped and j != i]
            h = _final_states(layer_view(model, keep), batches)
            score = float(torch.nn.functional.cosine_similarity(h, ref, dim=-1).mean())
            if score > best:
                best, best_i = score, i
        skipped.append(best_i)
    return sorted(skipped)


@register_technique
class LayerSkipTechnique(SelfDraftTechnique):
    config_class = LayerSkipConfig

    def view_layers(self) -> list[int]:
        cfg: LayerSkipConfig = self.config
        n = self.model.config.num_layers
        if cfg.skip:
            skipped = [i - 1 for i in cfg.skip]
        else:
            batches = [] if cfg.search == "interleave" else self.calibration_batches()
            skipped = SKIP_SEARCHES.get(cfg.search)(self.model, cfg, batches)
        self.skipped = sorted(skipped)
        return [i for i in range(n) if i not in set(skipped)]
