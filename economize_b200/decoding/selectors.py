"""Token selection rules (economize ``src/economize/decoding/selectors.py``): greedy and top-p/top-k sampling."""

from __future__ import annotations

from dataclasses import dataclass

import torch

from ..errors import ConfigError

__all__ = ["GreedySelector", "TokenSelector", "TopPSampler"]


class TokenSelector:
    """Turns logits into tokens; ``greedy`` selectors run on the graph-captured greedy engine."""

    greedy: bool = True

    def probs(self, logits: torch.Tensor) -> torch.Tensor:
        raise NotImplementedError

    def select(self, logits: torch.Tensor, generator: torch.Generator | None = None) -> torch.Tensor:
        raise NotImplementedError


@dataclass
class GreedySelector(TokenSelector):
    greedy: bool = True

    def probs(self, logits: torch.Tensor) -> torch.Tensor:
        return torch.nn.functional.one_hot(logits.argmax(-1), logits.shape[-1]).float()

    def select(self, logits: torch.Tensor, generator: torch.Generator | None = None) -> torch.Tensor:
        return logits.argmax(-1)


@dataclass
class TopPSampler(TokenSelector):
    """Temperature + nucleus (top-p) + top-k sampling."""

    temperature: float = 1.0
    top_p: float = 1.0
    top_k: int = 0
    seed: int | None = None

    def __post_init__(self) -> None:
        if not self.temperature > 0:
            raise ConfigError(f"temperature must be positive, got {self.temperature}")
        if not 0 < self.top_p <= 1:
            raise ConfigError(f"top_p must lie in (0, 1], got {self.top_p}")
        self.greedy = False

    def probs(self, logits: torch.Tensor) -> torch.Tensor:
        x = logits.float() / self.temperature
        if self.top_k > 0:
            kth = x.topk(min(self.top_k, x.shape[-1]), -1).values[..., -1:]
            x = x.masked_fill(x < kth, float("-inf"))
        p = torch.softmax(x, -1)
        if self.top_p < 1:
            sp, si = p.sort(-1, descending=True)
            drop = sp.cumsum(-1) - sp > self.top_p
            sp = sp.masked_fill(drop, 0)
            p = torch.zeros_like(p).scatter(-1, si, sp)
            p = p / p.sum(-1, keepdim=True)
        return p

    def select(self, logits: torch.Tensor, generator: torch.Generator | None = None) -> torch.Tensor:
        p = self.probs(logits)
        flat = p.reshape(-1, p.shape[-1])
        return torch.multinomial(flat, 1, generator=generator).reshape(p.shape[:-1])
