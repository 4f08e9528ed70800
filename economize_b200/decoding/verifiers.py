"""Verifiers: how the exact pass decides which drafts to keep (economize ``src/economize/decoding/verifiers.py``).

* ``greedy``: lossless for greedy decoding; a node is kept when it equals the target's argmax after its parent
  (chains and trees; the device kernel walks the tree).
* ``rejection``: lossless speculative sampling (chains): accept ``x ~ q`` with probability ``min(1, p(x)/q(x))``,
  resample from ``norm(max(0, p - q))`` at the first rejection; one fused device kernel.
* ``typical``: Medusa's typical acceptance (lossy): keep a node when the target gives it probability above
  ``min(threshold, alpha * exp(-entropy))``.
* ``accept_all``: keep every draft (lossy; the exact pass only refreshes the cache).
"""

from __future__ import annotations

from typing import Any, ClassVar

import torch

from ..errors import ConfigError
from ..registry import Registry

__all__ = ["VERIFIERS", "AcceptAllVerifier", "GreedyVerifier", "RejectionVerifier", "TypicalVerifier", "Verifier"]


class Verifier:
    name: ClassVar[str] = ""
    lossless: ClassVar[bool] = True
    supports_trees: ClassVar[bool] = True
    needs_draft_probs: ClassVar[bool] = False
    commits_drafts: ClassVar[bool] = False
    options: ClassVar[tuple[str, ...]] = ()

    def __init__(self, config: Any = None) -> None:
        opts = dict(getattr(config, "verifier_options", {}) or {})
        unknown = sorted(set(opts) - set(self.options))
        if unknown:
            raise ConfigError(f"verifier {self.name!r} has no options {unknown}; it takes {list(self.options)}")
        self.opts = opts


VERIFIERS: Registry[type[Verifier]] = Registry("verifier", "economize_b200.verifiers")


@VERIFIERS.register("greedy")
class GreedyVerifier(Verifier):
    name = "greedy"


@VERIFIERS.register("rejection")
class RejectionVerifier(Verifier):
    name = "rejection"
    supports_trees = False
    needs_draft_probs = True


@VERIFIERS.register("typical")
class TypicalVerifier(Verifier):
    name = "typical"
    lossless = False
    options = ("threshold", "alpha")

    def __init__(self, config: Any = None) -> None:
        super().__init__(config)
        self.threshold = float(self.opts.get("threshold", 0.09))
        self.alpha = float(self.opts.get("alpha", 0.3))
        if not (0 < self.threshold <= 1 and self.alpha > 0):
            raise ConfigError("typical acceptance needs 0 < threshold <= 1 and alpha > 0")

    def acceptable(self, probs_parent: torch.Tensor, tokens: torch.Tensor) -> torch.Tensor:
        """``[B, T]`` bools: node ``t``'s token has typical probability under its parent's distribution
        ``probs_parent [B, T, V]`` (the distribution after node ``t``'s parent, gathered per node)."""
        p_tok = probs_parent.gather(-1, tokens[..., None].clamp_min(0))[..., 0]
        entropy = -(probs_parent * torch.log(probs_parent.clamp_min(1e-20))).sum(-1)
        bound = torch.minimum(torch.full_like(entropy, self.threshold), self.alpha * torch.exp(-entropy))
        return p_tok > bound


@VERIFIERS.register("accept_all")
class AcceptAllVerifier(Verifier):
    name = "accept_all"
    lossless = False
    supports_trees = False
    commits_drafts = True
