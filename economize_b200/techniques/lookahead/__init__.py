"""Lookahead-style n-gram pool drafting (``lookahead``; Fu et al., 2024; economize ``techniques/lookahead``):
candidate n-grams that start with the last token are drawn from a pool and verified as a tree. Lookahead decoding
fills its pool from a Jacobi-iteration branch computed in the same forward pass; this engine fills the pool from
the request's own prompt and output (every n-gram of up to ``ngram`` tokens), so the pool is exact text the
request has already seen and costs no extra FLOPs."""

from __future__ import annotations

from dataclasses import dataclass
from typing import ClassVar

from ...core.technique import TechniqueConfig, register_technique
from ...validation import check_positive
from .._retrieval import RetrievalTechnique

__all__ = ["LookaheadConfig", "LookaheadTechnique"]


@dataclass(frozen=True)
class LookaheadConfig(TechniqueConfig):
    """``ngram`` length of pooled n-grams (the draft depth is ``ngram - 1``), ``candidates`` n-grams verified per
    cycle."""

    technique: ClassVar[str] = "lookahead"
    ngram: int = 5
    candidates: int = 7

    def __post_init__(self) -> None:
        check_positive("ngram", self.ngram)
        check_positive("candidates", self.candidates)

    @property
    def max_context(self) -> int:
        return 1

    @property
    def max_depth(self) -> int:
        return max(1, self.ngram - 1)

    @property
    def budget(self) -> int:
        return self.candidates * max(1, self.ngram - 1)


@register_technique
class LookaheadTechnique(RetrievalTechnique):
    config_class = LookaheadConfig

    def tree_for(self, row, local):
        c = self.config
        # candidates: the most frequent continuations of the last token, each extended greedily (a chain per
        # candidate); chains share their first node when they start alike (the tree merges common prefixes)
        return local.draft_tree(row, c.budget, c.max_depth, branch=c.candidates, min_match=1)
