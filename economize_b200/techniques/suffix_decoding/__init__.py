"""SuffixDecoding (``suffix_decoding``; Oliaro et al., 2024; economize ``techniques/suffix_decoding``): draft trees
from suffix matches of the current context in a per-request index (prompt and generated tokens) and a global index
of earlier requests' outputs, weighting continuations by their frequency."""

from __future__ import annotations

from dataclasses import dataclass
from typing import ClassVar

from ...core.technique import TechniqueConfig, register_technique
from ...decoding.ngram_index import NGramIndex
from ...validation import check_positive
from .._retrieval import RetrievalTechnique

__all__ = ["SuffixDecodingConfig", "SuffixDecodingTechnique"]


@dataclass(frozen=True)
class SuffixDecodingConfig(TechniqueConfig):
    """``max_context`` longest suffix matched, ``max_depth`` tree depth, ``budget`` nodes per tree, ``branch``
    children per node, ``min_match`` shortest usable match, ``global_index`` whether finished requests feed the
    shared index."""

    technique: ClassVar[str] = "suffix_decoding"
    max_context: int = 16
    max_depth: int = 8
    budget: int = 24
    branch: int = 3
    min_match: int = 2
    global_index: bool = True

    def __post_init__(self) -> None:
        for name in ("max_context", "max_depth", "budget", "branch", "min_match"):
            check_positive(name, getattr(self, name))


@register_technique
class SuffixDecodingTechnique(RetrievalTechnique):
    config_class = SuffixDecodingConfig

    def __init__(self, config, model) -> None:
        super().__init__(config, model)
        self.global_index = NGramIndex(config.max_context)

    def add_corpus(self, sequences) -> None:
        """Feed finished outputs (or any token sequences) to the global index."""
        self.global_index.extend([list(map(int, s)) for s in sequences])

    def tree_for(self, row, local):
        c = self.config
        others = (self.global_index,) if c.global_index and self.global_index.size else ()
        return local.draft_tree(row, c.budget, c.max_depth, c.branch, c.min_match, others)
