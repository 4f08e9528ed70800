"""Retrieval-based speculative decoding (``rest``; He et al., 2024; economize ``techniques/rest`` and the shared
``techniques/retrieval`` datastore): draft trees are the most frequent continuations, in a token datastore, of the
longest suffix of the context found there. The datastore is a persistent suffix-array index
(:class:`~economize_b200.techniques.retrieval.SuffixIndex`, ``datastore=`` a folder or an index), or is built in
memory from ``corpus`` sequences (or calibration tokens); generation does not modify it."""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, ClassVar

import torch

from ...core.technique import TechniqueConfig, register_technique
from ...decoding.ngram_index import NGramIndex
from ...errors import ConfigError
from ...validation import check_positive
from .._retrieval import RetrievalTechnique

__all__ = ["RestConfig", "RestTechnique"]


@dataclass(frozen=True)
class RestConfig(TechniqueConfig):
    technique: ClassVar[str] = "rest"
    max_context: int = 16
    max_depth: int = 6
    budget: int = 32
    branch: int = 4
    min_match: int = 2
    corpus: Any = None
    datastore: Any = None

    def __post_init__(self) -> None:
        for name in ("max_context", "max_depth", "budget", "branch", "min_match"):
            check_positive(name, getattr(self, name))

    def to_dict(self) -> dict[str, Any]:
        out = super().to_dict()
        out["corpus"] = None  # the datastore is rebuilt from the corpus, not serialised in the config
        if not isinstance(self.datastore, (str, type(None))):
            out["datastore"] = None  # an in-memory index: save it and pass its folder to reload
        else:
            out["datastore"] = self.datastore
        return out


@register_technique
class RestTechnique(RetrievalTechnique):
    config_class = RestConfig
    uses_local = False

    def __init__(self, config: RestConfig, model) -> None:
        super().__init__(config, model)
        self.datastore = NGramIndex(config.max_context)
        self.index = None  # a persistent suffix-array datastore, when configured
        if config.datastore is not None:
            from ..retrieval import SuffixIndex

            ds = config.datastore
            self.index = ds if isinstance(ds, SuffixIndex) else SuffixIndex.load(ds, mmap=True)
        if config.corpus is not None:
            self._build(config.corpus)

    def _build(self, corpus) -> None:
        seqs = corpus if not isinstance(corpus, torch.Tensor) else list(corpus.reshape(-1, corpus.shape[-1]))
        self.datastore.extend([list(map(int, s)) for s in seqs])

    def calibrate(self, calibration) -> None:
        if self.datastore.size == 0:
            self._build(calibration if not isinstance(calibration, torch.Tensor) else
                        calibration.reshape(-1, calibration.shape[-1]))

    def attach(self) -> None:
        if self.index is None and self.datastore.size == 0:
            raise ConfigError("rest needs a datastore: pass datastore=, corpus= or calibration tokens")

    def tree_for(self, row, local):
        c = self.config
        if self.index is not None:
            return self.index.draft_tree(row, c.budget, c.max_depth, c.branch, c.min_match, c.max_context)
        return self.datastore.draft_tree(row, c.budget, c.max_depth, c.branch, c.min_match)
