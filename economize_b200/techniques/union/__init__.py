"""Union of retrieval drafters (``union``; economize ``techniques/union``): the draft tree merges the trees of
several host-side proposers (suffix matches of the request, a REST datastore), so a cycle verifies every
proposal in one pass. Nodes with the same path are shared; the budget is split evenly."""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, ClassVar

from ...core.technique import TechniqueConfig, register_technique
from ...decoding.ngram_index import NGramIndex
from ...errors import ConfigError
from ...validation import check_positive
from .._retrieval import RetrievalTechnique

__all__ = ["UnionConfig", "UnionTechnique", "merge_trees"]


@dataclass(frozen=True)
class UnionConfig(TechniqueConfig):
    technique: ClassVar[str] = "union"
    max_context: int = 16
    max_depth: int = 6
    budget: int = 32
    branch: int = 3
    min_match: int = 2
    corpus: Any = None

    def __post_init__(self) -> None:
        for name in ("max_context", "max_depth", "budget", "branch", "min_match"):
            check_positive(name, getattr(self, name))

    def to_dict(self) -> dict[str, Any]:
        out = super().to_dict()
        out["corpus"] = None
        return out


def merge_trees(trees: list[tuple[list[int], list[int]]], budget: int) -> tuple[list[int], list[int]]:
    """Merge trees (tokens, parents) by path, round-robin over the inputs until ``budget`` nodes."""
    index: dict[tuple[int, ...], int] = {}
    tokens, parents = [], []
    paths = []
    for t, p in trees:
        pt = []
        for tok, par in zip(t, p):
            pt.append((pt[par] if par >= 0 else ()) + (tok,))
        paths.append(pt)
    i = 0
    while len(tokens) < budget and any(i < len(pt) for pt in paths):
        for pt in paths:
            if i < len(pt) and len(tokens) < budget:
                path = pt[i]
                if path in index or (len(path) > 1 and path[:-1] not in index):
                    continue
                index[path] = len(tokens)
                tokens.append(path[-1])
                parents.append(index[path[:-1]] if len(path) > 1 else -1)
        i += 1
    return tokens, parents


@register_technique
class UnionTechnique(RetrievalTechnique):
    config_class = UnionConfig

    def __init__(self, config: UnionConfig, model) -> None:
        super().__init__(config, model)
        self.datastore = NGramIndex(config.max_context)
        if config.corpus is not None:
            self.datastore.extend([list(map(int, s)) for s in config.corpus])

    def calibrate(self, calibration) -> None:
        if self.datastore.size == 0:
            self.datastore.extend([list(map(int, s)) for s in calibration.reshape(-1, calibration.shape[-1])])

    def attach(self) -> None:
        if self.datastore.size == 0:
            raise ConfigError("union needs a datastore for its retrieval member: pass corpus= or calibration")

    def tree_for(self, row, local):
        c = self.config
        half = max(1, c.budget // 2)
        a = local.draft_tree(row, half, c.max_depth, c.branch, c.min_match)
        b = self.datastore.draft_tree(row, half, c.max_depth, c.branch, c.min_match)
        return merge_trees([a, b], c.budget)
