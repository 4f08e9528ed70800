"""Shared base of the host-side retrieval drafters (``suffix_decoding``, ``rest``, ``lookahead``, ``union``).

They propose a static draft tree per row from :class:`~economize_b200.decoding.ngram_index.NGramIndex` lookups on
the host, so their cycles run without CUDA graphs (the engine checks ``graph_safe``); verification, acceptance and
KV compaction stay on the device kernels. Economize's retrieval drafters: ``techniques/rest``,
``techniques/suffix_decoding``, ``techniques/lookahead``, ``techniques/retrieval``.
"""

from __future__ import annotations

import torch

from ..core.technique import Capability, Family, Technique
from ..decoding.config import DecodeConfig
from ..decoding.ngram_index import NGramIndex, trees_to_tensors

__all__ = ["HostTreeDrafter", "RetrievalTechnique"]


class HostTreeDrafter:
    """Engine-side static proposer backed by host indexes."""

    observes = False
    graph_safe = False
    capture_layers: tuple[int, ...] = ()
    carry_size = 0

    def __init__(self, technique: RetrievalTechnique) -> None:
        self.t = technique
        self.local: list[NGramIndex] = []
        self.indexed: list[int] = []

    def begin(self, batch: int, capacity: int) -> None:
        self.local = [NGramIndex(self.t.config.max_context) for _ in range(batch)]
        self.indexed = [0] * batch

    def draft_depth(self, decode: DecodeConfig) -> int:
        return self.t.config.max_depth

    def draft_nodes(self, decode: DecodeConfig) -> int:
        return self.t.config.budget

    def propose(self, history: torch.Tensor, length: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        hist = history.cpu()
        lens = length.cpu().tolist()
        trees = []
        for b, n in enumerate(lens):
            row = hist[b, :n].tolist()
            if self.t.uses_local:
                self.local[b].add(row, self.indexed[b])
                self.indexed[b] = n
            trees.append(self.t.tree_for(row, self.local[b] if self.t.uses_local else None))
        return trees_to_tensors(trees, self.t.config.budget, history.device)

    def to_target(self, ids: torch.Tensor) -> torch.Tensor:
        return ids


class RetrievalTechnique(Technique):
    capabilities = Capability.DRAFTER
    family = Family.DRAFTER
    lossless = True
    graph_safe = False
    uses_local = True

    def tree_for(self, row: list[int], local: NGramIndex | None) -> tuple[list[int], list[int]]:
        raise NotImplementedError

    def drafter(self) -> HostTreeDrafter:
        return HostTreeDrafter(self)

    def default_decoding(self) -> DecodeConfig:
        return DecodeConfig(cycle_length=self.config.max_depth + 1)
