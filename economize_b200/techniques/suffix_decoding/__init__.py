"""SuffixDecoding (``suffix_decoding``; Oliaro et al., NeurIPS 2025; economize ``techniques/suffix_decoding``).

Drafts come from suffix tries (:mod:`.trie`): a global one over a datastore of earlier responses and a local one per
row over its own prompt and output. Each cycle matches the longest suffix of the row's context in both, speculates
below the match by empirical continuation probability (a path, or a best-first tree), limits the draft to
``min(max_spec_tokens, floor(max_spec_factor * m + max_spec_offset))`` tokens for a match of ``m`` tokens, and keeps
the draft with the larger summed probability (the longer match, then the local draft, on ties). No network runs.

    model = economize_b200.apply(target, SuffixDecodingConfig(tree=True), decoding=DecodeConfig(cycle_length=9))
    model.techniques["suffix_decoding"].add_corpus(earlier_outputs)   # or datastore="responses.jsonl"
"""

from __future__ import annotations

import json
import os
from dataclasses import dataclass
from typing import ClassVar

import torch

from ...core.technique import TechniqueConfig, register_technique
from ...decoding.config import DecodeConfig
from ...decoding.ngram_index import trees_to_tensors
from ...errors import ConfigError
from ...validation import check_positive
from .._retrieval import HostTreeDrafter, RetrievalTechnique
from .trie import Speculation, SuffixTrie

__all__ = ["Speculation", "SuffixDecodingConfig", "SuffixDecodingTechnique", "SuffixTrie", "load_datastore"]


@dataclass(frozen=True)
class SuffixDecodingConfig(TechniqueConfig):
    """Hyperparameters of SuffixDecoding (field names of economize's ``SuffixDecodingConfig``).

    Attributes:
        datastore: Token sequences of earlier responses for the global trie: a ``.jsonl`` file of token-id lists
            (one per line) or a ``.pt`` file of a list of 1-D tensors; ``None``: only :meth:`add_corpus` feeds it.
        local: Also match the row's own prompt and output.
        max_depth: Longest substring the tries hold (match plus continuation).
        max_spec_factor / max_spec_offset: The adaptive draft length ``floor(factor * match + offset)``.
        min_token_prob: Smallest probability of a drafted token.
        tree: Draft a best-first tree; otherwise the most frequent path.
        max_spec_tokens: Most draft tokens (``None``: the cycle's ``cycle_length - 1``).
    """

    technique: ClassVar[str] = "suffix_decoding"

    datastore: str | None = None
    local: bool = True
    max_depth: int = 64
    max_spec_factor: float = 1.0
    max_spec_offset: float = 0.0
    min_token_prob: float = 0.1
    tree: bool = False
    max_spec_tokens: int | None = None

    def __post_init__(self) -> None:
        if self.max_depth < 2:
            raise ConfigError(f"max_depth counts the tokens of a trie path (match and draft): at least 2, "
                              f"got {self.max_depth}")
        if isinstance(self.max_spec_factor, bool) or not isinstance(self.max_spec_factor, (int, float)) \
                or self.max_spec_factor < 0:
            raise ConfigError(f"max_spec_factor scales the match length and cannot be negative: "
                              f"{self.max_spec_factor!r}")
        if isinstance(self.max_spec_offset, bool) or not isinstance(self.max_spec_offset, (int, float)):
            raise ConfigError(f"max_spec_offset must be a number, got {self.max_spec_offset!r}")
        if not 0.0 < float(self.min_token_prob) <= 1.0:
            raise ConfigError(f"min_token_prob is a probability in (0, 1], got {self.min_token_prob!r}")
        if self.max_spec_tokens is not None:
            check_positive("max_spec_tokens", self.max_spec_tokens)

    def validate(self, model) -> None:
        if not self.local and not self.datastore:
            pass  # the global trie may still be fed through add_corpus before decoding


def load_datastore(path: str) -> list[list[int]]:
    """Token sequences of a datastore file (``.jsonl`` lines of id lists, or a ``.pt`` list of tensors/lists)."""
    if not os.path.exists(path):
        raise ConfigError(f"suffix_decoding datastore {path!r} does not exist")
    if path.endswith(".pt"):
        data = torch.load(path, map_location="cpu", weights_only=True)
        return [list(map(int, seq.tolist() if isinstance(seq, torch.Tensor) else seq)) for seq in data]
    with open(path) as fh:
        return [list(map(int, json.loads(line))) for line in fh if line.strip()]


class SuffixDrafter(HostTreeDrafter):
    """One local trie per row, extended with the tokens each row committed since the last cycle."""

    def begin(self, batch: int, capacity: int) -> None:
        self.tries = [SuffixTrie(self.t.config.max_depth) for _ in range(batch)]
        self.indexed = [0] * batch

    def draft_depth(self, decode: DecodeConfig) -> int:
        return self.t.max_tokens(decode)

    def draft_nodes(self, decode: DecodeConfig) -> int:
        return self.t.max_tokens(decode)

    def propose(self, history: torch.Tensor, length: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        hist = history.cpu()
        trees = []
        for b, n in enumerate(length.cpu().tolist()):
            row = hist[b, :n].tolist()
            if self.t.config.local:
                self.tries[b].append(row[self.indexed[b]:n])
                self.indexed[b] = n
            best = self.t.speculate(row, self.tries[b] if self.t.config.local else None)
            trees.append((list(best.tokens), list(best.parents)))
        return trees_to_tensors(trees, self.t.budget, history.device)


@register_technique
class SuffixDecodingTechnique(RetrievalTechnique):
    config_class = SuffixDecodingConfig

    def __init__(self, config: SuffixDecodingConfig, model) -> None:
        super().__init__(config, model)
        self.global_trie = SuffixTrie(config.max_depth)
        self.budget = config.max_spec_tokens or 8
        if config.datastore:
            self.add_corpus(load_datastore(config.datastore))

    def add_corpus(self, sequences) -> None:
        """Index finished outputs (or any token sequences) in the global trie."""
        for seq in sequences:
            self.global_trie.add_sequence([int(t) for t in seq])

    def max_tokens(self, decode: DecodeConfig) -> int:
        self.budget = self.config.max_spec_tokens or max(1, decode.cycle_length - 1)
        return self.budget

    def speculate(self, context: list[int], local: SuffixTrie | None) -> Speculation:
        c = self.config
        kw = dict(max_tokens=self.budget, min_prob=float(c.min_token_prob), tree=c.tree,
                  factor=float(c.max_spec_factor), offset=float(c.max_spec_offset))
        drafts = []
        if local is not None:  # the row's own text (its current occurrence has no continuation yet)
            drafts.append((local.speculate(context, **kw), 1))
        if self.global_trie.tokens:
            drafts.append((self.global_trie.speculate(context, **kw), 0))
        if not drafts:
            return Speculation()
        return max(drafts, key=lambda d: (d[0].score, d[0].match, d[1]))[0]

    def drafter(self) -> SuffixDrafter:
        return SuffixDrafter(self)

    def default_decoding(self) -> DecodeConfig:
        return DecodeConfig(cycle_length=(self.config.max_spec_tokens or 8) + 1)
