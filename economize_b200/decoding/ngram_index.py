"""Host-side token indexes for retrieval drafters (suffix decoding, REST, lookahead pools).

:class:`NGramIndex` maps every context of 1..``max_context`` tokens seen in the indexed sequences to the counts
of the tokens that followed it. :meth:`NGramIndex.draft_tree` grows a draft tree from the longest context that
matches the end of a row's history: a node's children are the most frequent continuations of the longest
indexed context ending at that node (suffix-tree style matching as in SuffixDecoding, Oliaro et al. 2024), nodes
being taken best-first by the product of the continuation frequencies until ``budget`` nodes.
"""

from __future__ import annotations

import heapq
from collections import Counter, defaultdict
from collections.abc import Iterable, Sequence

import torch

__all__ = ["NGramIndex", "trees_to_tensors"]


class NGramIndex:
    def __init__(self, max_context: int = 8) -> None:
        self.max_context = max_context
        self.table: dict[tuple[int, ...], Counter] = defaultdict(Counter)
        self.size = 0

    def add(self, tokens: Sequence[int], start: int = 0) -> None:
        """Index the continuations of ``tokens`` at positions ``>= start`` (so a growing sequence is indexed
        incrementally)."""
        toks = list(tokens)
        for i in range(max(start, 1), len(toks)):
            nxt = toks[i]
            for d in range(1, min(self.max_context, i) + 1):
                self.table[tuple(toks[i - d:i])][nxt] += 1
        self.size += max(0, len(toks) - max(start, 1))

    def extend(self, sequences: Iterable[Sequence[int]]) -> None:
        for seq in sequences:
            self.add(seq)

    def continuations(self, context: Sequence[int], min_match: int = 1) -> tuple[int, Counter | None]:
        """(match length, counts of next tokens) for the longest indexed suffix of ``context``."""
        ctx = list(context)
        for d in range(min(self.max_context, len(ctx)), min_match - 1, -1):
            c = self.table.get(tuple(ctx[len(ctx) - d:]))
            if c:
                return d, c
        return 0, None

    def draft_tree(self, context: Sequence[int], budget: int, depth: int, branch: int = 4,
                   min_match: int = 1, others: Sequence[NGramIndex] = ()) -> tuple[list[int], list[int]]:
        """Tokens and parent indices (``-1``: child of the root) of a best-first draft tree of up to ``budget``
        nodes and ``depth`` levels, from this index and ``others`` (counts added)."""
        ctx = list(context)
        tokens: list[int] = []
        parents: list[int] = []
        heap: list[tuple[float, int, int, list[int], int]] = []  # (-score, order, parent, path, level)
        order = 0

        def expand(path: list[int], parent: int, score: float, level: int) -> None:
            nonlocal order
            if level >= depth:
                return
            counts: Counter = Counter()
            best = 0
            for idx in (self, *others):
                m, c = idx.continuations(ctx + path, min_match)
                if c is not None and m >= best:
                    if m > best:
                        counts, best = Counter(), m
                    counts.update(c)
            total = sum(counts.values())
            for tok, n in counts.most_common(branch):
                heapq.heappush(heap, (-(score * n / total), order, parent, path + [tok], level + 1))
                order += 1

        expand([], -1, 1.0, 0)
        while heap and len(tokens) < budget:
            neg, _, parent, path, level = heapq.heappop(heap)
            tokens.append(path[-1])
            parents.append(parent)
            expand(path, len(tokens) - 1, -neg, level)
        return tokens, parents


def trees_to_tensors(trees: list[tuple[list[int], list[int]]], width: int,
                     device: torch.device) -> tuple[torch.Tensor, torch.Tensor]:
    """Pad per-row trees to ``[B, width]`` drafts (``-1`` where a row has fewer nodes) and parents (padding nodes
    hang off the root, so they are verified and rejected)."""
    batch = len(trees)
    tok = torch.full((batch, width), -1, dtype=torch.int64)
    par = torch.full((batch, width), -1, dtype=torch.int64)
    for b, (t, p) in enumerate(trees):
        n = min(len(t), width)
        if n:
            tok[b, :n] = torch.tensor(t[:n])
            par[b, :n] = torch.tensor(p[:n])
    return tok.to(device), par.to(device)
