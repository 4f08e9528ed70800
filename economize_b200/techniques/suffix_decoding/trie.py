"""A bounded-depth suffix trie with occurrence counts: the data structure of SuffixDecoding (Oliaro et al., 2025).

Every substring of the indexed text of length at most ``depth`` is a path from the root; a node's count is the
number of its occurrences. Text is appended incrementally: the trie keeps the nodes of the (at most ``depth``)
suffixes that are still open, and a new token extends each of them by one child, so indexing costs ``O(depth)``
per token. Substrings are closed under taking suffixes, so whether the context's last ``m`` tokens occur is
monotone in ``m`` and the longest match is found by growing ``m`` until a path breaks.

Speculation below a matched node uses the empirical continuation probability ``count(child) / count(node)``,
multiplied along the path (a node's occurrences that end the text have no child, so probabilities of siblings sum
to at most one). Path mode follows the most frequent child; tree mode grows best-first from a heap, the most
probable frontier node first. Nodes are kept in flat Python lists (children as one dict per node).
"""

from __future__ import annotations

import heapq
from collections.abc import Iterable, Sequence
from dataclasses import dataclass

__all__ = ["Speculation", "SuffixTrie"]


@dataclass(frozen=True)
class Speculation:
    """A draft from a trie: ``tokens`` with ``parents`` (``-1``: a child of the root), the summed probability of
    its nodes (``score``) and the length of the matched context suffix (``match``)."""

    tokens: tuple[int, ...] = ()
    parents: tuple[int, ...] = ()
    score: float = 0.0
    match: int = 0


class SuffixTrie:
    """Counts of every substring of at most ``depth`` tokens of the appended text."""

    def __init__(self, depth: int) -> None:
        if depth < 2:
            raise ValueError(f"a suffix trie needs depth >= 2, got {depth}")
        self.depth = depth
        self.children: list[dict[int, int]] = [{}]
        self.count: list[int] = [0]
        self._open: list[int] = []  # nodes of the suffixes of the current sequence shorter than depth
        self.tokens = 0

    def __len__(self) -> int:
        return len(self.count)

    def _child(self, node: int, token: int) -> int:
        nxt = self.children[node].get(token)
        if nxt is None:
            nxt = len(self.count)
            self.children[node][token] = nxt
            self.children.append({})
            self.count.append(0)
        self.count[nxt] += 1
        return nxt

    def append(self, tokens: Iterable[int]) -> None:
        """Extend the current sequence by ``tokens``."""
        for token in tokens:
            token = int(token)
            grown = [self._child(node, token) for node in self._open]
            grown.append(self._child(0, token))  # the suffix that starts at this token
            self.count[0] += 1
            # a suffix that reached depth tokens cannot grow any further
            self._open = [n for n, length in zip(grown, range(len(grown), 0, -1)) if length < self.depth]
            self.tokens += 1

    def end_sequence(self) -> None:
        """Close the current sequence: the next appended token starts an unrelated one."""
        self._open = []

    def add_sequence(self, tokens: Sequence[int]) -> None:
        """Index ``tokens`` as a sequence of its own."""
        self.end_sequence()
        self.append(tokens)
        self.end_sequence()

    def match(self, context: Sequence[int]) -> tuple[int, int]:
        """``(node, m)``: the node of the longest suffix of ``context`` (at most ``depth - 1`` tokens) that occurs,
        and its length (``(0, 0)`` when not even the last token occurs)."""
        best = (0, 0)
        limit = min(len(context), self.depth - 1)
        for m in range(1, limit + 1):
            node = 0
            for token in context[len(context) - m:]:
                node = self.children[node].get(int(token), -1)
                if node < 0:
                    return best
            best = (node, m)
        return best

    def speculate(self, context: Sequence[int], *, max_tokens: int, min_prob: float, tree: bool,
                  factor: float = 1.0, offset: float = 0.0) -> Speculation:
        """The best draft over every match length: for each ``m = 1, 2, ...`` whose context suffix occurs (up to
        ``depth - 1``, stopping at the first that does not), a draft of at most ``min(max_tokens, floor(factor * m
        + offset))`` tokens of probability at least ``min_prob`` below the match, no path longer than ``depth - m``.
        The draft with the largest summed probability wins (the longer match on ties). Trying every length matters
        when the trie also holds the context itself: its longest matches are the context's own, unfinished
        occurrence, which has no continuation yet."""
        best = Speculation()
        limit = min(len(context), self.depth - 1)
        for m in range(1, limit + 1):
            node = 0
            for token in context[len(context) - m:]:
                node = self.children[node].get(int(token), -1)
                if node < 0:
                    return best
            if not self.children[node]:
                continue
            draft = self._grow(node, m, min(max_tokens, int(factor * m + offset)), min_prob, tree)
            if draft.tokens and (draft.score, draft.match) >= (best.score, best.match):
                best = draft
        return best

    def _grow(self, node: int, m: int, budget: int, min_prob: float, tree: bool) -> Speculation:
        room = self.depth - m
        tokens: list[int] = []
        parents: list[int] = []
        score = 0.0
        if not tree:
            prob, parent, level = 1.0, -1, 0
            while len(tokens) < budget and level < room and self.children[node]:
                token, child = max(self.children[node].items(), key=lambda kv: (self.count[kv[1]], -kv[0]))
                prob *= self.count[child] / self.count[node]
                if prob < min_prob:
                    break
                tokens.append(token)
                parents.append(parent)
                score += prob
                parent, node, level = len(tokens) - 1, child, level + 1
            return Speculation(tuple(tokens), tuple(parents), score, m)
        heap: list[tuple[float, int, int, int, int, int]] = []  # (-prob, order, node, parent slot, token, level)
        order = 0

        def offer(at: int, prob: float, slot: int, level: int) -> None:
            nonlocal order
            if level >= room:
                return
            total = self.count[at]
            for token, child in self.children[at].items():
                p = prob * self.count[child] / total
                if p >= min_prob:
                    heapq.heappush(heap, (-p, order, child, slot, token, level + 1))
                    order += 1

        offer(node, 1.0, -1, 0)
        while heap and len(tokens) < budget:
            neg, _, child, slot, token, level = heapq.heappop(heap)
            tokens.append(token)
            parents.append(slot)
            score -= neg
            offer(child, -neg, len(tokens) - 1, level)
        return Speculation(tuple(tokens), tuple(parents), score, m)
