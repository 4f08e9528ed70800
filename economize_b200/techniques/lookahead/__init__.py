"""Lookahead decoding (``lookahead``; Fu et al., 2024; economize ``techniques/lookahead``).

Every cycle is one exact pass over a single tree hanging below the root (the last committed token) with two
branches:

* the **verification branch**: the n-grams of the pool whose first token is the root, merged into a trie (at most
  ``guesses`` of them, the most recently made ones);
* the **lookahead branch**: the 2D Jacobi window. Level 0 is a chain continuing the root; column ``j`` of level
  ``l >= 1`` hangs below column ``j`` of level ``l - 1`` (below the root or level 0's column ``j - 1`` for
  ``l = 1``), so it sees the first block up to column ``j`` and its column's earlier levels, the attention pattern of
  the official lookahead branch written as a tree.

The engine verifies the whole tree greedily (a window path the target agrees with is accepted too: it is a valid
draft); afterwards :meth:`LookaheadDrafter.after_verify` reads the target's greedy predictions at the window's last
level, makes that the window's newest level (one Jacobi step) and, once the window holds ``ngram - 1`` levels, adds
one ``ngram``-gram per column to the pool. The window starts as ``window + ngram - 3`` tokens drawn from the prompt
and gains a level per pass.

The engine's tree passes carry at most 64 new tokens (one int64 of ancestor bits per node), so the window and the
guesses must fit 63 nodes together (the paper's 7B setting W = 15, N = 5, G = 15 does not; W = 7, N = 5, G = 7 does).
"""

from __future__ import annotations

import random
from collections import OrderedDict
from dataclasses import dataclass
from typing import ClassVar

import torch

from ...core.technique import Capability, Family, Technique, TechniqueConfig, register_technique
from ...decoding.config import DecodeConfig
from ...decoding.ngram_index import trees_to_tensors
from ...errors import ConfigError
from ...validation import check_positive

__all__ = ["JacobiWindow", "LookaheadConfig", "LookaheadDrafter", "LookaheadTechnique", "NGramPool"]

MAX_NODES = 63  # new tokens of a tree pass besides the root


@dataclass(frozen=True)
class LookaheadConfig(TechniqueConfig):
    """``window`` columns W of the Jacobi window, ``ngram`` length N of the n-grams (the window has N - 1 levels),
    ``guesses`` n-grams kept per first token (default W), ``pool_from_prompt``: also pool every n-gram of the
    committed tokens, ``seed`` of the window's initial tokens."""

    technique: ClassVar[str] = "lookahead"
    window: int = 7
    ngram: int = 5
    guesses: int | None = None
    pool_from_prompt: bool = False
    seed: int = 0

    def __post_init__(self) -> None:
        check_positive("window", self.window)
        if self.ngram < 3:
            raise ConfigError(f"ngram must be at least 3 (a window of two levels), got {self.ngram}")
        if self.guesses is not None and self.guesses < 0:
            raise ConfigError(f"guesses must be >= 0, got {self.guesses}")
        if self.seed < 0:
            raise ConfigError(f"seed must be >= 0, got {self.seed}")
        if self.budget > MAX_NODES:
            raise ConfigError(f"a lookahead tree of window {self.window}, ngram {self.ngram} and "
                              f"{self.pool_size} guesses has {self.budget} nodes; a tree pass verifies at most "
                              f"{MAX_NODES}")

    @property
    def pool_size(self) -> int:
        return self.window if self.guesses is None else self.guesses

    @property
    def window_nodes(self) -> int:
        """Nodes of a full window: W - 1 in level 0, W in each of the other N - 2 levels."""
        return self.window - 1 + (self.ngram - 2) * self.window

    @property
    def budget(self) -> int:
        # the filling window has more level-0 tokens (W + N - 3) and fewer levels; this bounds every pass
        return self.pool_size * (self.ngram - 1) + max(self.window_nodes, self.window + self.ngram - 3)

    @property
    def max_depth(self) -> int:
        return max(self.ngram - 1, self.window + self.ngram - 3)


class NGramPool:
    """Continuations of ``n``-grams keyed by their first token; the most recently made ``capacity`` per key."""

    def __init__(self, capacity: int) -> None:
        self.capacity = capacity
        self.grams: dict[int, OrderedDict[tuple[int, ...], None]] = {}

    def add(self, first: int, continuation: tuple[int, ...]) -> None:
        if self.capacity <= 0:
            return
        slot = self.grams.setdefault(first, OrderedDict())
        slot.pop(continuation, None)
        slot[continuation] = None  # most recent last
        while len(slot) > self.capacity:
            slot.popitem(last=False)

    def lookup(self, first: int) -> list[tuple[int, ...]]:
        """The continuations of ``first``, most recent first."""
        return list(reversed(self.grams.get(first, {})))


class JacobiWindow:
    """The lookahead branch of one row: ``levels`` lists of guessed tokens (level 0 continues the root)."""

    def __init__(self, initial: list[int], depth: int) -> None:
        self.levels: list[list[int]] = [list(initial)]
        self.depth = depth  # N - 1 levels when full

    @property
    def full(self) -> bool:
        return len(self.levels) == self.depth

    def nodes(self, offset: int) -> tuple[list[int], list[int], list[int]]:
        """Tokens and parents (draft indices, -1 = root) of the window's nodes numbered from ``offset``, and the node
        indices of its last level."""
        tokens: list[int] = []
        parents: list[int] = []
        last: list[int] = []
        for l, level in enumerate(self.levels):
            start = offset + len(tokens)
            ids = list(range(start, start + len(level)))
            if l == 0:  # a chain below the root
                parents += [-1] + ids[:-1]
                above = [-1] + ids  # column j of the first block: the root, then level 0's tokens
            else:  # column j below column j of the level above
                parents += above[:len(level)]
                above = ids
            tokens += level
            last = ids
        return tokens, parents, last

    def step(self, predictions: list[int], root: int) -> list[tuple[int, tuple[int, ...]]]:
        """One Jacobi step with the target's predictions at the last level after a pass whose root was ``root``;
        returns the completed n-grams (one per column) once the window is full."""
        if not self.full:
            if len(self.levels) == 1:
                self.levels = [self.levels[0][1:], list(predictions)]
            else:
                self.levels = [lv[1:] for lv in self.levels] + [list(predictions[1:])]
            return []
        block = [root] + self.levels[0]
        grams = []
        for j, p in enumerate(predictions):
            grams.append((block[j], tuple(lv[j] for lv in self.levels[1:]) + (p,)))
        self.levels = [self.levels[1][1:]] + self.levels[2:] + [list(predictions)]
        return grams


def _trie(root: int, grams: list[tuple[int, ...]]) -> tuple[list[int], list[int]]:
    """Merge continuations of ``root`` into one trie of draft nodes (parents as draft indices, -1 = the root)."""
    tokens: list[int] = []
    parents: list[int] = []
    children: dict[tuple[int, int], int] = {}
    for gram in grams:
        at = -1
        for tok in gram:
            key = (at, tok)
            if key not in children:
                children[key] = len(tokens)
                tokens.append(tok)
                parents.append(at)
            at = children[key]
    return tokens, parents


class LookaheadDrafter:
    """Engine-side proposer: builds each row's tree on the host and reads the window's predictions back."""

    observes = False
    graph_safe = False
    capture_layers: tuple[int, ...] = ()
    carry_size = 0

    def __init__(self, config: LookaheadConfig) -> None:
        self.config = config
        self.windows: list[JacobiWindow | None] = []
        self.pools: list[NGramPool] = []
        self.pooled: list[int] = []
        self.layout: list[tuple[int, list[int]]] = []  # per row: (root token, last-level draft indices)

    def begin(self, batch: int, capacity: int) -> None:
        self.windows = [None] * batch
        self.pools = [NGramPool(self.config.pool_size) for _ in range(batch)]
        self.pooled = [0] * batch
        self.layout = []

    def draft_depth(self, decode: DecodeConfig) -> int:
        return self.config.max_depth

    def draft_nodes(self, decode: DecodeConfig) -> int:
        return self.config.budget

    def _init_window(self, b: int, row: list[int]) -> JacobiWindow:
        c = self.config
        rng = random.Random(c.seed * 1000003 + b)
        initial = [row[rng.randrange(len(row))] for _ in range(c.window + c.ngram - 3)]
        return JacobiWindow(initial, c.ngram - 1)

    def propose(self, history: torch.Tensor, length: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        c = self.config
        hist = history.cpu()
        trees = []
        self.layout = []
        for b, n in enumerate(length.cpu().tolist()):
            row = hist[b, :n].tolist()
            if self.windows[b] is None:
                self.windows[b] = self._init_window(b, row)
            if c.pool_from_prompt:  # every n-gram of the committed tokens not pooled yet
                for s in range(max(0, self.pooled[b] - c.ngram + 1), n - c.ngram + 1):
                    self.pools[b].add(row[s], tuple(row[s + 1:s + c.ngram]))
                self.pooled[b] = n
            root = row[-1]
            tokens, parents = _trie(root, self.pools[b].lookup(root)[:c.pool_size])
            w_tokens, w_parents, last = self.windows[b].nodes(len(tokens))
            trees.append((tokens + w_tokens, parents + w_parents))
            self.layout.append((root, last))
        return trees_to_tensors(trees, c.budget, history.device)

    def after_verify(self, tokens: torch.Tensor, pred: torch.Tensor) -> None:
        """The target's greedy predictions ``pred [B, T]`` of the verified pass (node ``i + 1`` = draft ``i``)."""
        pred = pred.cpu()
        for b, (root, last) in enumerate(self.layout):
            predictions = [int(pred[b, i + 1]) for i in last]
            for first, cont in self.windows[b].step(predictions, root):
                self.pools[b].add(first, cont)

    def to_target(self, ids: torch.Tensor) -> torch.Tensor:
        return ids


@register_technique
class LookaheadTechnique(Technique):
    config_class = LookaheadConfig
    capabilities = Capability.DRAFTER
    family = Family.DRAFTER
    lossless = True
    graph_safe = False

    def drafter(self) -> LookaheadDrafter:
        return LookaheadDrafter(self.config)

    def default_decoding(self) -> DecodeConfig:
        return DecodeConfig(cycle_length=self.config.max_depth + 1)
