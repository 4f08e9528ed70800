"""SpecExec draft trees: best-first parallel search over the drafter's continuations (Svirschevski et al., 2024,
"SpecExec: Massively Parallel Speculative Decoding for Interactive LLM Inference on Consumer Devices"; economize
``decoding/specexec.py:1-230``).

``DecodeConfig(draft_policy="specexec", draft_policy_options={"depth": 8, "width": 8, "topk": 8,
"total_tokens": 60, "decay": 0.95})`` turns any drafter with tree steps into a search over a pool of candidates,
each scored by the cumulative log-probability of its path plus ``log(decay)`` per depth (deep nodes are discounted
for the chance that an ancestor is rejected):

1. the root's ``topk`` most likely tokens seed the pool;
2. each of ``depth - 1`` search steps runs the ``width`` best candidates not yet expanded, whatever their depth,
   through one batched draft step under a tree mask, and adds each one's ``topk`` children to the pool;
3. the ``total_tokens`` best candidates form the draft (a child never scores above its parent, and ties go to the
   shallower node, so the selection is closed under ancestors).

All ``depth - 1`` steps always run, so every cycle has the same shapes and runs inside one CUDA graph. The pool lives
in preallocated buffers written in place; the forwarded nodes' output states sit in one buffer indexed by their slot
(the root's state first), and their ancestor bits are built from their parents' bits as they are forwarded.
"""

from __future__ import annotations

from collections.abc import Mapping
from dataclasses import dataclass

from ..errors import ConfigError
from ..validation import is_positive_int

__all__ = ["SearchOptions"]

MAX_TREE_NODES = 64


@dataclass(frozen=True)
class SearchOptions:
    """``depth``: largest depth (``depth - 1`` search steps); ``width``: candidates expanded per step; ``topk``:
    children added per expanded candidate; ``total_tokens``: draft size; ``decay``: factor on every depth's
    probability, in ``(0, 1]``."""

    depth: int
    width: int
    topk: int
    total_tokens: int
    decay: float = 0.95

    @property
    def steps(self) -> int:
        return self.depth - 1

    @property
    def forwarded(self) -> int:
        """Nodes the search runs through the drafter besides the root."""
        return self.steps * self.width

    @property
    def candidates(self) -> int:
        """Pool size after the search."""
        return self.topk + self.steps * self.width * self.topk

    @classmethod
    def from_options(cls, options: Mapping[str, object], cycle_length: int) -> SearchOptions:
        """Parse ``draft_policy_options`` of the ``specexec`` policy (``depth`` defaults to ``cycle_length - 1``),
        refusing shapes the fixed-size search buffers cannot hold."""
        known = {"depth": max(cycle_length - 1, 1), "width": 8, "topk": 8, "total_tokens": 60, "decay": 0.95}
        stray = [name for name in options if name not in known]
        if stray:
            raise ConfigError(f"unknown specexec option(s) {sorted(stray)} (known: {', '.join(known)})")
        merged = dict(known)
        merged.update(options)
        sizes = {}
        for name in ("depth", "width", "topk", "total_tokens"):
            if not is_positive_int(merged[name]):
                raise ConfigError(f"specexec's {name} is a count and must be a positive integer, not {merged[name]!r}")
            sizes[name] = int(merged[name])
        decay = merged["decay"]
        if isinstance(decay, bool) or not isinstance(decay, (int, float)) or decay <= 0.0 or decay > 1.0:
            raise ConfigError(f"specexec's decay scales each deeper level's probability: it lies in (0, 1], "
                              f"not {decay!r}")
        search = cls(sizes["depth"], sizes["width"], sizes["topk"], sizes["total_tokens"], float(decay))
        if search.topk > 16:
            raise ConfigError(f"topk={search.topk}, but the fused top-k kernel ranks at most 16 children per node")
        if search.width > search.topk:
            raise ConfigError(f"width={search.width} exceeds topk={search.topk}: the first search step can only "
                              "expand the root's topk children")
        if search.total_tokens > search.candidates:
            raise ConfigError(f"total_tokens={search.total_tokens} exceeds the {search.candidates} candidates a "
                              f"search of depth {search.depth}, width {search.width} and topk {search.topk} "
                              "produces")
        if max(search.total_tokens + 1, search.forwarded) > MAX_TREE_NODES:
            raise ConfigError(f"the search forwards {search.forwarded} nodes and verifies {search.total_tokens} + 1; "
                              f"both must fit the {MAX_TREE_NODES}-bit ancestor words")
        return search
