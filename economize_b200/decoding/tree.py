"""Draft-tree shapes and the tensor functions of tree drafting and verification.

A verified tree has ``T = N + 1`` nodes: node 0 is the root (the last committed token), nodes ``1..N`` are drafts
in topological order with ``parents[:, i] < i``. The attention kernels read the tree as one 64-bit word per node
(bit ``j``: node ``j`` is an ancestor or the node itself), so a tree pass holds at most 64 nodes.

EAGLE-2 dynamic trees (``dynamic_tree`` policy, economize ``src/economize/decoding/dynamic_tree.py:47-231`` and
``tree_search.py:select_candidates``): candidates are grown level by level from the ``topk`` best nodes of the
previous level, and the ``total_tokens`` candidates of highest cumulative log-probability form the tree; a tie
goes to the shallower candidate so the selection stays closed under ancestors.
"""

from __future__ import annotations

from collections.abc import Mapping
from dataclasses import dataclass

import torch

from ..errors import ConfigError
from ..validation import is_positive_int

__all__ = ["DEFAULT_TOPK", "DEFAULT_TOTAL_TOKENS", "LOGP_FLOOR", "TreeOptions", "ancestor_bits", "chain_parents",
           "popcount64", "select_candidates"]

DEFAULT_TOPK = 10
DEFAULT_TOTAL_TOKENS = 60
#: Floor of a candidate's log-probability (a zero-probability token keeps a finite score).
LOGP_FLOOR = -1e4
MAX_TREE_NODES = 64


@dataclass(frozen=True)
class TreeOptions:
    """``depth`` levels below the root, ``topk`` frontier width / children per node, ``total_tokens`` verified nodes."""

    depth: int
    topk: int
    total_tokens: int

    @property
    def forwarded(self) -> int:
        """Nodes a proposal runs through the drafter besides the root."""
        return (self.depth - 1) * self.topk

    @property
    def candidates(self) -> int:
        return self.topk + (self.depth - 1) * self.topk * self.topk

    @classmethod
    def from_options(cls, options: Mapping[str, object], cycle_length: int) -> TreeOptions:
        """Parse the ``dynamic_tree`` options. ``depth`` defaults to ``cycle_length - 1`` and ``topk`` to EAGLE-2's
        10; without ``total_tokens`` the tree verifies EAGLE-2's 60 nodes, or every candidate when a shallow search
        produces fewer."""
        allowed = ("depth", "topk", "total_tokens")
        stray = [name for name in options if name not in allowed]
        if stray:
            raise ConfigError(f"unknown dynamic_tree option(s) {sorted(stray)} (known: {', '.join(allowed)})")
        depth = options.get("depth", max(cycle_length - 1, 1))
        topk = options.get("topk", DEFAULT_TOPK)
        for name, value in (("depth", depth), ("topk", topk)):
            if not is_positive_int(value):
                raise ConfigError(f"dynamic_tree's {name} must be a positive integer, not {value!r}")
        pool = int(topk) + (int(depth) - 1) * int(topk) ** 2  # candidates the search ranks
        total = options.get("total_tokens", min(DEFAULT_TOTAL_TOKENS, pool))
        if not is_positive_int(total):
            raise ConfigError(f"dynamic_tree's total_tokens must be a positive integer, not {total!r}")
        tree = cls(int(depth), int(topk), int(total))
        if tree.total_tokens > pool:
            raise ConfigError(f"only {pool} candidates exist for depth {tree.depth} and topk {tree.topk}, fewer than "
                              f"total_tokens={tree.total_tokens}")
        if tree.total_tokens >= MAX_TREE_NODES:
            raise ConfigError(f"total_tokens={tree.total_tokens}: one verified pass holds at most "
                              f"{MAX_TREE_NODES - 1} draft nodes next to the root")
        if tree.forwarded > MAX_TREE_NODES:
            raise ConfigError(f"the search runs (depth - 1) x topk = {tree.forwarded} nodes through the drafter, "
                              f"more than the {MAX_TREE_NODES} an ancestor word covers")
        return tree


def chain_parents(batch: int, length: int, device: torch.device | str) -> torch.Tensor:
    """Parents ``[B, T]`` of a chain of ``T`` nodes (``parents[:, t] = t - 1``, root's entry 0)."""
    idx = torch.arange(length, device=device).clamp_min(1) - 1
    return idx.expand(batch, length).contiguous()


def ancestor_bits(parents: torch.Tensor, max_depth: int) -> torch.Tensor:
    """``[B, T]`` int64 words: bit ``j`` of node ``i`` is set when ``j`` is ``i`` or one of its ancestors.

    Pointer doubling over ``parents`` (root's entry ignored): ``ceil(log2(max_depth + 1))`` gathers, no host sync.
    """
    batch, length = parents.shape
    device = parents.device
    idx = torch.arange(length, device=device)
    self_bit = torch.ones(batch, length, dtype=torch.int64, device=device) << idx.expand(batch, length)
    par = parents.long().clone()
    par[:, 0] = 0
    bits = self_bit | torch.where(idx[None] > 0, self_bit.gather(1, par), torch.zeros_like(self_bit))
    hop = par.gather(1, par)  # grandparent
    reach = 2
    while reach < max_depth + 1:
        bits = bits | bits.gather(1, par)
        par = hop
        hop = par.gather(1, par)
        reach *= 2
    # one more pass covers the remaining levels after doubling
    bits = bits | bits.gather(1, par)
    return bits


def popcount64(x: torch.Tensor) -> torch.Tensor:
    """Bit count of int64 words (SWAR; arithmetic shifts of negative words are masked)."""
    m1, m2, m4 = 0x5555555555555555, 0x3333333333333333, 0x0F0F0F0F0F0F0F0F
    def srl(v: torch.Tensor, n: int) -> torch.Tensor:  # logical shift right
        return (v >> n) & ((1 << (64 - n)) - 1)
    x = x - (srl(x, 1) & m1)
    x = (x & m2) + (srl(x, 2) & m2)
    x = (x + srl(x, 4)) & m4
    return srl(x * 0x0101010101010101, 56) & 0xFF


def select_candidates(tokens: torch.Tensor, scores: torch.Tensor, parents: torch.Tensor, depth: torch.Tensor,
                      total: int) -> tuple[torch.Tensor, torch.Tensor]:
    """The ``total`` best candidates as a tree in topological order: tokens ``[B, total]`` and the parent of every
    node among them ``[B, total]`` (``-1`` for the root's children). Candidates are numbered parents first."""
    batch, device = tokens.shape[0], tokens.device
    key = scores.double() - depth.double() * 1e-9
    chosen = key.topk(total, -1).indices.sort(-1).values
    place = torch.full_like(tokens, -1).scatter(1, chosen, torch.arange(total, device=device).expand(batch, total))
    parent = parents.gather(1, chosen)
    tree_parents = torch.where(parent >= 0, place.gather(1, parent.clamp_min(0)), -1)
    return tokens.gather(1, chosen), tree_parents
