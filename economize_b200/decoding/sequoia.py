"""Sequoia draft trees: one static tree of the best shape for measured acceptance rates and latencies (Chen et al.,
2024, "Sequoia: Scalable, Robust, and Hardware-aware Speculative Decoding"; economize ``decoding/sequoia.py:1-572``).

``DecodeConfig(draft_policy="sequoia", draft_policy_options={"acceptance": (0.6, 0.15, 0.06, 0.03),
"total_tokens": 32, "depth": 8})`` turns a chain drafter (any drafter with tree steps) into a drafter of one fixed
tree per cycle. Every node names its rank among its siblings; a proposal fills the tree with the drafter's
``rank``-th most likely token after every parent, one batched draft step per depth over the nodes of that depth that
have children. The exact pass verifies it as any draft tree, so decoding stays lossless.

``acceptance[r]`` is the probability that the exact model's token after an accepted node is the drafter's ``r``-th
most likely token (or one such vector per depth of the parent node, the root's first and the last reused below).
Siblings are disjoint events, so a node contributes its *reach* (the product of the rates along its rank path) to
the expected tokens per cycle, and a tree's value is one (the root) plus the reaches of its nodes.

Shape search. A node's reach never exceeds its parent's (every factor is at most one), so among all sets of ``n``
rank paths of depth at most ``D`` that are closed under taking parents, the ``n`` paths of largest reach are one
(ties go to the shallower path, which keeps every parent ahead of its children) and no other set has a larger sum.
:func:`sequoia_tree` therefore grows the tree best-first from a heap of candidate children: it takes the candidate of
largest reach and offers that node's children, until ``total_tokens`` nodes are placed or no candidate reaches
anything. Ranks that a measured profile makes worth less than a higher rank are simply placed later (siblings need
not be consecutive ranks). With measured latencies (``verify_latency[i]``: one exact pass over ``i + 1`` tokens;
``draft_latency``: one draft step) every prefix of the best-first order, for every depth limit, is a candidate, and
the one of most tokens per second wins (Sequoia's hardware-aware choice).

:func:`measure_acceptance` estimates the rates by decoding prompts with a probe tree and counting which rank the
exact token had at every accepted node; an explicit tree can be given as rank ``paths`` instead (the format of
Medusa's tree choices).
"""

from __future__ import annotations

import heapq
from collections.abc import Mapping, Sequence
from dataclasses import dataclass, field

import numpy as np
import torch

from ..errors import ConfigError
from ..validation import is_positive_int

__all__ = ["AcceptanceProfile", "StaticPlan", "StaticTree", "expected_tokens", "measure_acceptance", "probe_paths",
           "record_cycle", "sequoia_tree", "tree_from_options"]

Path = tuple[int, ...]
MAX_FORWARDED = 64  # ancestor bits of the drafter's tree steps are one 64-bit word per node


@dataclass(frozen=True)
class StaticTree:
    """A draft tree as rank paths in breadth-first order (by depth, then lexicographically), so that every node
    comes after its parent.

    Attributes:
        paths: ``paths[i]`` is the rank path of node ``i`` (``(0, 2)``: the 3rd best token after the best first
            token).
        expected: Expected tokens per cycle under the rates it was built for (``None`` for an explicit tree).
    """

    paths: tuple[Path, ...]
    expected: float | None = None

    @classmethod
    def from_paths(cls, paths: Sequence[Sequence[int]], expected: float | None = None) -> StaticTree:
        unique: set[Path] = set()
        for raw in paths:
            path = tuple(int(r) for r in raw)
            if len(path) == 0:
                raise ConfigError("an empty rank path names the root, which every tree has implicitly; list only "
                                  "draft nodes")
            bad = [r for r in path if r < 0]
            if bad:
                raise ConfigError(f"ranks are 0-based positions in the drafter's ranking; {path} holds {bad[0]}")
            unique.add(path)
        if not unique:
            raise ConfigError("the draft tree has no nodes")
        orphans = [p for p in unique if len(p) > 1 and p[:-1] not in unique]
        if orphans:
            p = min(orphans, key=lambda q: (len(q), q))
            raise ConfigError(f"node {p} hangs below {p[:-1]}, which is not in the tree")
        ordered = sorted(unique, key=lambda q: (len(q), q))
        return cls(tuple(ordered), expected)

    @property
    def size(self) -> int:
        return len(self.paths)

    @property
    def depth(self) -> int:
        return max(map(len, self.paths))

    @property
    def parents(self) -> tuple[int, ...]:
        """Parent node of every node (``-1``: a child of the root)."""
        where = {path: i for i, path in enumerate(self.paths)}
        return tuple(-1 if len(path) == 1 else where[path[:-1]] for path in self.paths)

    @property
    def ranks(self) -> tuple[int, ...]:
        return tuple(path[-1] for path in self.paths)

    @property
    def forwarded(self) -> int:
        """Nodes that run through the drafter (those with children)."""
        return len({path[:-1] for path in self.paths} - {()})


def rate_table(acceptance: Sequence[float] | Sequence[Sequence[float]], depth: int) -> np.ndarray:
    """``acceptance`` as a ``[depth, width]`` table: row ``l`` holds the rates after a node of depth ``l`` (the root
    is depth 0); a single vector serves every depth, and per-depth vectors repeat their last one downwards."""
    nested = len(acceptance) > 0 and isinstance(acceptance[0], (Sequence, np.ndarray))
    vectors = [list(map(float, v)) for v in (acceptance if nested else [acceptance])]
    width = max(map(len, vectors), default=0)
    if width == 0:
        raise ConfigError("sequoia needs at least one acceptance rate")
    for v in vectors:
        low, total = min(v, default=0.0), sum(v)
        if low < 0.0 or max(v, default=0.0) > 1.0:
            raise ConfigError(f"acceptance rates are probabilities; {v} has an entry outside [0, 1]")
        if total > 1.0 + 1e-6:
            raise ConfigError(f"the exact token can match at most one rank, so the rates of one depth sum to at "
                              f"most 1; {v} sums to {total:.4f}")
    table = np.zeros((depth, width))
    for level in range(depth):
        v = vectors[level] if level < len(vectors) else vectors[-1]
        table[level, :len(v)] = v
    return table


def _reach_of(path: Path, table: np.ndarray) -> float:
    reach = 1.0
    for level, rank in enumerate(path):
        reach *= table[level, rank] if rank < table.shape[1] else 0.0
    return reach


def expected_tokens(tree: StaticTree | Sequence[Sequence[int]],
                    acceptance: Sequence[float] | Sequence[Sequence[float]]) -> float:
    """Expected tokens per cycle of ``tree`` (the root's token included) under the rates ``acceptance``."""
    tree = tree if isinstance(tree, StaticTree) else StaticTree.from_paths(tree)
    table = rate_table(acceptance, tree.depth)
    return 1.0 + float(sum(_reach_of(path, table) for path in tree.paths))


def best_first(table: np.ndarray, limit: int, depth: int) -> list[tuple[Path, float]]:
    """Up to ``limit`` rank paths of depth at most ``depth`` in decreasing reach (ties: shallower, then smaller
    ranks first), each with its reach; paths of zero reach are never taken. Every prefix of the result is a tree."""
    width = table.shape[1]
    heap: list[tuple[float, int, Path]] = []

    def offer(parent: Path, reach: float) -> None:
        level = len(parent)
        if level >= depth:
            return
        for rank in range(width):
            r = reach * table[level, rank]
            if r > 0.0:
                heapq.heappush(heap, (-r, level + 1, parent + (rank,)))

    offer((), 1.0)
    order: list[tuple[Path, float]] = []
    while heap and len(order) < limit:
        neg, _, path = heapq.heappop(heap)
        order.append((path, -neg))
        offer(path, -neg)
    return order


def sequoia_tree(acceptance: Sequence[float] | Sequence[Sequence[float]], total_tokens: int, depth: int, *,
                 verify_latency: Sequence[float] | None = None, draft_latency: float = 0.0) -> StaticTree:
    """The Sequoia tree for ``acceptance`` with at most ``total_tokens`` nodes and depth at most ``depth``.

    Without ``verify_latency`` the tree maximizes expected tokens per cycle; with it (one entry per exact pass of
    ``1 .. total_tokens + 1`` tokens) it maximizes expected tokens per second over every size and depth limit, a
    cycle whose tree is ``d`` deep costing ``verify_latency[n] + d * draft_latency``.
    """
    if not is_positive_int(total_tokens):
        raise ConfigError(f"total_tokens counts draft nodes and must be a positive integer, got {total_tokens!r}")
    if not is_positive_int(depth):
        raise ConfigError(f"depth must be a positive integer, got {depth!r}")
    if draft_latency < 0:
        raise ConfigError(f"draft_latency is a time and cannot be negative, got {draft_latency}")
    table = rate_table(acceptance, depth)
    if verify_latency is None:
        order = best_first(table, total_tokens, depth)
        if not order:
            raise ConfigError("no draft node can be accepted under these rates (all of them are 0)")
        return StaticTree.from_paths([p for p, _ in order], 1.0 + sum(r for _, r in order))
    times = [float(v) for v in verify_latency]
    if len(times) <= total_tokens or min(times[:total_tokens + 1]) <= 0:
        raise ConfigError(f"verify_latency must give a positive time for every exact pass of 1 to "
                          f"{total_tokens + 1} tokens ({total_tokens + 1} entries)")
    choice: tuple[float, list[Path], float] | None = None
    for limit in range(1, depth + 1):
        order = best_first(table[:limit], total_tokens, limit)
        value, deepest = 1.0, 0
        for n, (path, reach) in enumerate(order, start=1):
            value += reach
            deepest = max(deepest, len(path))
            speed = value / (times[n] + deepest * draft_latency)
            if choice is None or speed > choice[0] * (1.0 + 1e-12):
                choice = (speed, [p for p, _ in order[:n]], value)
    if choice is None:
        raise ConfigError("no draft node can be accepted under these rates (all of them are 0)")
    return StaticTree.from_paths(choice[1], choice[2])


def probe_paths(depth: int, width: int) -> tuple[Path, ...]:
    """The probe tree of :func:`measure_acceptance`: below the root and below each of the first ``depth - 1`` nodes
    of the all-best spine ``(0,), (0, 0), ...``, the children of ranks ``0 .. width - 1``."""
    spine: Path = ()
    out: list[Path] = []
    for _ in range(depth):
        out.extend(spine + (rank,) for rank in range(width))
        spine = spine + (0,)
    return tuple(out)


@dataclass
class AcceptanceProfile:
    """Counts of the exact token's rank among the drafter's candidates at accepted tree nodes.

    ``hits[l, r]``: accepted nodes of depth ``l`` whose exact next token was their rank-``r`` child; ``trials[l, r]``:
    accepted nodes of depth ``l`` that had a child of rank ``r``.
    """

    hits: np.ndarray = field(default_factory=lambda: np.zeros((0, 0)))
    trials: np.ndarray = field(default_factory=lambda: np.zeros((0, 0)))

    def _grow(self, rows: int, cols: int) -> None:
        if rows <= self.hits.shape[0] and cols <= self.hits.shape[1]:
            return
        shape = (max(rows, self.hits.shape[0]), max(cols, self.hits.shape[1]))
        for name in ("hits", "trials"):
            old = getattr(self, name)
            new = np.zeros(shape)
            new[:old.shape[0], :old.shape[1]] = old
            setattr(self, name, new)

    def add(self, level: int, child_ranks: Sequence[int], outcome: int | None) -> None:
        """One accepted node of depth ``level`` whose children have the ranks ``child_ranks``; ``outcome`` is the rank
        of the child that matched the exact token (``None``: none did)."""
        if not child_ranks:
            return
        self._grow(level + 1, max(child_ranks) + 1)
        self.trials[level, list(child_ranks)] += 1
        if outcome is not None:
            self.hits[level, outcome] += 1

    def rates(self, per_depth: bool = False) -> tuple[float, ...] | tuple[tuple[float, ...], ...]:
        """``hits / trials`` pooled over depths (or one vector per depth); 0 where nothing was tried. The result is
        a valid ``acceptance`` option of the ``sequoia`` policy."""
        def ratio(h: np.ndarray, t: np.ndarray) -> np.ndarray:
            return np.divide(h, t, out=np.zeros_like(h), where=t > 0)
        if per_depth:
            return tuple(tuple(float(v) for v in row) for row in ratio(self.hits, self.trials))
        return tuple(float(v) for v in ratio(self.hits.sum(0), self.trials.sum(0)))


_OPTIONS = ("acceptance", "paths", "total_tokens", "depth", "verify_latency", "draft_latency", "record_acceptance")


def tree_from_options(options: Mapping[str, object], cycle_length: int) -> tuple[StaticTree, bool]:
    """The tree of the ``sequoia`` policy's options and whether acceptance is recorded."""
    stray = [name for name in options if name not in _OPTIONS]
    if stray:
        raise ConfigError(f"unknown sequoia option(s) {sorted(stray)} (known: {', '.join(_OPTIONS)})")
    record = options.get("record_acceptance", False)
    if record not in (True, False) or not isinstance(record, bool):
        raise ConfigError(f"record_acceptance is a flag (True or False), not {record!r}")
    explicit, rated = "paths" in options, "acceptance" in options
    if explicit and rated:
        raise ConfigError("give sequoia either an explicit tree ('paths') or the rates to shape one ('acceptance'), "
                          "not both")
    if not (explicit or rated):
        raise ConfigError("sequoia needs a tree: pass 'paths' (rank paths) or 'acceptance' (rates to shape one)")
    if explicit:
        shaping = [name for name in ("total_tokens", "depth", "verify_latency", "draft_latency") if name in options]
        if shaping:
            raise ConfigError(f"{shaping} only shape a tree from 'acceptance'; with explicit 'paths' drop them")
        tree = StaticTree.from_paths(options["paths"])
    else:
        depth = options.get("depth", max(cycle_length - 1, 1))
        total = options.get("total_tokens", 32)
        draft = options.get("draft_latency", 0.0)
        if isinstance(draft, bool) or not isinstance(draft, (int, float)) or draft < 0:
            raise ConfigError(f"draft_latency is a non-negative time, got {draft!r}")
        latency = options.get("verify_latency")
        if latency is None and "draft_latency" in options:
            raise ConfigError("draft_latency only matters next to verify_latency; give both or neither")
        tree = sequoia_tree(options["acceptance"], total, depth, verify_latency=latency, draft_latency=float(draft))
    if tree.size >= MAX_FORWARDED or tree.forwarded > MAX_FORWARDED:
        raise ConfigError(f"the tree has {tree.size} draft nodes; one verified pass holds at most "
                          f"{MAX_FORWARDED - 1}")
    return tree, record


class StaticPlan:
    """Index tensors that fill a :class:`StaticTree` level by level on one device.

    For level ``L`` (depth ``L`` nodes, contiguous in the node order): ``k[L-1]`` candidates are ranked after each
    parent and ``pick[L-1]`` selects every node's token from the flattened ``[parents, k]`` ranking. ``fwd[L-1]``
    lists the level's nodes that run through the drafter (local indices), ``fwd_parent[L-1]`` their parents'
    positions in the previous level's forwarded list, ``offset[L-1]`` their first slot and ``bits[L-1]`` their
    ancestor bits over the forwarded slots.
    """

    def __init__(self, tree: StaticTree, device: torch.device) -> None:
        paths, parents = tree.paths, tree.parents
        self.depth = tree.depth
        self.size = tree.size
        self.parents = torch.tensor(parents, dtype=torch.int64, device=device)
        has_children = {p[:-1] for p in paths if len(p) > 1}
        by_level = [[i for i, p in enumerate(paths) if len(p) == L] for L in range(1, self.depth + 1)]
        self.k, self.pick, self.fwd, self.fwd_parent, self.offset, self.bits = [], [], [], [], [], []
        fwd_pos: dict[int, int] = {}  # node -> position in its level's forwarded list
        slot: dict[int, int] = {}
        bits: dict[int, int] = {}
        for L, nodes in enumerate(by_level, start=1):
            k = max(paths[i][-1] for i in nodes) + 1
            src = [paths[i][-1] if L == 1 else fwd_pos[parents[i]] * k + paths[i][-1] for i in nodes]
            self.k.append(k)
            self.pick.append(torch.tensor(src, dtype=torch.int64, device=device))
            fw = [i for i in nodes if paths[i] in has_children]
            self.offset.append(len(slot))
            for j, i in enumerate(fw):
                fwd_pos[i] = j
                slot[i] = len(slot)
                bits[i] = (1 << slot[i]) | (bits[parents[i]] if parents[i] >= 0 else 0)
            first = nodes[0]
            self.fwd.append(torch.tensor([i - first for i in fw], dtype=torch.int64, device=device))
            self.fwd_parent.append(torch.tensor([fwd_pos[parents[i]] if L > 1 else 0 for i in fw],
                                                dtype=torch.int64, device=device))
            self.bits.append(torch.tensor([bits[i] - (1 << 64) if bits[i] >= 1 << 63 else bits[i] for i in fw],
                                          dtype=torch.int64, device=device))
        self.widths = [len(f) for f in self.fwd]
        # children of every node (root: -1) by rank, for acceptance recording on the host
        self.children: dict[int, dict[int, int]] = {}
        for i, par in enumerate(parents):
            self.children.setdefault(par, {})[paths[i][-1]] = i


def record_cycle(profile: AcceptanceProfile, tree: StaticTree, plan: StaticPlan, tokens: torch.Tensor,
                 path: torch.Tensor, n_acc: torch.Tensor, out: torch.Tensor) -> None:
    """Count one verified cycle: ``tokens [B, 1 + N]`` (the root first), accepted ``path [B, *]`` of tree nodes
    (0: the root), ``n_acc [B]`` accepted drafts and the exact tokens ``out [B, *]`` after every path node."""
    tokens, path, n_acc, out = (t.cpu() for t in (tokens, path, n_acc, out))
    for b in range(tokens.shape[0]):
        for i in range(int(n_acc[b]) + 1):
            node = int(path[b, i]) - 1  # -1: the root
            kids = plan.children.get(node, {})
            if not kids:
                continue
            exact = int(out[b, i])
            outcome = next((r for r, c in sorted(kids.items()) if int(tokens[b, c + 1]) == exact), None)
            level = 0 if node < 0 else len(tree.paths[node])
            profile.add(level, sorted(kids), outcome)


def measure_acceptance(model, prompts: Sequence[torch.Tensor], max_new_tokens: int, *, depth: int = 6,
                       width: int = 8, per_depth: bool = False,
                       decoding: Mapping[str, object] | None = None
                       ) -> tuple[float, ...] | tuple[tuple[float, ...], ...]:
    """The acceptance rates of ``model``'s drafter on ``prompts``, for the ``acceptance`` option of ``sequoia``.

    Decodes the prompts with the probe tree of :func:`probe_paths` (``depth`` deep, ``width`` ranks per spine node)
    and counts which rank the exact token had at every accepted node (one host synchronization per cycle).
    """
    from .config import DecodeConfig

    config = DecodeConfig(cycle_length=depth + 1, draft_policy="sequoia",
                          draft_policy_options={"paths": probe_paths(depth, width), "record_acceptance": True},
                          **dict(decoding or {}))
    engine = model.decoder(config)
    if engine.static_tree is None:
        raise ConfigError("measure_acceptance needs a model whose drafter takes tree steps")
    engine.acceptance = AcceptanceProfile()
    for prompt in prompts:
        engine.generate([prompt], max_new_tokens)
    return engine.acceptance.rates(per_depth)
