"""Sequoia draft trees: one static tree of the best shape for measured acceptance rates and latencies (Chen et al.,
2024, "Sequoia: Scalable, Robust, and Hardware-aware Speculative Decoding"; economize ``decoding/sequoia.py:1-572``).

``DecodeConfig(draft_policy="sequoia", draft_policy_options={"acceptance": (0.6, 0.15, 0.06, 0.03),
"total_tokens": 32, "depth": 8})`` turns a chain drafter (any drafter with tree steps) into a drafter of one fixed
tree per cycle. Every node names its rank among its siblings; a proposal fills the tree with the drafter's
``rank``-th most likely token after every parent, one batched draft step per depth over the nodes of that depth that
have children. The exact pass verifies it as any draft tree, so decoding stays lossless.

``acceptance[r]`` is the probability that the exact model's token after an accepted node is the drafter's ``r``-th
most likely token (or one such vector per depth of the parent node, the root's first and the last reused below).
The events are disjoint across siblings, so a tree's expected tokens per cycle is the sum over its nodes of the
product of the rates along the node's rank path, plus one for the root. :func:`sequoia_tree` maximizes this over
trees of at most ``total_tokens`` nodes and depth at most ``depth`` by dynamic programming: ``G[l][n]`` is the best
value of a subtree of at most ``n`` nodes whose root has depth ``l``, and the root's children are placed rank by
rank as a knapsack over the remaining ``n - 1`` nodes (a rank may also be left out, so measured rates that are not
decreasing are used as they are). With measured latencies (``verify_latency[i]``: one exact pass over ``i + 1``
tokens; ``draft_latency``: one draft step) the size and depth are those of the most tokens per second, which is
Sequoia's hardware-aware choice.

:func:`measure_acceptance` estimates the rates by decoding prompts with a probe tree and counting which rank the
exact token had at every accepted node; an explicit tree can be given as rank ``paths`` instead (the format of
Medusa's tree choices).
"""

from __future__ import annotations

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
    """A draft tree as rank paths, sorted by depth then rank (so every parent precedes its children).

    Attributes:
        paths: ``paths[i]`` is the rank path of node ``i`` (``(0, 2)``: the 3rd best token after the best first
            token).
        expected: Expected tokens per cycle under the rates it was built for (``None`` for an explicit tree).
    """

    paths: tuple[Path, ...]
    expected: float | None = None

    @classmethod
    def from_paths(cls, paths: Sequence[Sequence[int]], expected: float | None = None) -> StaticTree:
        clean = sorted({tuple(int(r) for r in p) for p in paths}, key=lambda q: (len(q), q))
        if not clean:
            raise ConfigError("a static draft tree needs at least one path")
        have = set(clean)
        for p in clean:
            if not p or any(r < 0 for r in p):
                raise ConfigError(f"tree path {p} must be a non-empty sequence of ranks >= 0")
            if len(p) > 1 and p[:-1] not in have:
                raise ConfigError(f"tree path {p} has no parent path {p[:-1]}")
        return cls(tuple(clean), expected)

    @property
    def size(self) -> int:
        return len(self.paths)

    @property
    def depth(self) -> int:
        return max(len(p) for p in self.paths)

    @property
    def parents(self) -> tuple[int, ...]:
        """Parent node of every node (``-1``: a child of the root)."""
        index = {p: i for i, p in enumerate(self.paths)}
        return tuple(index[p[:-1]] if len(p) > 1 else -1 for p in self.paths)

    @property
    def ranks(self) -> tuple[int, ...]:
        return tuple(p[-1] for p in self.paths)

    @property
    def forwarded(self) -> int:
        """Nodes that run through the drafter (those with children)."""
        return len({p[:-1] for p in self.paths if len(p) > 1})


def _rates(acceptance: Sequence[float] | Sequence[Sequence[float]], depth: int) -> np.ndarray:
    """The rates as a matrix ``[depth, R]``: row ``l`` holds the rates after a node of depth ``l`` (root: 0)."""
    rows = acceptance if len(acceptance) and isinstance(acceptance[0], (Sequence, np.ndarray)) else [acceptance]
    rows = [[float(v) for v in row] for row in rows]
    width = max((len(r) for r in rows), default=0)
    if width == 0:
        raise ConfigError("the acceptance vector is empty")
    for row in rows:
        if any(not 0.0 <= v <= 1.0 for v in row) or sum(row) > 1.0 + 1e-6:
            raise ConfigError(f"acceptance rates {row} must lie in [0, 1] and sum to at most 1 (they are "
                              "probabilities of disjoint events)")
    out = np.zeros((depth, width))
    for level in range(depth):
        row = rows[min(level, len(rows) - 1)]
        out[level, :len(row)] = row
    return out


def expected_tokens(tree: StaticTree | Sequence[Sequence[int]],
                    acceptance: Sequence[float] | Sequence[Sequence[float]]) -> float:
    """Expected tokens per cycle of ``tree`` (the root's token included) under the rates ``acceptance``."""
    if not isinstance(tree, StaticTree):
        tree = StaticTree.from_paths(tree)
    p = _rates(acceptance, tree.depth)
    reach: dict[Path, float] = {(): 1.0}
    for path in tree.paths:
        level, rank = len(path) - 1, path[-1]
        reach[path] = reach[path[:-1]] * (p[level, rank] if rank < p.shape[1] else 0.0)
    return float(sum(reach.values()))


def _solve(p: np.ndarray, nodes: int) -> tuple[np.ndarray, list[list[np.ndarray]]]:
    """Dynamic program over the rate matrix ``p [D, R]``: ``G [D + 1, nodes + 1]`` and, for every level and rank,
    the subtree size given to that rank's child for every remaining budget (0: the rank is left out)."""
    depth, ranks = p.shape
    g = np.zeros((depth + 1, nodes + 1))
    g[depth, 1:] = 1.0  # a node at the largest depth has no children
    m = np.arange(nodes + 1)[:, None]
    t = np.arange(nodes + 1)[None, :]
    fits = (t >= 1) & (t <= m)
    rest = np.clip(m - t, 0, nodes)
    sizes: list[list[np.ndarray]] = [[] for _ in range(depth)]
    for level in range(depth - 1, -1, -1):
        h = np.zeros(nodes + 1)  # best use of a budget by the ranks after the current one
        per_rank: list[np.ndarray] = []
        for rank in range(ranks - 1, -1, -1):
            gain = np.where(fits, p[level, rank] * g[level + 1][t] + h[rest], -np.inf)
            best_t = gain.argmax(1)
            best = gain[np.arange(nodes + 1), best_t]
            take = best > h + 1e-15
            per_rank.append(np.where(take, best_t, 0))
            h = np.where(take, best, h)
        sizes[level] = per_rank[::-1]
        g[level, 1:] = 1.0 + h[:-1]
    return g, sizes


def _paths(sizes: list[list[np.ndarray]], level: int, nodes: int, prefix: Path, out: list[Path]) -> None:
    """Append the rank paths of the best subtree of ``nodes`` nodes rooted at ``prefix`` (of depth ``level``)."""
    budget = nodes - 1
    if level >= len(sizes):
        return
    for rank, table in enumerate(sizes[level]):
        if budget <= 0:
            break
        take = int(table[budget])
        if take:
            child = prefix + (rank,)
            out.append(child)
            _paths(sizes, level + 1, take, child, out)
            budget -= take


def sequoia_tree(acceptance: Sequence[float] | Sequence[Sequence[float]], total_tokens: int, depth: int, *,
                 verify_latency: Sequence[float] | None = None, draft_latency: float = 0.0) -> StaticTree:
    """The Sequoia tree for ``acceptance`` with at most ``total_tokens`` nodes and depth at most ``depth``.

    Without ``verify_latency`` the tree maximizes expected tokens per cycle; with it (one entry per exact pass of
    ``1 .. total_tokens + 1`` tokens) it maximizes expected tokens per second over every size and depth, a cycle of
    depth ``d`` costing ``verify_latency[n] + d * draft_latency``.
    """
    if not (is_positive_int(total_tokens) and is_positive_int(depth)):
        raise ConfigError(f"a sequoia tree needs total_tokens >= 1 and depth >= 1, got {total_tokens} and {depth}")
    if draft_latency < 0:
        raise ConfigError(f"draft_latency must be >= 0, got {draft_latency}")
    p = _rates(acceptance, depth)
    if verify_latency is None:
        g, sizes = _solve(p, total_tokens + 1)
        paths: list[Path] = []
        _paths(sizes, 0, total_tokens + 1, (), paths)
        if not paths:
            raise ConfigError("every acceptance rate is 0: no tree adds an expected token")
        return StaticTree.from_paths(paths, float(g[0, total_tokens + 1]))
    if len(verify_latency) < total_tokens + 1 or any(float(v) <= 0 for v in verify_latency):
        raise ConfigError(f"verify_latency needs a positive entry for every pass of 1..{total_tokens + 1} tokens")
    best: tuple[float, int, int, list] | None = None
    for d in range(1, depth + 1):
        g, sizes = _solve(p[:d], total_tokens + 1)
        for n in range(1, total_tokens + 1):
            rate = g[0, n + 1] / (float(verify_latency[n]) + d * draft_latency)
            if best is None or rate > best[0] * (1 + 1e-12):
                best = (rate, d, n, sizes)
    _, d, n, sizes = best
    paths = []
    _paths(sizes, 0, n + 1, (), paths)
    if not paths:
        raise ConfigError("every acceptance rate is 0: no tree adds an expected token")
    tree = StaticTree.from_paths(paths)
    return StaticTree(tree.paths, expected_tokens(tree, p[:d].tolist()))


def probe_paths(depth: int, width: int) -> tuple[Path, ...]:
    """A probe tree: a spine of rank-0 nodes ``depth`` deep; the root and every spine node but the last have the
    children of ranks ``0 .. width - 1``."""
    return tuple((0,) * level + (rank,) for level in range(depth) for rank in range(width))


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
    unknown = sorted(set(options) - set(_OPTIONS))
    if unknown:
        raise ConfigError(f"draft_policy 'sequoia' has no options {unknown}; it takes {', '.join(_OPTIONS)}")
    record = options.get("record_acceptance", False)
    if not isinstance(record, bool):
        raise ConfigError(f"record_acceptance must be a bool, got {record!r}")
    if ("paths" in options) == ("acceptance" in options):
        raise ConfigError("draft_policy 'sequoia' needs exactly one of 'acceptance' and 'paths'")
    if "paths" in options:
        extra = sorted(set(options) & {"total_tokens", "depth", "verify_latency", "draft_latency"})
        if extra:
            raise ConfigError(f"options {extra} shape a tree from 'acceptance'; an explicit 'paths' tree takes none")
        tree = StaticTree.from_paths(options["paths"])
    else:
        depth = options.get("depth", max(cycle_length - 1, 1))
        total = options.get("total_tokens", 32)
        for name, value in (("depth", depth), ("total_tokens", total)):
            if not is_positive_int(value):
                raise ConfigError(f"draft_policy 'sequoia' needs a positive integer {name}, got {value!r}")
        draft = options.get("draft_latency", 0.0)
        if isinstance(draft, bool) or not isinstance(draft, (int, float)) or draft < 0:
            raise ConfigError(f"draft_latency must be a number >= 0, got {draft!r}")
        latency = options.get("verify_latency")
        if "draft_latency" in options and latency is None:
            raise ConfigError("draft_latency needs verify_latency")
        tree = sequoia_tree(options["acceptance"], int(total), int(depth), verify_latency=latency,
                            draft_latency=float(draft))
    if tree.size + 1 > MAX_FORWARDED or tree.forwarded > MAX_FORWARDED:
        raise ConfigError(f"a verified tree holds at most {MAX_FORWARDED - 1} draft nodes, got {tree.size}")
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
