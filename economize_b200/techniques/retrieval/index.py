"""A persistent token datastore for retrieval drafting: a suffix array over records of tokens.

The records are concatenated with a separator (-1) between them; the suffix array orders every start position by
the suffix's first ``depth`` tokens (prefix doubling: ranks of length-``k`` prefixes give ranks of length-``2k``
prefixes through pairs ``(rank_k(i), rank_k(i + k))``, sorted with ``numpy.lexsort``). A context's longest suffix
found in the datastore is located by binary search; because the array is sorted, the occurrences of a pattern are
one contiguous range, and the tokens that follow them are sorted within it, so every continuation's count and
sub-range come from one pass over that column (REST, He et al. 2024: the most frequent continuations of the
longest matching suffix).

On disk an index is a folder: ``tokens.npy`` (int32, separators included), ``sa.npy`` (int64) and ``meta.json``;
loading can memory-map the arrays, so the datastore need not fit in RAM.
"""

from __future__ import annotations

import heapq
import json
from collections.abc import Iterable
from pathlib import Path

import numpy as np

__all__ = ["FORMAT", "SEPARATOR", "SuffixIndex", "suffix_array"]

SEPARATOR = -1
FORMAT = "economize_b200.suffix_index.v1"
MAX_SCAN = 1 << 16  # occurrences of one pattern read when counting its continuations


def suffix_array(tokens: np.ndarray, depth: int = 64) -> np.ndarray:
    """Start positions of ``tokens`` (int, separators < 0) ordered by their first ``depth`` tokens."""
    n = len(tokens)
    if n == 0:
        return np.zeros(0, dtype=np.int64)
    rank = np.asarray(tokens, dtype=np.int64) - SEPARATOR  # separators rank 0, tokens >= 1
    sep = rank == 0
    order = np.argsort(rank, kind="stable")
    k = 1
    while k < depth:
        nxt = np.zeros(n, dtype=np.int64)
        nxt[: n - k] = rank[k:]
        order = np.lexsort((nxt, rank))
        r, x = rank[order], nxt[order]
        fresh = np.ones(n, dtype=np.int64)
        fresh[1:] = (r[1:] != r[:-1]) | (x[1:] != x[:-1])
        new = np.empty(n, dtype=np.int64)
        new[order] = np.cumsum(fresh)
        new[sep] = 0  # a separator stays the smallest "token"
        rank = new
        if fresh.sum() == n:  # every prefix distinct: the order is final
            break
        k *= 2
    return order.astype(np.int64)


class SuffixIndex:
    def __init__(self, tokens: np.ndarray, sa: np.ndarray, depth: int, num_records: int) -> None:
        self.tokens, self.sa, self.depth, self.num_records = tokens, sa, int(depth), int(num_records)

    def __len__(self) -> int:
        return int(len(self.tokens) - self.num_records)

    # ---- building and persistence -----------------------------------------------------------------------------
    @classmethod
    def build(cls, records: Iterable, depth: int = 64) -> SuffixIndex:
        """Index ``records`` (token sequences: lists, arrays or tensors)."""
        parts, count = [], 0
        for rec in records:
            arr = np.asarray(rec.tolist() if hasattr(rec, "tolist") else rec, dtype=np.int64).reshape(-1)
            parts += [arr, np.array([SEPARATOR], dtype=np.int64)]
            count += 1
        tokens = np.concatenate(parts) if parts else np.zeros(0, dtype=np.int64)
        return cls(tokens.astype(np.int32), suffix_array(tokens, depth), depth, count)

    def save(self, folder: str | Path) -> None:
        folder = Path(folder)
        folder.mkdir(parents=True, exist_ok=True)
        np.save(folder / "tokens.npy", np.asarray(self.tokens, dtype=np.int32))
        np.save(folder / "sa.npy", np.asarray(self.sa, dtype=np.int64))
        (folder / "meta.json").write_text(json.dumps({"format": FORMAT, "depth": self.depth,
                                                      "records": self.num_records, "tokens": len(self)}))

    @classmethod
    def load(cls, folder: str | Path, mmap: bool = False) -> SuffixIndex:
        folder = Path(folder)
        meta = json.loads((folder / "meta.json").read_text())
        if meta.get("format") != FORMAT:
            raise ValueError(f"{folder} is not a suffix index ({meta.get('format')!r})")
        mode = "r" if mmap else None
        return cls(np.load(folder / "tokens.npy", mmap_mode=mode), np.load(folder / "sa.npy", mmap_mode=mode),
                   meta["depth"], meta["records"])

    # ---- queries ----------------------------------------------------------------------------------------------
    def _compare(self, pos: int, pattern: list[int]) -> int:
        """-1 / 0 / 1: the suffix at ``pos`` against ``pattern`` over the pattern's length."""
        seg = self.tokens[pos:pos + len(pattern)]
        for a, b in zip(seg, pattern):
            if a != b:
                return -1 if a < b else 1
        return 0 if len(seg) == len(pattern) else -1

    def find(self, pattern: list[int], lo: int = 0, hi: int | None = None) -> tuple[int, int]:
        """The suffix-array range of the suffixes that start with ``pattern`` (empty: ``lo == hi``)."""
        hi = len(self.sa) if hi is None else hi
        a, b = lo, hi
        while a < b:  # first suffix >= pattern
            mid = (a + b) // 2
            if self._compare(int(self.sa[mid]), pattern) < 0:
                a = mid + 1
            else:
                b = mid
        first = a
        b = hi
        while a < b:  # first suffix > pattern
            mid = (a + b) // 2
            if self._compare(int(self.sa[mid]), pattern) <= 0:
                a = mid + 1
            else:
                b = mid
        return first, a

    def match(self, context: list[int], max_context: int, min_match: int) -> tuple[int, int, int]:
        """``(length, lo, hi)`` of the longest suffix of ``context`` (at most ``max_context`` tokens, at least
        ``min_match``) that the datastore holds; length 0 when none does."""
        for m in range(min(max_context, len(context), self.depth), min_match - 1, -1):
            lo, hi = self.find(context[len(context) - m:])
            if hi > lo:
                return m, lo, hi
        return 0, 0, 0

    def _children(self, lo: int, hi: int, offset: int) -> list[tuple[int, int, int, int]]:
        """``(count, token, lo, hi)`` of every token that follows the range's suffixes at ``offset``."""
        hi_scan = min(hi, lo + MAX_SCAN)
        pos = np.asarray(self.sa[lo:hi_scan], dtype=np.int64) + offset
        inside = pos < len(self.tokens)
        col = np.full(len(pos), SEPARATOR, dtype=np.int64)
        col[inside] = np.asarray(self.tokens, dtype=np.int64)[pos[inside]]
        if len(col) == 0:
            return []
        starts = np.flatnonzero(np.concatenate([[True], col[1:] != col[:-1]]))
        ends = np.append(starts[1:], len(col))
        out = []
        for s, e in zip(starts, ends):
            tok = int(col[s])
            if tok != SEPARATOR:
                out.append((int(e - s), tok, lo + int(s), lo + int(e)))
        return out

    def draft_tree(self, context: list[int], budget: int, max_depth: int, branch: int, min_match: int,
                   max_context: int = 16) -> tuple[list[int], list[int]]:
        """The draft tree (tokens, parents as draft indices, -1 = the root) of the most frequent continuations of
        the longest matching suffix: best-first by occurrence count, at most ``branch`` children per node."""
        m, lo, hi = self.match(context, max_context, min_match)
        if m == 0:
            return [], []
        tokens: list[int] = []
        parents: list[int] = []
        heap = [(-c, tok, -1, 1, clo, chi) for c, tok, clo, chi in
                sorted(self._children(lo, hi, m), reverse=True)[:branch]]
        heapq.heapify(heap)
        while heap and len(tokens) < budget:
            neg, tok, parent, depth, clo, chi = heapq.heappop(heap)
            node = len(tokens)
            tokens.append(tok)
            parents.append(parent)
            if depth < max_depth:
                for c, t2, l2, h2 in sorted(self._children(clo, chi, m + depth), reverse=True)[:branch]:
                    heapq.heappush(heap, (-c, t2, node, depth + 1, l2, h2))
        return tokens, parents
