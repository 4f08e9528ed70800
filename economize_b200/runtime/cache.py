"""The slot-addressed KV caches of the engine: contiguous (:class:`KVCache`) and paged (:class:`PagedKVCache`).

One tensor ``[L, 2, B, H_kv, S, D]`` holds every layer's keys and values: row ``b`` keeps position ``p`` of its
committed sequence in slot ``p`` (economize's ``KVCache`` layout, ``src/economize/runtime/cache.py:158``, without
the trash slot: invalid tokens are simply never written). A pass over ``T`` new tokens writes them after the
committed prefix (slots ``kv_len .. kv_len + T - 1``); tree passes are compacted afterwards so the accepted path is
contiguous again. Per-head ``[S, D]`` rows are contiguous, which is the layout the attention kernel's TMA tiles read.

The cache is zero-initialised: attention tiles read whole blocks of slots and mask the invalid ones, and stale
entries must be finite so that a masked key contributes exactly zero.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

__all__ = ["KVCache", "PAGE", "PagedKVCache", "SplitKVCache", "StepBatch", "ring_pages"]

#: slots per page of a paged cache (one key tile of the attention kernel)
PAGE = 128


class KVCache:
    """Keys and values of ``num_layers`` layers for ``batch`` rows of ``capacity`` slots.

    ``dtype=torch.float8_e4m3fn`` stores e4m3 codes with one static fp32 scale per (layer, KV head): ``scales`` is
    ``(k_scale, v_scale)``, each ``[L, H_kv]`` (economize's ``kv_fp8`` with per-head scales instead of its
    ``none/token/tensor`` modes, ``src/economize/techniques/kv_quant/fp8.py:55-270``)."""

    def __init__(self, num_layers: int, batch: int, num_kv_heads: int, capacity: int, head_dim: int,
                 dtype: torch.dtype, device: torch.device | str,
                 scales: tuple[torch.Tensor, torch.Tensor] | None = None) -> None:
        self.num_layers, self.batch, self.capacity = num_layers, batch, capacity
        self.data = torch.zeros(num_layers, 2, batch, num_kv_heads, capacity, head_dim, dtype=dtype, device=device)
        self.scales = None
        if dtype == torch.float8_e4m3fn:
            if scales is None:
                ones = torch.ones(num_layers, num_kv_heads, dtype=torch.float32, device=device)
                scales = (ones, ones.clone())
            self.scales = tuple(s.to(device=device, dtype=torch.float32).contiguous() for s in scales)

    def layer(self, index: int) -> tuple[torch.Tensor, torch.Tensor]:
        return self.data[index, 0], self.data[index, 1]

    def layer_scales(self, index: int) -> tuple[torch.Tensor | None, torch.Tensor | None]:
        if self.scales is None:
            return None, None
        return self.scales[0][index], self.scales[1][index]

    @property
    def nbytes(self) -> int:
        return self.data.numel() * self.data.element_size()

    def reset(self) -> None:
        self.data.zero_()

    def pages(self, index: int) -> None:
        """A contiguous cache has no page table."""
        return None

    def compact(self, kv_len: torch.Tensor, path: torch.Tensor, n_acc: torch.Tensor) -> None:
        """Move every row's accepted tree path to consecutive slots in every layer (the compaction kernel)."""
        from .. import ops

        ops.kv_compact(self.data, kv_len, path, n_acc)

    tables = None
    paged = False


def ring_pages(window: int, reserve: int) -> int:
    """Pages of a ring that serves a sliding window of ``window`` positions while a pass writes up to ``reserve``
    new slots: the window and the pass's tokens, plus one page for the window's misaligned first page."""
    return (window + reserve + PAGE - 1) // PAGE + 1


class PagedKVCache:
    """Keys and values in a pool of 128-slot pages shared by every layer and row: ``data [P, 2, H_kv, 128, D]``
    (page ``p`` holds K and V of one (layer, row) block of 128 consecutive slots) and one page table per layer,
    ``tables [L, B, C]`` int32 (logical chunk ``c`` of row ``b`` in layer ``l`` lives in page ``tables[l, b, c]``).

    A layer of a full-attention model gets one page per chunk of its capacity. A sliding-window layer whose window
    is given in ``windows`` gets a ring instead: ``R = ring_pages(window, reserve)`` pages per row and chunk ``c``
    in page ``c mod R`` (the ring cache of economize's ``RingSpec``, ``src/economize/runtime/cache.py:72-135``), so
    its memory follows the window, not the context. ``reserve`` bounds the new slots one pass writes (a tree pass,
    or a prefill chunk: longer prompts must be prefilled in chunks of at most ``reserve`` tokens), which keeps every
    key a pass can see out of the pages it overwrites.

    The attention, rotary-store, compaction, KIVI and eviction-score kernels read the tables (``kv_row`` in
    ``csrc/common.cuh``); :meth:`layer` returns the pool views those ops take with :meth:`pages`.
    """

    paged = True

    def __init__(self, num_layers: int, batch: int, num_kv_heads: int, capacity: int, head_dim: int,
                 dtype: torch.dtype, device: torch.device | str,
                 scales: tuple[torch.Tensor, torch.Tensor] | None = None, windows: list[int] | None = None,
                 reserve: int = 512) -> None:
        self.num_layers, self.batch, self.num_kv_heads, self.head_dim = num_layers, batch, num_kv_heads, head_dim
        chunks = (capacity + PAGE - 1) // PAGE
        self.capacity = chunks * PAGE
        self.reserve = reserve
        windows = list(windows or [0] * num_layers)
        self.rings = [min(chunks, ring_pages(w, reserve)) if w else 0 for w in windows]
        tables = torch.empty(num_layers, batch, chunks, dtype=torch.int32)
        first = 0
        col = torch.arange(chunks)
        for layer in range(num_layers):
            per_row = self.rings[layer] or chunks
            for b in range(batch):
                tables[layer, b] = first + col % per_row
                first += per_row
        self.tables = tables.to(device)
        self.data = torch.zeros(first, 2, num_kv_heads, PAGE, head_dim, dtype=dtype, device=device)
        self.scales = None
        if dtype == torch.float8_e4m3fn:
            if scales is None:
                ones = torch.ones(num_layers, num_kv_heads, dtype=torch.float32, device=device)
                scales = (ones, ones.clone())
            self.scales = tuple(s.to(device=device, dtype=torch.float32).contiguous() for s in scales)

    @property
    def num_pages(self) -> int:
        return self.data.shape[0]

    def layer(self, index: int) -> tuple[torch.Tensor, torch.Tensor]:
        """Views ``[P, H_kv, 128, D]`` of every page's K and V blocks (pages 2 H_kv 128 rows apart)."""
        return self.data[:, 0], self.data[:, 1]

    def pages(self, index: int) -> torch.Tensor:
        """Layer ``index``'s page table ``[B, C]``."""
        return self.tables[index]

    def compact(self, kv_len: torch.Tensor, path: torch.Tensor, n_acc: torch.Tensor) -> None:
        from .. import ops

        ops.kv_compact(self.data, kv_len, path, n_acc, self.tables)

    def window_of(self, index: int) -> int:
        return self.rings[index] * PAGE if self.rings[index] else 0

    def layer_scales(self, index: int) -> tuple[torch.Tensor | None, torch.Tensor | None]:
        if self.scales is None:
            return None, None
        return self.scales[0][index], self.scales[1][index]

    @property
    def nbytes(self) -> int:
        return self.data.numel() * self.data.element_size()

    def reset(self) -> None:
        self.data.zero_()

    def logical(self, index: int, kv: int) -> torch.Tensor:
        """Layer ``index``'s K (``kv = 0``) or V as a logical ``[B, H_kv, S, D]`` copy (a ring layer's chunks repeat
        their page: only the window's slots are meaningful)."""
        pages = self.data[self.tables[index].long(), kv]  # [B, C, H_kv, 128, D]
        b, c, h, _, d = pages.shape
        return pages.permute(0, 2, 1, 3, 4).reshape(b, h, c * PAGE, d)


@dataclass
class StepBatch:
    """Where the tokens of one pass sit.

    Attributes:
        kv_len: ``[B]`` int32 committed slots per row; the pass's tokens go after them.
        n_new: ``[B]`` int32 valid slots of the pass's new region per row (padding tokens beyond are not written
            and are invisible).
        positions: ``[B, T]`` int32 rotary position of every query token.
        mask: ``[B, T]`` int64 ancestor bits over the new region (bit ``j``: slot ``kv_len + j`` is visible), or
            ``None`` for causal visibility (``j <= q_offset + t``).
        q_offset: Index of the first query token inside the new region (tree steps of a drafter append a frontier
            after the nodes they already wrote).
    """

    kv_len: torch.Tensor
    n_new: torch.Tensor
    positions: torch.Tensor
    mask: torch.Tensor | None = None
    q_offset: int = 0
    #: a prompt pass starting at slot 0 (KV eviction scores the prompt during it)
    is_prefill: bool = False
    #: a pass over prompt tokens (a whole prefill or one chunk of a chunked prefill): attention reduces its keys by
    #: slot, without the exact tail of decode passes, so a chunked prefill matches a whole one
    prompt: bool = False

    def to(self, device: torch.device | str) -> StepBatch:
        """This batch with its tensors on ``device``."""
        move = (lambda t: None if t is None else t.to(device))
        return StepBatch(move(self.kv_len), move(self.n_new), move(self.positions), move(self.mask), self.q_offset,
                         self.is_prefill, self.prompt)

    @staticmethod
    def prefill(lengths: torch.Tensor, width: int) -> StepBatch:
        """A causal pass over prompts of ``lengths`` padded to ``width`` tokens, starting at slot 0."""
        batch = lengths.shape[0]
        device = lengths.device
        positions = torch.arange(width, device=device, dtype=torch.int32).expand(batch, width).contiguous()
        return StepBatch(torch.zeros(batch, dtype=torch.int32, device=device), lengths.to(torch.int32), positions,
                         is_prefill=True, prompt=True)


class SplitKVCache:
    """The cache of a model whose layers are split over devices (pipeline placement): one contiguous
    :class:`KVCache` per stage, on the stage's device, holding that stage's layers."""

    paged = False
    tables = None

    def __init__(self, parts: list[tuple[range, KVCache]]) -> None:
        self.parts = parts
        self._of: dict[int, tuple[int, KVCache]] = {}
        for layers, part in parts:
            for i in layers:
                self._of[i] = (i - layers.start, part)
        first = parts[0][1]
        self.num_layers = sum(len(r) for r, _ in parts)
        self.batch, self.capacity = first.batch, first.capacity

    def layer(self, index: int) -> tuple[torch.Tensor, torch.Tensor]:
        local, part = self._of[index]
        return part.layer(local)

    def layer_scales(self, index: int) -> tuple[torch.Tensor | None, torch.Tensor | None]:
        local, part = self._of[index]
        return part.layer_scales(local)

    def pages(self, index: int) -> None:
        return None

    @property
    def data(self) -> torch.Tensor:
        raise AttributeError("a split cache has one tensor per stage (see parts)")

    @property
    def nbytes(self) -> int:
        return sum(part.nbytes for _, part in self.parts)

    def reset(self) -> None:
        for _, part in self.parts:
            part.reset()

    def compact(self, kv_len: torch.Tensor, path: torch.Tensor, n_acc: torch.Tensor) -> None:
        for _, part in self.parts:
            dev = part.data.device
            part.compact(kv_len.to(dev), path.to(dev), n_acc.to(dev))
