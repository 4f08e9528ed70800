"""The slot-addressed KV cache of the engine.

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

__all__ = ["KVCache", "StepBatch"]


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

    @staticmethod
    def prefill(lengths: torch.Tensor, width: int) -> StepBatch:
        """A causal pass over prompts of ``lengths`` padded to ``width`` tokens, starting at slot 0."""
        batch = lengths.shape[0]
        device = lengths.device
        positions = torch.arange(width, device=device, dtype=torch.int32).expand(batch, width).contiguous()
        return StepBatch(torch.zeros(batch, dtype=torch.int32, device=device), lengths.to(torch.int32), positions,
                         is_prefill=True, prompt=True)
