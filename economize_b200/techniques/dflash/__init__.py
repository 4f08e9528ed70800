"""DFlash block drafting (``dflash``; Chen et al., 2026; economize ``techniques/dflash``): a draft layer conditioned
on fused target features drafts a whole block in one forward from ``[anchor, mask, ..., mask]``.

The draft layer is EAGLE-3's (fused low/mid/high target states, its own KV cache of the committed context). After
the context catch-up, the anchor (the target's token after the last committed position) is the root step, and one
more forward over ``block_size - 1`` mask tokens at the following positions, with bidirectional attention inside the
block (every block slot's ancestor bit set), produces the remaining drafts, read out through the head. The target
verifies (lossless). The ``dflash_block`` objective (:mod:`.objective`) trains the root and the block drafts against
the target's distributions. Not built: the z-lab / speculators checkpoint readers.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import ClassVar

import torch

from ...core.technique import register_technique
from ...decoding.config import DecodeConfig
from ...errors import ConfigError
from ...runtime.cache import StepBatch
from ..eagle3.config import Eagle3Config
from ..eagle3.technique import Eagle3Drafter, Eagle3Technique

__all__ = ["DFlashConfig", "DFlashDrafter", "DFlashTechnique"]


@dataclass(frozen=True)
class DFlashConfig(Eagle3Config):
    """``block_size``: tokens per drafted block (the anchor included); ``mask_token_id``: the mask token (``None``:
    the last vocabulary id)."""

    technique: ClassVar[str] = "dflash"
    block_size: int = 8
    mask_token_id: int | None = None

    def __post_init__(self) -> None:
        super().__post_init__()
        if not 2 <= self.block_size <= 64:
            raise ConfigError("block_size must lie in 2 .. 64 (the block's ancestor bits are one int64)")


class DFlashDrafter(Eagle3Drafter):
    def __init__(self, technique: DFlashTechnique) -> None:
        super().__init__(technique)
        self.block = technique.config.block_size
        v = technique.model.config.vocab_size
        self.mask_id = technique.config.mask_token_id if technique.config.mask_token_id is not None else v - 1
        self.stash: torch.Tensor | None = None
        self._depth = 0

    def begin(self, batch: int, capacity: int) -> None:
        super().begin(batch, capacity + self.block)
        vd = self.t.draft_vocab
        if self.stash is None or self.stash.shape[0] != batch:
            self.stash = torch.zeros(batch, self.block - 1, vd, dtype=torch.float32, device=self.t.model.device)

    def observe(self, tokens, sources, kv_len, n_valid, root):
        logits, out = super().observe(tokens, sources, kv_len, n_valid, root)
        batch = tokens.shape[0]
        dev = tokens.device
        m = self.block - 1
        base = (kv_len + root + 1).to(torch.int32)  # the slots after the anchor
        pos = (base[:, None] + torch.arange(m, device=dev, dtype=torch.int32)[None]).contiguous()
        masks = torch.full((batch, m), self.mask_id, dtype=torch.long, device=dev)
        every = torch.full((batch, m), (1 << m) - 1, dtype=torch.int64, device=dev)  # bidirectional block
        feats = torch.zeros(batch, m, out.shape[-1], dtype=self.t.fc.dtype, device=dev)
        mlp, a = self._step(masks, feats, StepBatch(base, torch.full((batch,), m, dtype=torch.int32, device=dev),
                                                     pos, every, 0))
        block_logits, _ = self._head(mlp, a)
        self.stash.copy_(block_logits)
        self._depth = 0
        return logits, out

    def tree_step(self, tokens, states, positions, kv_base, n_forwarded, q_offset, mask):
        i = min(self._depth, self.stash.shape[1] - 1)
        self._depth += 1
        return self.stash[:, i][:, None].expand(-1, tokens.shape[1], -1), states


@register_technique
class DFlashTechnique(Eagle3Technique):
    config_class = DFlashConfig
    objective_name = "dflash_block"

    def drafter(self) -> DFlashDrafter:
        return DFlashDrafter(self)

    def default_decoding(self) -> DecodeConfig:
        return DecodeConfig(cycle_length=self.config.block_size)


from . import objective as _objective  # noqa: E402,F401  (registers the dflash_block objective)
