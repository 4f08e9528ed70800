"""KV-cache memory accounting of a generation (economize ``techniques/_kv/wrapper.py:62-130``, ``RowStats`` and
``KVStats``).

Per row, in bytes: the committed entries in the cache's storage format at the row's last exact pass (``kv_bytes``)
and in the plain compute dtype (``kv_bytes_full``), and the sums over the row's exact passes of the committed bytes
attention read (``kv_bytes_read``, ``kv_bytes_read_full``). The formats are modelled entry by entry:

* fp8 caches: one byte per element (the per-head scales are static and counted once per layer, not per entry);
* KIVI: the 128-token chunks that lie ``residual`` slots behind the committed length cost their coded size
  (codes + scales + zeros), the rest bf16;
* sliding-window layers: at most ``window`` entries (what a ring of the window's size would hold and what the
  windowed kernel reads);
* eviction keep bitmaps: only the kept committed entries.

``allocated_bytes`` is the measured counterpart: every device buffer the generation's cache held.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

__all__ = ["KVStats", "RowKVStats", "held_bytes", "keep_snapshot", "row_kv_stats"]


@dataclass
class RowKVStats:
    kv_bytes: float = 0.0
    kv_bytes_full: float = 0.0
    kv_bytes_read: float = 0.0
    kv_bytes_read_full: float = 0.0
    passes: int = 0

    @property
    def compression(self) -> float:
        return self.kv_bytes_full / self.kv_bytes if self.kv_bytes > 0 else 1.0

    def as_dict(self) -> dict[str, float]:
        return {"kv_bytes": self.kv_bytes, "kv_bytes_full": self.kv_bytes_full, "kv_bytes_read": self.kv_bytes_read,
                "kv_bytes_read_full": self.kv_bytes_read_full, "kv_passes": float(self.passes),
                "kv_compression": self.compression}


@dataclass
class KVStats:
    """One generation: modelled bytes per row and the measured bytes of the cache's buffers."""

    rows: list[RowKVStats]
    allocated_bytes: int = 0


def held_bytes(model, cache) -> int:
    """Bytes of every device buffer that holds the generation's keys and values (cache, KIVI codes, keep bitmaps)."""
    total = cache.nbytes
    quantizer = getattr(model, "kv_quantizer", None)
    if quantizer is not None and hasattr(quantizer, "storage"):
        data, chunks = quantizer.storage(cache)
        total += data.numel() * data.element_size() + chunks.numel() * chunks.element_size()
    keep = getattr(getattr(model, "kv_evictor", None), "keep", None)
    if isinstance(keep, torch.Tensor):
        total += keep.numel() * keep.element_size()
    return int(total)


def _kept_counts(keep_row: torch.Tensor) -> torch.Tensor:
    """Running counts of kept slots ``[L, H_kv, S + 1]`` (entry ``n``: kept slots below ``n``) of one row's bit
    words ``[L, H_kv, S / 32]``."""
    bits = ((keep_row.long()[..., None] >> torch.arange(32)) & 1).reshape(*keep_row.shape[:2], -1).int()
    return torch.nn.functional.pad(bits.cumsum(-1, dtype=torch.int32), (1, 0))


def _bytes_at(model, n: int, kept: torch.Tensor | None) -> tuple[float, float]:
    """(stored, full) bytes of ``n`` committed entries of one row over all layers."""
    c = model.config
    hkv, d = model.local["num_kv_heads"], c.head_dim
    full_entry = 2 * hkv * d * model.dtype.itemsize  # K and V of one position, one layer
    stored_entry = 2 * hkv * d * (1 if model.kv_dtype == torch.float8_e4m3fn else model.dtype.itemsize)
    quantizer = getattr(model, "kv_quantizer", None)
    stored = full = 0.0
    for layer in range(c.num_layers):
        window = c.window_of(layer)
        visible = min(n, window) if window else n
        if kept is not None:
            visible = min(visible, int(kept[layer].max()))  # kept entries of the fullest head
        full += n * full_entry
        if quantizer is not None and hasattr(quantizer, "config") and hasattr(quantizer.config, "bits"):
            from ..ops.kivi import chunk_bytes

            residual = quantizer.config.residual
            coded = min(max(0, (n - residual) // 128) * 128, visible // 128 * 128)
            # one coded chunk holds 128 positions' keys and values of one KV head
            stored += (coded // 128) * hkv * chunk_bytes(quantizer.config.bits, d) + (visible - coded) * stored_entry
        else:
            stored += visible * stored_entry
    return stored, full


def keep_snapshot(model) -> torch.Tensor | None:
    """The eviction keep bitmaps ``[L, B, H_kv, S / 32]`` of the last generation on the host (None without)."""
    keep = getattr(getattr(model, "kv_evictor", None), "keep", None)
    return keep.cpu() if isinstance(keep, torch.Tensor) and keep.dim() == 4 else None


def row_kv_stats(model, keep: torch.Tensor | None, row: int, prompt_len: int, accepted: list[int]) -> RowKVStats:
    """The accounting of one row: ``accepted`` drafts per exact pass after a prompt of ``prompt_len`` tokens;
    ``keep``: :func:`keep_snapshot` taken when the generation ended."""
    counts = _kept_counts(keep[:, row]) if keep is not None else None

    def kept(n: int):
        return None if counts is None else counts[..., min(n, counts.shape[-1] - 1)]

    stats = RowKVStats()
    n = prompt_len
    for a in accepted:
        s, f = _bytes_at(model, n, kept(n))
        stats.kv_bytes_read += s
        stats.kv_bytes_read_full += f
        stats.passes += 1
        n += int(a) + 1
    stats.kv_bytes, stats.kv_bytes_full = _bytes_at(model, n, kept(n))
    return stats
