"""2:4 semi-structured sparse weights: packed storage and the PyTorch reference.

Every group of four consecutive input columns of a row keeps at most two values. :class:`Sparse24Weight` stores
the kept values ``[N, K/2]`` (bf16) and their positions ``[N/2, K/4]`` (uint8: per row and 64-wide K block 8
bytes, 4 bits per group = the two positions, rows ``2p`` and ``2p+1`` sharing a 16-byte line so that one TMA box
covers a 128-row tile). ``ops.linear`` runs the weight-streaming tcgen05 GEMM of ``csrc/gemm_wq.cu``, which expands
the tile to dense bf16 in shared memory: a decode pass, bound by weight bytes, reads 56 % of them (economize
stores 2:4 weights through torch's cuSPARSELt/CUTLASS semi-structured tensors, ``techniques/prune/
semi_kernels.py:46-211``).
"""

from __future__ import annotations

import torch
from torch import nn

from ..errors import ConfigError

__all__ = ["Sparse24Weight", "mask_24", "pack_24", "unpack_24"]


def mask_24(score: torch.Tensor) -> torch.Tensor:
    """Boolean mask keeping the two highest-scoring entries of every group of four along the last dim."""
    n, k = score.shape
    g = score.reshape(n, k // 4, 4)
    top = g.topk(2, -1).indices
    m = torch.zeros_like(g, dtype=torch.bool).scatter_(-1, top, True)
    return m.reshape(n, k)


def pack_24(w: torch.Tensor, mask: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Kept values ``[N, K/2]`` and positions ``[N/2, K/4]`` of a 2:4-sparse ``w`` (``mask`` selects the kept entries;
    default: the two largest magnitudes per group)."""
    n, k = w.shape
    if k % 64 or n % 2:
        raise ConfigError(f"2:4 packing needs K % 64 == 0 and an even row count, got {tuple(w.shape)}")
    mask = mask_24(w.abs().float()) if mask is None else mask
    g = mask.reshape(n, k // 4, 4)
    if (g.sum(-1) > 2).any():
        raise ConfigError("the mask keeps more than two entries of a group of four")
    # pad groups with fewer than two kept entries with the first free positions (their values are zero)
    order = torch.argsort((~g).to(torch.int8), dim=-1, stable=True)[..., :2]  # kept positions first, ascending
    pos = order.sort(-1).values
    vals = w.reshape(n, k // 4, 4).gather(-1, pos) * g.gather(-1, pos)
    nib = (pos[..., 0] | (pos[..., 1] << 2)).to(torch.int64)  # [N, K/4] 4-bit codes
    per_block = nib.reshape(n, k // 64, 16)
    word = torch.zeros(n, k // 64, dtype=torch.int64, device=w.device)
    for i in range(16):
        word |= per_block[..., i] << (4 * i)
    bytes_ = torch.stack([(word >> (8 * b)) & 0xFF for b in range(8)], -1).to(torch.uint8)  # [N, K/64, 8]
    meta = bytes_.reshape(n // 2, 2, k // 64, 8).permute(0, 2, 1, 3).reshape(n // 2, k // 4)
    return vals.reshape(n, k // 2).to(w.dtype).contiguous(), meta.contiguous()


def unpack_24(values: torch.Tensor, meta: torch.Tensor) -> torch.Tensor:
    """Dense ``[N, K]`` weight of packed 2:4 storage."""
    n, half = values.shape
    k = 2 * half
    b = meta.reshape(n // 2, k // 64, 2, 8).permute(0, 2, 1, 3).reshape(n, k // 64, 8).to(torch.int64)
    word = torch.zeros(n, k // 64, dtype=torch.int64, device=values.device)
    for i in range(8):
        word |= b[..., i] << (8 * i)
    nib = torch.stack([(word >> (4 * i)) & 0xF for i in range(16)], -1).reshape(n, k // 4)
    pos = torch.stack([nib & 3, (nib >> 2) & 3], -1)
    dense = torch.zeros(n, k // 4, 4, dtype=values.dtype, device=values.device)
    dense.scatter_(-1, pos, values.reshape(n, k // 4, 2))
    return dense.reshape(n, k)


class Sparse24Weight(nn.Module):
    """A 2:4-sparse ``[out_features, in_features]`` weight (kept values + positions as buffers)."""

    fmt = "sp24"

    def __init__(self, values: torch.Tensor, meta: torch.Tensor) -> None:
        super().__init__()
        self.out_features, self.in_features = int(values.shape[0]), int(values.shape[1] * 2)
        self.compute_dtype = values.dtype
        self.register_buffer("values", values.contiguous())
        self.register_buffer("meta", meta.contiguous())

    @classmethod
    def from_dense(cls, w: torch.Tensor, mask: torch.Tensor | None = None) -> Sparse24Weight:
        return cls(*pack_24(w, mask))

    @property
    def shape(self) -> torch.Size:
        return torch.Size((self.out_features, self.in_features))

    @property
    def device(self) -> torch.device:
        return self.values.device

    @property
    def dtype(self) -> torch.dtype:
        return self.compute_dtype

    def nbytes(self) -> int:
        return self.values.numel() * self.values.element_size() + self.meta.numel()

    def dequantize(self, dtype: torch.dtype | None = None) -> torch.Tensor:
        return unpack_24(self.values, self.meta).to(dtype or self.compute_dtype)

    def linear(self, x: torch.Tensor, splits: int = 0) -> torch.Tensor:
        shape = x.shape
        if x.is_cuda and self.values.dtype == torch.bfloat16:
            from ._ext import require

            y = require().linear_sp24(x.reshape(-1, shape[-1]).to(torch.bfloat16), self.values, self.meta,
                                      int(splits))
            return y.reshape(*shape[:-1], self.out_features).to(x.dtype)
        return (x.float() @ self.dequantize(torch.float32).t()).to(x.dtype)
