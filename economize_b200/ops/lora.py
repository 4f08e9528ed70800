"""Low-rank adapters on the engine's weights (economize ``modules/lora.py``).

:class:`LoRAWeight` wraps a ``[out, in]`` weight (a tensor, or a weight object with ``linear``) and adds the
trainable update ``(x A^T) B^T * alpha / rank`` (``A`` small random, ``B`` zero, so the wrapped map is unchanged until
trained). ``ops.linear`` dispatches to :meth:`LoRAWeight.linear`; the base product runs on the engine's kernels and
the update in PyTorch (it is ``rank`` wide).
"""

from __future__ import annotations

import math

import torch
from torch import nn

__all__ = ["LoRAWeight"]


class LoRAWeight(nn.Module):
    def __init__(self, base, rank: int, alpha: float, seed: int = 0) -> None:
        super().__init__()
        self._base = [base]  # not a submodule: the wrapped weight belongs to its owner
        out_f, in_f = base.shape
        gen = torch.Generator().manual_seed(seed)
        self.a = nn.Parameter((torch.randn(rank, in_f, generator=gen) / math.sqrt(in_f)).to(base.device))
        self.b = nn.Parameter(torch.zeros(out_f, rank, device=base.device))
        self.scale = alpha / rank

    @property
    def base(self):
        return self._base[0]

    @property
    def shape(self) -> torch.Size:
        return self.base.shape

    @property
    def dtype(self) -> torch.dtype:
        return self.base.dtype

    @property
    def device(self) -> torch.device:
        return self.base.device

    def delta(self, x: torch.Tensor) -> torch.Tensor:
        return (x.float() @ self.a.float().t()) @ self.b.float().t() * self.scale

    def linear(self, x: torch.Tensor) -> torch.Tensor:
        from . import linear

        return (linear(x, self.base).float() + self.delta(x)).to(x.dtype)

    def dequantize(self, dtype: torch.dtype | None = None) -> torch.Tensor:
        base = self.base if isinstance(self.base, torch.Tensor) else self.base.dequantize(torch.float32)
        w = base.float() + (self.b.float() @ self.a.float()) * self.scale
        return w.to(dtype or self.dtype)

    def merged(self) -> torch.Tensor:
        """The adapted weight as one tensor in the base dtype."""
        return self.dequantize(self.dtype)
