"""LittleBit weights: ``W = sum_p diag(h_p) sign(U_p) diag(l_p) sign(V_p) diag(g_p)`` with bit-packed signs
(economize ``techniques/littlebit/{module,pack,kernel}.py``).

:class:`LittleBitWeight` stores, per path, the signs of ``U [out, r]`` and ``V [r, in]`` packed 32 per int32 along
the reduced dimension (bit set = -1) and the fp32 scales. Decoding calls of at most 16 rows run two sign products per
path on the CUDA cores (``sign_matvec`` of ``csrc/binary.cu``: the factors are a fraction of a bit per weight, so
the call is bound by launch latency, not bytes); other calls multiply by the dense reconstruction.
"""

from __future__ import annotations

import torch
from torch import nn

__all__ = ["LittleBitWeight", "pack_signs", "unpack_signs"]


def pack_signs(x: torch.Tensor) -> torch.Tensor:
    """Signs of ``x [R, C]`` packed along ``C``: int32 ``[R, ceil(C / 32)]``, bit ``j`` of word ``w`` set when
    ``x[:, 32 w + j] < 0``."""
    r, c = x.shape
    words = (c + 31) // 32
    neg = torch.zeros(r, words * 32, dtype=torch.int64, device=x.device)
    neg[:, :c] = (x < 0).long()
    weights = (torch.ones(32, dtype=torch.int64, device=x.device) << torch.arange(32, device=x.device))
    packed = (neg.reshape(r, words, 32) * weights).sum(-1)
    return torch.where(packed >= 2 ** 31, packed - 2 ** 32, packed).to(torch.int32)


def unpack_signs(bits: torch.Tensor, cols: int) -> torch.Tensor:
    """``+1 / -1`` fp32 ``[R, cols]`` from :func:`pack_signs`."""
    b = bits.long() & 0xFFFFFFFF
    j = torch.arange(32, device=bits.device)
    neg = (b[..., None] >> j) & 1
    return (1.0 - 2.0 * neg.reshape(bits.shape[0], -1)[:, :cols].float())


class LittleBitWeight(nn.Module):
    """Paths of binary factors of an ``[out, in]`` weight (buffers ``u_bits [P, out, ceil(r / 32)]``, ``v_bits
    [P, r, ceil(in / 32)]``, ``h [P, out]``, ``g [P, in]``, ``l [P, r]``)."""

    def __init__(self, u: torch.Tensor, v: torch.Tensor, h: torch.Tensor, g: torch.Tensor, l: torch.Tensor,
                 dtype: torch.dtype) -> None:
        super().__init__()
        self.out_features, self.in_features, self.rank = u.shape[1], v.shape[2], u.shape[2]
        self.compute_dtype = dtype
        self.register_buffer("u_bits", torch.stack([pack_signs(x) for x in u]))
        self.register_buffer("v_bits", torch.stack([pack_signs(x) for x in v]))
        self.register_buffer("h", h.float().contiguous())
        self.register_buffer("g", g.float().contiguous())
        self.register_buffer("l", l.float().contiguous())

    @property
    def shape(self) -> torch.Size:
        return torch.Size((self.out_features, self.in_features))

    @property
    def dtype(self) -> torch.dtype:
        return self.compute_dtype

    @property
    def device(self) -> torch.device:
        return self.h.device

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.u_bits, self.v_bits, self.h, self.g, self.l))

    def bits_per_weight(self) -> float:
        p = self.h.shape[0]
        signs = p * self.rank * (self.out_features + self.in_features)
        scales = 16 * p * (self.out_features + self.in_features + self.rank)
        return (signs + scales) / (self.out_features * self.in_features)

    def dequantize(self, dtype: torch.dtype | None = None) -> torch.Tensor:
        w = 0
        for p in range(self.h.shape[0]):
            su = unpack_signs(self.u_bits[p], self.rank)
            sv = unpack_signs(self.v_bits[p], self.in_features)
            w = w + (self.h[p][:, None] * su * self.l[p][None]) @ (sv * self.g[p][None])
        return w.to(dtype or self.compute_dtype)

    def linear(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        x2 = x.reshape(-1, shape[-1]).float()
        if x.is_cuda and x2.shape[0] <= 16:
            from ._ext import require

            C = require()
            y = 0
            for p in range(self.h.shape[0]):
                t = C.sign_matvec(self.v_bits[p], (x2 * self.g[p][None]).contiguous())  # [M, r]
                y = y + C.sign_matvec(self.u_bits[p], (t * self.l[p][None]).contiguous()) * self.h[p][None]
        else:
            y = x2 @ self.dequantize(torch.float32).t()
        return y.to(x.dtype).reshape(*shape[:-1], self.out_features)
