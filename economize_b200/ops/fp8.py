"""Block-scaled fp8 weights (128 x 128 weight blocks, 1 x 128 activation blocks) and their PyTorch reference.

:class:`FP8BlockWeight` replaces a ``[N, K]`` weight: e4m3 codes with one fp32 scale per 128 x 128 block.
``linear`` quantises the activations per token and 128-wide K block (``scale = max|x| / 448``) and runs the
tcgen05 ``kind::f8f6f4`` GEMM of ``csrc/gemm_fp8.cu``; the CPU reference performs the same quantisation and an fp32
product of the dequantised operands.
"""

from __future__ import annotations

import torch
from torch import nn

from ..errors import ConfigError

__all__ = ["FP8BlockWeight", "quantize_activations", "quantize_weight_blocks"]

E4M3_MAX = 448.0
BLOCK = 128


def quantize_weight_blocks(w: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """e4m3 codes ``[N, K]`` (uint8) and fp32 scales ``[N / 128, K / 128]`` of ``w``."""
    n, k = w.shape
    if n % BLOCK or k % BLOCK:
        raise ConfigError(f"block-scaled fp8 needs both dimensions divisible by {BLOCK}, got {tuple(w.shape)}")
    blocks = w.float().reshape(n // BLOCK, BLOCK, k // BLOCK, BLOCK)
    amax = blocks.abs().amax(dim=(1, 3))
    scale = torch.where(amax > 0, amax / E4M3_MAX, torch.ones_like(amax))
    codes = (blocks / scale[:, None, :, None]).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)
    return codes.reshape(n, k).view(torch.uint8), scale.contiguous()


def quantize_activations(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """The kernel's activation quantisation in PyTorch: e4m3 values (as fp32) ``[M, K]`` and scales ``[M, K/128]``."""
    m, k = x.shape
    xb = x.float().reshape(m, k // BLOCK, BLOCK)
    amax = xb.abs().amax(-1)
    scale = torch.where(amax > 0, amax / E4M3_MAX, torch.ones_like(amax))
    q = (xb / scale[..., None]).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn).float()
    return q.reshape(m, k), scale


class FP8BlockWeight(nn.Module):
    """A ``[out_features, in_features]`` weight stored as block-scaled e4m3 (codes and scales as buffers)."""

    fmt = "fp8_block"

    def __init__(self, codes: torch.Tensor, scales: torch.Tensor, dtype: torch.dtype = torch.bfloat16) -> None:
        super().__init__()
        self.out_features, self.in_features = int(codes.shape[0]), int(codes.shape[1])
        self.compute_dtype = dtype
        self.register_buffer("codes", codes.contiguous())
        self.register_buffer("scales", scales.float().contiguous())

    @classmethod
    def from_weight(cls, w: torch.Tensor) -> FP8BlockWeight:
        codes, scales = quantize_weight_blocks(w)
        return cls(codes, scales, w.dtype)

    @property
    def shape(self) -> torch.Size:
        return torch.Size((self.out_features, self.in_features))

    @property
    def device(self) -> torch.device:
        return self.codes.device

    @property
    def dtype(self) -> torch.dtype:
        return self.compute_dtype

    def nbytes(self) -> int:
        return self.codes.numel() + self.scales.numel() * 4

    def dequantize(self, dtype: torch.dtype | None = None) -> torch.Tensor:
        n, k = self.shape
        w = self.codes.view(torch.float8_e4m3fn).float().reshape(n // BLOCK, BLOCK, k // BLOCK, BLOCK)
        w = w * self.scales[:, None, :, None]
        return w.reshape(n, k).to(dtype or self.compute_dtype)

    def linear(self, x: torch.Tensor, splits: int = 0) -> torch.Tensor:
        shape = x.shape
        x2 = x.reshape(-1, shape[-1])
        if x.is_cuda:
            from ._ext import require

            y = require().linear_fp8(x2.to(torch.bfloat16).contiguous(), self.codes, self.scales, int(splits))
        else:
            q, s = quantize_activations(x2)
            xd = (q.reshape(q.shape[0], -1, BLOCK) * s[..., None]).reshape_as(q)
            y = xd @ self.dequantize(torch.float32).t()
        return y.reshape(*shape[:-1], self.out_features).to(x.dtype)

    def rows(self, start: int, stop: int) -> FP8BlockWeight:
        if start % BLOCK or stop % BLOCK:
            raise ConfigError("fp8 block shards must align to 128 rows")
        return FP8BlockWeight(self.codes[start:stop], self.scales[start // BLOCK: stop // BLOCK], self.compute_dtype)

    def cols(self, start: int, stop: int) -> FP8BlockWeight:
        if start % BLOCK or stop % BLOCK:
            raise ConfigError("fp8 block shards must align to 128 columns")
        return FP8BlockWeight(self.codes[:, start:stop], self.scales[:, start // BLOCK: stop // BLOCK],
                              self.compute_dtype)
