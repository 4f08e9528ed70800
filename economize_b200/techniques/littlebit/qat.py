"""Quantization-aware training of LittleBit factors (Lee et al., 2025, "LittleBit: Ultra Low-Bit Quantization via
Latent Factorization", Section 3.4; economize ``techniques/littlebit/qat.py``).

The trainable form of a map keeps real-valued latent sign factors and real scales; its forward uses the signs of
the latents, and the sign's gradient is the SmoothSign surrogate: forward ``sign(x)``, backward the derivative of
``tanh(k x)`` (``k = 100`` in the paper). This build trains map by map with an activation-aware objective: the
relative output error ``||X W^T - X W_q^T||^2 / ||X W^T||^2`` on calibration activations ``X`` of that map
(collected from the dense model before it is replaced), starting from the Dual-SVID factors. It needs one map's
latents and optimizer state at a time instead of the whole model's (the paper's end-to-end distillation is the
larger-budget variant).
"""

from __future__ import annotations

import torch
from torch import nn

__all__ = ["LatentLittleBit", "SmoothSign", "smooth_sign", "train_map"]


class SmoothSign(torch.autograd.Function):
    """``sign`` (0 counts as positive, as the packed storage does) with the gradient of ``tanh(k x)``."""

    @staticmethod
    def forward(ctx, x: torch.Tensor, k: float) -> torch.Tensor:
        ctx.save_for_backward(x)
        ctx.k = k
        return torch.where(x < 0, -torch.ones_like(x), torch.ones_like(x))

    @staticmethod
    def backward(ctx, grad: torch.Tensor):
        (x,) = ctx.saved_tensors
        t = torch.tanh(ctx.k * x)
        return grad * ctx.k * (1.0 - t * t), None


def smooth_sign(x: torch.Tensor, k: float = 100.0) -> torch.Tensor:
    return SmoothSign.apply(x, k)


class LatentLittleBit(nn.Module):
    """Latent factors of the paths of one map: ``u [P, out, r]``, ``v [P, r, in]`` (signs used), ``h [P, out]``,
    ``g [P, in]``, ``l [P, r]`` (used as they are); all float32."""

    def __init__(self, u, v, h, g, l, k: float = 100.0) -> None:
        super().__init__()
        self.u, self.v = nn.Parameter(u.float().clone()), nn.Parameter(v.float().clone())
        self.h, self.g, self.l = (nn.Parameter(t.float().clone()) for t in (h, g, l))
        self.k = k

    def weight(self) -> torch.Tensor:
        """The dense ``[out, in]`` weight the current signs and scales represent."""
        su, sv = smooth_sign(self.u, self.k), smooth_sign(self.v, self.k)
        left = self.h[:, :, None] * su * self.l[:, None, :]  # [P, out, r]
        right = sv * self.g[:, None, :]  # [P, r, in]
        return torch.einsum("por,pri->oi", left, right)

    def factors(self) -> tuple[torch.Tensor, ...]:
        return tuple(t.detach() for t in (self.u, self.v, self.h, self.g, self.l))


def train_map(weight: torch.Tensor, x: torch.Tensor, factors, steps: int, lr: float = 1e-3,
              k: float = 100.0) -> tuple[tuple[torch.Tensor, ...], float, float]:
    """Train the factors of ``weight [out, in]`` on activations ``x [N, in]``; returns the factors and the relative
    output error before and after."""
    latent = LatentLittleBit(*factors, k=k).to(weight.device)
    w = weight.detach().float()
    xs = x.detach().float().to(weight.device)
    ref = xs @ w.t()
    denom = ref.pow(2).sum().clamp_min(1e-12)

    def error() -> torch.Tensor:
        return (xs @ latent.weight().t() - ref).pow(2).sum() / denom

    opt = torch.optim.Adam(latent.parameters(), lr=lr)
    with torch.no_grad():
        before = float(error())
    best, best_state = before, latent.factors()
    for _ in range(steps):
        loss = error()
        opt.zero_grad()
        loss.backward()
        opt.step()
        with torch.no_grad():
            now = float(error())
        if now < best:
            best, best_state = now, latent.factors()
    return best_state, before, best
