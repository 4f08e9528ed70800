"""Differentiable EAGLE-3 forward for training (plain PyTorch ops with autograd; the inference path runs on the
sm_100a kernels).

Training-time test (EAGLE-3, Li et al. 2025): step 1 runs the draft layer teacher-forced on the target's fused
features; step ``j`` feeds step ``j - 1``'s outputs back as sources. Query ``p`` of step ``j`` sees what a draft
step at that depth sees at inference: step-1 entries at positions ``<= p - j + 1`` (the committed prefix and the
root) and the entry of every earlier step ``i`` at position ``p - (j - i)`` (its own draft chain). Scores against
those chain entries are computed as per-position dot products, so memory stays ``O(S^2 + S * steps)``.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from ...ops.reference import rmsnorm

__all__ = ["unrolled_logits"]


def _rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    half = x.shape[-1] // 2
    c = torch.cat((cos, cos), -1)[None, None].to(x.dtype)
    s = torch.cat((sin, sin), -1)[None, None].to(x.dtype)
    rot = torch.cat((-x[..., half:], x[..., :half]), -1)
    return x * c + rot * s


def _shift(x: torch.Tensor, n: int) -> torch.Tensor:
    """``x[:, :, p - n]`` at position ``p`` (zeros before the start), for ``x [B, H, S, D]``."""
    if n == 0:
        return x
    return torch.cat([torch.zeros_like(x[:, :, :n]), x[:, :, :-n]], 2)


def unrolled_logits(tech, aux: dict[int, torch.Tensor], tokens: torch.Tensor, steps: int) -> list[torch.Tensor]:
    """Draft logits ``[B, S, V_d]`` of every unrolled step for sequences ``tokens [B, S]`` whose captured target
    block outputs are ``aux {layer: [B, S, H]}``. Position ``p`` of step ``j`` predicts the target's token after
    ``tokens[:, p]``; positions ``p < j`` have no root and are to be masked out of a loss."""
    layer = tech.layer
    eps = tech.eps
    batch, length = tokens.shape
    heads, kv_heads, hd = layer.heads, layer.kv_heads, layer.head_dim
    group = heads // kv_heads
    cos, sin = layer.rope()
    cos, sin = cos[:length], sin[:length]
    g = F.linear(torch.cat([aux[i] for i in tech.aux_layers], -1).to(tech.fc.dtype), tech.fc)  # [B, S, H]
    emb = tech.model.embed_tokens(tokens).to(tech.fc.dtype)
    x_e = rmsnorm(emb, tech.input_norm, eps)[0]
    zeros = torch.zeros_like(g[:, :1])
    source = torch.cat([zeros, g[:, :-1]], 1)  # step 1: position p reads the features of token p - 1
    norm_w, head_w = tech.head_weights()
    qkv_sizes = [heads * hd, kv_heads * hd, kv_heads * hd]
    positions = torch.arange(length, device=tokens.device)
    own_keys, own_values, outs = [], [], []
    k1 = v1 = None
    for j in range(1, steps + 1):
        x_h = rmsnorm(source, tech.hidden_norm, eps)[0]
        residual = x_h if tech.config.norm_before_residual else source
        qkv = F.linear(torch.cat([x_e, x_h], -1), layer.wqkv, layer.bqkv)
        q, k, v = qkv.split(qkv_sizes, -1)
        q = _rope(q.reshape(batch, length, heads, hd).transpose(1, 2), cos, sin)
        k = _rope(k.reshape(batch, length, kv_heads, hd).transpose(1, 2), cos, sin)
        v = v.reshape(batch, length, kv_heads, hd).transpose(1, 2)
        if j == 1:
            k1, v1 = k, v
        else:
            own_keys.append(k)
            own_values.append(v)
        kr = k1.repeat_interleave(group, 1)
        vr = v1.repeat_interleave(group, 1)
        scale = hd ** -0.5
        scores = torch.matmul(q, kr.transpose(-1, -2)) * scale  # [B, H, S, S]
        limit = positions[:, None] - (j - 1)  # step-1 entries visible up to p - j + 1
        scores = scores.masked_fill(positions[None, :] > limit, float("-inf"))
        extra = []
        for i, (ki, vi) in enumerate(zip(own_keys, own_values), start=2):
            ks = _shift(ki, j - i).repeat_interleave(group, 1)
            extra.append((q * ks).sum(-1, keepdim=True) * scale)
        probs = torch.softmax(torch.cat([scores, *extra], -1).float(), -1).to(q.dtype).nan_to_num(0.0)
        att = torch.matmul(probs[..., :length], vr)
        for idx, (i, vi) in enumerate(zip(range(2, j + 1), own_values)):
            vs = _shift(vi, j - i).repeat_interleave(group, 1)
            att = att + probs[..., length + idx: length + idx + 1] * vs
        h = F.linear(att.transpose(1, 2).reshape(batch, length, heads * hd), layer.wo)
        a = residual + h
        m = rmsnorm(a, layer.post_norm, eps)[0]
        gate, up = F.linear(m, layer.w_gate_up).chunk(2, -1)
        out = a + F.linear(F.silu(gate) * up, layer.w_down)
        outs.append(F.linear(rmsnorm(out, norm_w, eps)[0], head_w).float())
        source = torch.cat([zeros, out[:, :-1]], 1)  # step j + 1 at p reads step j's output at p - 1
    return outs
