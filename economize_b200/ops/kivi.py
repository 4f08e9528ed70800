"""KIVI-coded KV chunks (2- or 4-bit) and their PyTorch reference.

Committed 128-key chunks of a layer's cache that lie at least ``residual`` slots behind the committed length are
coded as in KIVI (Liu et al., 2024): keys per channel (scale and zero over the chunk's 128 tokens), values per token
(scale and zero per group of 32 channels), codes ``round((x - zero) / scale)`` packed little-endian along channels.
A chunk's bytes (``chunk_bytes``): key codes ``[128 tokens][128 * bits / 8]``, key scales ``bf16[128]``, key zeros
``bf16[128]``, value codes, value scales ``bf16[128][4]``, value zeros ``bf16[128][4]``. The attention kernel
dequantises ``bf16(code * scale + zero)`` (product and sum rounded separately in fp32) into its shared-memory tiles,
so a decode pass reads 16 % (2-bit) or 29 % (4-bit) of the bf16 bytes for those chunks.
"""

from __future__ import annotations

import torch

__all__ = ["chunk_bytes", "dequant_chunks", "pack_chunks"]

CHUNK = 128
GROUP = 32


def chunk_bytes(bits: int, dim: int = 128) -> int:
    """Bytes of one coded chunk (``dim`` channels; the CUDA kernels take 128)."""
    return 2 * CHUNK * dim * bits // 8 + 2 * dim * 2 + 2 * CHUNK * (dim // GROUP) * 2


def _bf16_bytes(t: torch.Tensor) -> torch.Tensor:
    return t.to(torch.bfloat16).contiguous().view(torch.uint8).reshape(*t.shape[:-1], -1)


def _pack(codes: torch.Tensor, bits: int) -> torch.Tensor:
    per = 8 // bits
    c = codes.to(torch.int32).reshape(*codes.shape[:-1], codes.shape[-1] // per, per)
    shifts = torch.arange(per, device=codes.device, dtype=torch.int32) * bits
    return (c << shifts).sum(-1).to(torch.uint8)


def _unpack(data: torch.Tensor, bits: int) -> torch.Tensor:
    per = 8 // bits
    shifts = torch.arange(per, device=data.device, dtype=torch.int32) * bits
    return ((data.to(torch.int32)[..., None] >> shifts) & ((1 << bits) - 1)).reshape(*data.shape[:-1], -1)


def _grid(x: torch.Tensor, dim: int, bits: int) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    levels = (1 << bits) - 1
    lo, hi = x.amin(dim, keepdim=True), x.amax(dim, keepdim=True)
    s = ((hi - lo) / levels).to(torch.bfloat16).float()
    s = torch.where(s > 0, s, torch.ones_like(s))
    z = lo.to(torch.bfloat16).float()
    q = torch.clamp(torch.round((x - z) / s), 0, levels)
    return q, s, z


def pack_chunks(k: torch.Tensor, v: torch.Tensor, bits: int) -> torch.Tensor:
    """Code chunks ``k, v [..., 128 tokens, 128 channels]`` (bf16 values) into ``[..., chunk_bytes]`` uint8."""
    kf, vf = k.float(), v.float()
    dim = k.shape[-1]
    kq, ks, kz = _grid(kf, -2, bits)  # per channel over tokens: [..., 1, dim]
    vg = vf.reshape(*vf.shape[:-1], dim // GROUP, GROUP)
    vq, vs, vz = _grid(vg, -1, bits)  # per token and group: [..., 128, 4, 1]
    parts = [_pack(kq, bits).reshape(*k.shape[:-2], -1), _bf16_bytes(ks[..., 0, :]), _bf16_bytes(kz[..., 0, :]),
             _pack(vq.reshape(vf.shape), bits).reshape(*k.shape[:-2], -1),
             _bf16_bytes(vs[..., 0].reshape(*vs.shape[:-3], -1)), _bf16_bytes(vz[..., 0].reshape(*vz.shape[:-3], -1))]
    return torch.cat(parts, -1)


def dequant_chunks(data: torch.Tensor, bits: int, dim: int = 128) -> tuple[torch.Tensor, torch.Tensor]:
    """Keys and values ``[..., 128, dim]`` (fp32 holding bf16 values) of coded chunks ``[..., chunk_bytes]``."""
    cb = CHUNK * dim * bits // 8
    ng = dim // GROUP
    lead = data.shape[:-1]
    o = 0

    def take(n):
        nonlocal o
        out = data[..., o:o + n]
        o += n
        return out

    kc = _unpack(take(cb), bits).reshape(*lead, CHUNK, dim).float()
    ks = take(2 * dim).contiguous().view(torch.bfloat16).float()
    kz = take(2 * dim).contiguous().view(torch.bfloat16).float()
    vc = _unpack(take(cb), bits).reshape(*lead, CHUNK, dim).float()
    vs = take(CHUNK * ng * 2).contiguous().view(torch.bfloat16).float().reshape(*lead, CHUNK, ng)
    vz = take(CHUNK * ng * 2).contiguous().view(torch.bfloat16).float().reshape(*lead, CHUNK, ng)
    keys = (kc * ks[..., None, :] + kz[..., None, :]).to(torch.bfloat16).float()
    vs_full = vs.repeat_interleave(GROUP, -1)
    vz_full = vz.repeat_interleave(GROUP, -1)
    values = (vc * vs_full + vz_full).to(torch.bfloat16).float()
    return keys, values
