"""Packed weight formats of the weight-only quantized GEMM (``csrc/gemm_wq.cu``) and their PyTorch reference.

A :class:`QWeight` replaces a ``[N, K]`` bf16 weight of the engine model: ``ops.linear(x, qweight)`` runs the
W4A16 / W8A16 tcgen05 kernel on CUDA tensors and ``x @ dequantize().T`` on the CPU. The quantization *methods*
(round to nearest, GPTQ, AWQ) live in :mod:`economize_b200.techniques.quant`; this module only stores and unpacks.

Formats (economize's ``QUANT_FORMATS`` names, ``src/economize/techniques/quant/grid.py:237-238``):

* ``int4``: unsigned codes 0..15 with one zero point ``z`` and scale ``s`` per (output row, group):
  ``w = (q - z) * s``. Packed two per byte with the nibble order ``k0 k2 k4 k6 k1 k3 k5 k7`` inside each 32-bit word
  so the kernel extracts the bf16 pair ``(k_2i, k_2i+1)`` with one shift and one mask; zero points are stored as the
  bf16 value ``128 + z``.
* ``int8``: symmetric codes -128..127, ``w = q * s``; stored as ``q + 128`` with the byte order ``k0 k2 k1 k3`` per
  word (the kernel splits each byte into nibbles to build exact bf16 values).
* ``fp8``: e4m3 codes, ``w = q * s``.
* ``int3``: codes 0..7 with zero points, stored in the ``int4`` layout (the kernel's int4 path dequantizes them).
* ``int2``: codes 0..3 with zero points, 16 per 32-bit word (bits ``2m`` of the low half hold ``k_2m``, of the high
  half ``k_2m+1``), so the kernel extracts a bf16 pair with one shift and one mask as for int4.
* ``mxfp4`` / ``nvfp4``: FP4 E2M1 codes (bits 0-2 index :data:`E2M1_VALUES`, bit 3 the sign), two per byte with
  ``k = 2b`` in the low nibble of byte ``b``; one scale per 32 (MX) or 16 (NV) input columns. The stored bf16 scale
  is the effective one: MX's E8M0 power of two, or NV's e4m3 group scale divided by the tensor's global scale
  (chosen as a power of two here, so the quotient stays exact in bf16).

Scales (and zeros) are ``[K / group, N]`` bf16: one 256-byte row per 128 output features and group, which the kernel
reads with one TMA box. The dequantized weight is ``bf16((q - z) * s)`` in every path (the kernel's bf16x2
arithmetic rounds once, like the reference's fp32 product rounded to bf16).
"""

from __future__ import annotations

import torch
from torch import nn

from ..errors import ConfigError

__all__ = ["CODES_PER_BYTE", "E2M1_VALUES", "FORMAT_CODES", "FP4_GROUP", "ZERO_POINT_FORMATS", "QWeight", "dequantize",
           "e2m1_round", "install", "pack", "unpack"]

#: kernel format codes (``WqFormat`` in ``csrc/launchers.h``); int3 codes (0..7) are stored in the int4 layout
FORMAT_CODES = {"int4": 0, "int8": 1, "fp8": 2, "int3": 0, "int2": 4, "mxfp4": 5, "nvfp4": 6}
#: formats with a zero point per (row, group) (the bf16 value ``128 + z``)
ZERO_POINT_FORMATS = ("int2", "int3", "int4")
#: codes per stored byte (1 for the 8-bit formats)
CODES_PER_BYTE = {"int4": 2, "int3": 2, "int2": 4, "mxfp4": 2, "nvfp4": 2}
#: the fixed scale group of the FP4 formats
FP4_GROUP = {"mxfp4": 32, "nvfp4": 16}
#: the non-negative FP4 E2M1 values, indexed by the low three bits of a code
E2M1_VALUES = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)


def e2m1_round(x: torch.Tensor) -> torch.Tensor:
    """``x`` rounded to the nearest E2M1 value (magnitudes above 6 clip to 6; a tie goes to the value with the even
    code, IEEE round-half-to-even on the 3-bit magnitude index)."""
    table = torch.tensor(E2M1_VALUES, dtype=torch.float32, device=x.device)
    a = x.float().abs().clamp(max=6.0)
    hi = torch.bucketize(a, table)  # table[hi - 1] < a <= table[hi]
    lo = (hi - 1).clamp(min=0)
    d_lo, d_hi = a - table[lo], table[hi] - a
    pick = torch.where((d_hi < d_lo) | ((d_hi == d_lo) & (hi % 2 == 0)), hi, lo)
    return torch.copysign(table[pick], x.float()) * (pick > 0)


def _fp4_codes(values: torch.Tensor) -> torch.Tensor:
    """E2M1 values -> 4-bit codes (int64); zero is code 0 whatever its sign."""
    twice = (values.float().abs() * 2).round().to(torch.int64)  # 0, 1, 2, 3, 4, 6, 8, 12
    index = torch.tensor([0, 1, 2, 3, 4, -1, 5, -1, 6, -1, -1, -1, 7], device=values.device)[twice.clamp(max=12)]
    if (index < 0).any() or (values.float().abs() > 6).any():
        raise ConfigError("fp4 packing takes E2M1 values (0, 0.5, 1, 1.5, 2, 3, 4, 6 and their negatives)")
    return index | ((values < 0) & (index > 0)).to(torch.int64) << 3
_INT4_ORDER = (0, 2, 4, 6, 1, 3, 5, 7)
_INT8_ORDER = (0, 2, 1, 3)


def _words_to_bytes(words: torch.Tensor) -> torch.Tensor:
    """int64 words holding 32-bit values ``[N, W]`` -> little-endian bytes ``[N, 4 W]`` uint8."""
    shifts = torch.tensor([0, 8, 16, 24], device=words.device, dtype=torch.int64)
    return ((words[..., None] >> shifts) & 0xFF).to(torch.uint8).reshape(words.shape[0], -1)


def _bytes_to_words(data: torch.Tensor) -> torch.Tensor:
    b = data.reshape(data.shape[0], -1, 4).to(torch.int64)
    return b[..., 0] | (b[..., 1] << 8) | (b[..., 2] << 16) | (b[..., 3] << 24)


def pack(codes: torch.Tensor, fmt: str) -> torch.Tensor:
    """Pack integer codes ``[N, K]`` (int4: 0..15, int8: -128..127) or e4m3 values (fp8) into the kernel layout."""
    n, k = codes.shape
    if fmt == "int2":  # 16 codes per word: bits 2m of the low half = k_2m, of the high half = k_2m+1
        c = codes.to(torch.int64).reshape(n, k // 16, 8, 2)
        words = torch.zeros(n, k // 16, dtype=torch.int64, device=codes.device)
        for m in range(8):
            words |= (c[..., m, 0] & 3) << (2 * m)
            words |= (c[..., m, 1] & 3) << (16 + 2 * m)
        return _words_to_bytes(words)
    if fmt in ("int4", "int3"):
        c = codes.to(torch.int64).reshape(n, k // 8, 8)[..., list(_INT4_ORDER)]
        words = torch.zeros(n, k // 8, dtype=torch.int64, device=codes.device)
        for i in range(8):
            words |= (c[..., i] & 0xF) << (4 * i)
        return _words_to_bytes(words)
    if fmt == "int8":
        u = (codes.to(torch.int64) + 128).reshape(n, k // 4, 4)[..., list(_INT8_ORDER)]
        return u.to(torch.uint8).reshape(n, k)
    if fmt == "fp8":
        return codes.to(torch.float8_e4m3fn).contiguous().view(torch.uint8)
    if fmt in FP4_GROUP:  # E2M1 values; k = 2b in the low nibble of byte b
        c = _fp4_codes(codes).reshape(n, k // 2, 2)
        return (c[..., 0] | (c[..., 1] << 4)).to(torch.uint8)
    raise ConfigError(f"unknown weight format {fmt!r}")


def unpack(data: torch.Tensor, fmt: str) -> torch.Tensor:
    """Inverse of :func:`pack`: int64 codes (int2, int4, int8) or fp32 values (fp8, fp4) ``[N, K]``."""
    n = data.shape[0]
    if fmt == "int2":
        words = _bytes_to_words(data)
        out = torch.empty(n, words.shape[1], 8, 2, dtype=torch.int64, device=data.device)
        for m in range(8):
            out[..., m, 0] = (words >> (2 * m)) & 3
            out[..., m, 1] = (words >> (16 + 2 * m)) & 3
        return out.reshape(n, -1)
    if fmt in ("int4", "int3"):
        words = _bytes_to_words(data)
        nib = torch.stack([(words >> (4 * i)) & 0xF for i in range(8)], -1)  # in packed order
        out = torch.empty_like(nib)
        out[..., list(_INT4_ORDER)] = nib
        return out.reshape(n, -1)
    if fmt == "int8":
        u = data.to(torch.int64).reshape(n, -1, 4)
        out = torch.empty_like(u)
        out[..., list(_INT8_ORDER)] = u
        return out.reshape(n, -1) - 128
    if fmt == "fp8":
        return data.contiguous().view(torch.float8_e4m3fn).float()
    if fmt in FP4_GROUP:
        b = data.to(torch.int64)
        codes = torch.stack([b & 0xF, b >> 4], -1).reshape(n, -1)
        table = torch.tensor(E2M1_VALUES, dtype=torch.float32, device=data.device)
        return torch.where(codes >= 8, -table[codes & 7], table[codes & 7])
    raise ConfigError(f"unknown weight format {fmt!r}")


def dequantize(qweight: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor | None, fmt: str, group: int,
               dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    """``bf16((q - z) * s)`` as ``[N, K]`` in ``dtype`` (the value every kernel path multiplies with)."""
    q = unpack(qweight, fmt).float()
    s = scales.float().t().repeat_interleave(group, dim=1)  # [N, K]
    if zeros is not None:
        q = q - (zeros.float().t().repeat_interleave(group, dim=1) - 128.0)
    return (q * s).to(torch.bfloat16).to(dtype)


class QWeight(nn.Module):
    """A quantized ``[out_features, in_features]`` weight (packed codes + scales (+ zeros) as buffers).

    Args:
        qweight: Packed codes (:func:`pack`).
        scales: ``[K / group, N]`` bf16.
        zeros: ``[K / group, N]`` bf16 holding ``128 + z`` (int4), else ``None``.
        fmt: ``"int2"``, ``"int3"``, ``"int4"``, ``"int8"``, ``"fp8"``, ``"mxfp4"`` or ``"nvfp4"``.
        group: Input columns per scale (``in_features`` for one scale per output row).
        dtype: The activation dtype the layer computes in.
    """

    def __init__(self, qweight: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor | None, fmt: str, group: int,
                 dtype: torch.dtype = torch.bfloat16) -> None:
        super().__init__()
        if fmt not in FORMAT_CODES:
            raise ConfigError(f"unknown weight format {fmt!r}")
        self.fmt = fmt
        self.group = int(group)
        self.out_features = int(qweight.shape[0])
        self.in_features = int(qweight.shape[1] * CODES_PER_BYTE.get(fmt, 1))
        self.compute_dtype = dtype
        self.register_buffer("qweight", qweight.contiguous())
        self.register_buffer("scales", scales.to(torch.bfloat16).contiguous())
        self.register_buffer("zeros", None if zeros is None else zeros.to(torch.bfloat16).contiguous())

    @property
    def shape(self) -> torch.Size:
        return torch.Size((self.out_features, self.in_features))

    @property
    def device(self) -> torch.device:
        return self.qweight.device

    @property
    def dtype(self) -> torch.dtype:
        return self.compute_dtype

    @property
    def bits(self) -> int:
        return {"int2": 2, "int3": 3, "int4": 4, "mxfp4": 4, "nvfp4": 4}.get(self.fmt, 8)

    def dequantize(self, dtype: torch.dtype | None = None) -> torch.Tensor:
        return dequantize(self.qweight, self.scales, self.zeros, self.fmt, self.group, dtype or self.compute_dtype)

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in (self.qweight, self.scales, self.zeros) if t is not None)

    def linear(self, x: torch.Tensor, splits: int = 0) -> torch.Tensor:
        """``x @ dequantize().T`` (the tcgen05 kernel for CUDA bf16 inputs)."""
        if x.is_cuda:
            from ._ext import require

            shape = x.shape
            y = require().linear_wq(x.reshape(-1, shape[-1]).to(torch.bfloat16), self.qweight, self.scales,
                                    self.zeros, FORMAT_CODES[self.fmt], self.group, int(splits))
            return y.reshape(*shape[:-1], self.out_features).to(x.dtype)
        w = self.dequantize(torch.float32)
        return (x.float() @ w.t()).to(x.dtype)

    def rows(self, start: int, stop: int) -> QWeight:
        """The output rows ``[start, stop)`` (a column-parallel shard)."""
        z = None if self.zeros is None else self.zeros[:, start:stop]
        return QWeight(self.qweight[start:stop], self.scales[:, start:stop], z, self.fmt, self.group,
                       self.compute_dtype)

    def cols(self, start: int, stop: int) -> QWeight:
        """The input columns ``[start, stop)`` (a row-parallel shard); both ends must sit on group boundaries."""
        if start % self.group or stop % self.group:
            raise ConfigError(f"column shard [{start}, {stop}) cuts a quantization group of {self.group}")
        per = CODES_PER_BYTE.get(self.fmt, 1)
        z = None if self.zeros is None else self.zeros[start // self.group: stop // self.group]
        return QWeight(self.qweight[:, start // per: stop // per], self.scales[start // self.group: stop // self.group],
                       z, self.fmt, self.group, self.compute_dtype)

    def extra_repr(self) -> str:
        return f"{self.out_features}x{self.in_features}, fmt={self.fmt}, group={self.group}"


def install(owner: nn.Module, name: str, value) -> None:
    """Put ``value`` (a :class:`QWeight` or a parameter) at ``owner.name``, replacing a parameter of that name."""
    if name in owner._parameters and not isinstance(value, nn.Parameter):
        del owner._parameters[name]
    setattr(owner, name, value)
