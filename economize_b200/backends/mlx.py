"""Export a model to an ``mlx_lm`` folder (Apple silicon; economize ``backends/mlx``): ``config.json`` plus
``model.safetensors`` under Hugging Face parameter names. Written on any platform; ``mlx_lm`` runs it.

Projections this build holds as integer codes (``QWeight`` int2/int3/int4/int8) are stored as MLX's affine
quantized linear maps: ``p.weight`` ``uint32 [out, in * bits / 32]`` (each row's codes one little-endian bit stream,
lowest bits first), ``p.scales`` and ``p.biases`` ``[out, in / group]`` with ``w = scales * code + biases``. Zero-point
grids (``w = s (q - z)``) keep their codes with ``biases = -s z``; symmetric int8 (``w = s q``, ``q`` in -128..127)
stores ``q + 128`` with ``biases = -128 s``. The engine's fused projections are split back into ``q/k/v_proj`` and
``gate/up_proj``. ``config["quantization"]`` names the group size and bits (one setting per model).
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import torch

from ..errors import ConfigError
from ..ops.quant import QWeight, unpack

__all__ = ["MLX_BITS", "mlx_affine", "pack_bits", "to_mlx"]

MLX_BITS = {"int2": 2, "int3": 3, "int4": 4, "int8": 8}
MLX_GROUPS = (32, 64, 128)


def pack_bits(codes: np.ndarray, bits: int) -> np.ndarray:
    """Unsigned codes ``[out, in]`` (below ``2 ** bits``) as ``uint32 [out, in * bits / 32]``: every row one bit
    stream, code ``j`` at bits ``j * bits ..``, little-endian words."""
    rows, count = codes.shape
    if (count * bits) % 32:
        raise ConfigError(f"{count} codes of {bits} bits do not fill whole 32-bit words")
    weights = (1 << np.arange(bits, dtype=np.uint64))
    bitplane = ((codes.astype(np.uint64)[..., None] & weights) > 0).astype(np.uint8)  # [rows, count, bits]
    stream = bitplane.reshape(rows, count * bits)
    packed = np.packbits(stream, axis=-1, bitorder="little")
    return np.ascontiguousarray(packed).view("<u4").astype(np.uint32)


def mlx_affine(qw: QWeight) -> tuple[np.ndarray, torch.Tensor, torch.Tensor]:
    """``(codes [N, K] unsigned, scales [N, K / g], biases [N, K / g])`` of a :class:`QWeight` in MLX's form."""
    if qw.fmt not in MLX_BITS:
        raise ConfigError(f"{qw.fmt} codes have no MLX affine form")
    if qw.group not in MLX_GROUPS:
        raise ConfigError(f"group size {qw.group} is not one of MLX's {MLX_GROUPS}")
    codes = unpack(qw.qweight.cpu(), qw.fmt)  # int64 [N, K]
    scales = qw.scales.float().cpu().t()  # [N, K / g]
    if qw.fmt == "int8":
        return (codes + 128).numpy(), scales, -128.0 * scales
    zeros = qw.zeros.float().cpu().t() - 128.0
    return codes.numpy(), scales, -scales * zeros


_SPLITS = {"wqkv": ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj"), "wo": ("self_attn.o_proj",),
           "w_gate_up": ("mlp.gate_proj", "mlp.up_proj"), "w_down": ("mlp.down_proj",)}


def to_mlx(model, folder: str | Path, dtype: torch.dtype = torch.bfloat16) -> Path:
    """Write ``model`` (an engine :class:`~economize_b200.models.CausalLM` or an EfficientModel) as an ``mlx_lm``
    folder; returns the folder."""
    from safetensors.torch import save_file

    target = getattr(model, "model", model)
    from .exporters import refuse_online_rotation

    refuse_online_rotation(target, "mlx_lm")
    c = target.config
    folder = Path(folder)
    folder.mkdir(parents=True, exist_ok=True)
    state = {k: v.to(dtype) if v.is_floating_point() else v for k, v in target.hf_state_dict().items()}
    quant: dict[str, int] = {}
    for i, layer in enumerate(target.layers):
        for name, parts in _SPLITS.items():
            qw = getattr(layer, name, None)
            if not isinstance(qw, QWeight):
                continue
            codes, scales, biases = mlx_affine(qw)
            sizes = [c.q_size, c.kv_size, c.kv_size] if name == "wqkv" else [qw.out_features // len(parts)] * len(parts)
            start = 0
            for part, n in zip(parts, sizes):
                key = f"model.layers.{i}.{part}"
                state.pop(key + ".weight", None)
                words = pack_bits(codes[start:start + n], MLX_BITS[qw.fmt])
                state[key + ".weight"] = torch.from_numpy(words.view(np.int32)).view(torch.uint32)
                state[key + ".scales"] = scales[start:start + n].to(dtype).contiguous()
                state[key + ".biases"] = biases[start:start + n].to(dtype).contiguous()
                start += n
            quant[f"{qw.group}:{MLX_BITS[qw.fmt]}"] = quant.get(f"{qw.group}:{MLX_BITS[qw.fmt]}", 0) + 1
    if c.tie_word_embeddings:
        state.pop("lm_head.weight", None)
    save_file({k: v.contiguous().cpu() for k, v in state.items()}, str(folder / "model.safetensors"))
    config = c.to_hf().to_dict()
    config.pop("torch_dtype", None)
    config["dtype"] = str(dtype).removeprefix("torch.")
    if len(quant) > 1:
        raise ConfigError(f"MLX folders take one quantization setting; this model mixes {sorted(quant)}")
    if quant:
        group, bits = map(int, next(iter(quant)).split(":"))
        config["quantization"] = {"group_size": group, "bits": bits}
    (folder / "config.json").write_text(json.dumps(config, indent=2, default=str))
    return folder
