"""The target's quantized weights as a compressed-tensors checkpoint (economize
``integrations/compressed_tensors.py:1-354``).

compressed-tensors is the checkpoint format of ``llm-compressor``, which vLLM, SGLang and ``transformers`` load.
:func:`export_compressed_tensors` writes a model quantized by the ``quant`` technique (RTN, GPTQ or AWQ codes in any
of its formats) as a Hugging Face folder whose ``config.json`` carries a ``quantization_config`` with
``quant_method="compressed-tensors"`` and whose ``model.safetensors`` holds, per quantized ``nn.Linear``:

* ``int2`` / ``int3`` / ``int4`` (format ``pack-quantized``): ``weight_packed`` int32 ``[N, K * bits / 32]`` with the
  signed codes ``q - 2^(bits-1)`` offset back to unsigned and packed little-end first, ``weight_scale [N, K / g]``,
  ``weight_zero_point [N, K / g]`` (signed, asymmetric grids only) and ``weight_shape``;
* ``int8`` (``int-quantized``): ``weight`` int8 and ``weight_scale``;
* ``fp8`` (``float-quantized``): ``weight`` float8 e4m3 and ``weight_scale``;
* ``nvfp4`` (``nvfp4-pack-quantized``): ``weight_packed`` uint8 ``[N, K / 2]`` (low nibble first),
  ``weight_scale`` float8 e4m3 ``[N, K / 16]`` and ``weight_global_scale`` (``w = q * scale / global``);
* ``mxfp4`` (``mxfp4-pack-quantized``): ``weight_packed`` uint8 and ``weight_scale`` uint8 E8M0 exponents
  ``[N, K / 32]``.

The fused projections of the engine are split back into ``q/k/v_proj`` and ``gate/up_proj``. Every other tensor is
written under its Hugging Face name in the model's dtype. :func:`read_compressed_tensors` reads such a folder back
into a dense Hugging Face state dict (the weights each scheme decodes to), which is how the tests check that the
codes survive the trip; the tensor names, config keys and packing are the public format's.
"""

from __future__ import annotations

import json
from pathlib import Path
from typing import Any

import torch

from ..errors import CheckpointFormatError, ConfigError
from ..ops.quant import FP4_GROUP, ZERO_POINT_FORMATS, QWeight, unpack

__all__ = ["export_compressed_tensors", "read_compressed_tensors"]

_BITS = {"int2": 2, "int3": 3, "int4": 4, "int8": 8}
_CT_FORMAT = {"int2": "pack-quantized", "int3": "pack-quantized", "int4": "pack-quantized", "int8": "int-quantized",
              "fp8": "float-quantized", "nvfp4": "nvfp4-pack-quantized", "mxfp4": "mxfp4-pack-quantized"}


def _pack_int32(q: torch.Tensor, bits: int) -> torch.Tensor:
    """Signed codes ``[N, K]`` -> int32 words ``[N, ceil(K * bits / 32)]`` (offset to unsigned, low bits first)."""
    n, k = q.shape
    per = 32 // bits
    u = (q.to(torch.int64) + (1 << (bits - 1))) & ((1 << bits) - 1)
    pad = (-k) % per
    u = torch.nn.functional.pad(u, (0, pad)).reshape(n, -1, per)
    words = torch.zeros(n, u.shape[1], dtype=torch.int64)
    for i in range(per):
        words |= u[..., i] << (bits * i)
    return torch.where(words >= 1 << 31, words - (1 << 32), words).to(torch.int32)


def _unpack_int32(words: torch.Tensor, bits: int, k: int) -> torch.Tensor:
    per = 32 // bits
    w = words.to(torch.int64) & 0xFFFFFFFF
    u = torch.stack([(w >> (bits * i)) & ((1 << bits) - 1) for i in range(per)], -1).reshape(words.shape[0], -1)
    return u[:, :k] - (1 << (bits - 1))


def _linear_entries(qw: QWeight, prefix: str) -> tuple[dict[str, torch.Tensor], dict[str, Any]]:
    """The compressed-tensors tensors of one quantized ``nn.Linear`` and its weight scheme."""
    fmt, n, k = qw.fmt, qw.out_features, qw.in_features
    scale = qw.scales.t().contiguous()  # [N, K / g]
    out: dict[str, torch.Tensor] = {}
    scheme: dict[str, Any] = {"strategy": "group" if qw.group < k else "channel", "dynamic": False,
                              "observer": "minmax"}
    if fmt in _BITS:
        bits = _BITS[fmt]
        codes = unpack(qw.qweight, "int4" if fmt == "int3" else fmt)  # int2/3/4: 0..2^b - 1 (int3 in int4 layout)
        symmetric = fmt not in ZERO_POINT_FORMATS
        if fmt in ZERO_POINT_FORMATS:
            zero = (qw.zeros.t().float() - 128.0).round().to(torch.int64)  # unsigned zero points
            half = 1 << (bits - 1)
            signed, zp = codes - half, zero - half
            symmetric = bool((zp == 0).all())
        else:
            signed, zp = codes, None
        if bits == 8:
            out[prefix + "weight"] = signed.to(torch.int8)
        else:
            out[prefix + "weight_packed"] = _pack_int32(signed, bits)
            out[prefix + "weight_shape"] = torch.tensor([n, k], dtype=torch.int64)
        if not symmetric:
            out[prefix + "weight_zero_point"] = zp.to(torch.int8)
        out[prefix + "weight_scale"] = scale
        scheme.update({"num_bits": bits, "type": "int", "symmetric": symmetric})
    elif fmt == "fp8":
        out[prefix + "weight"] = qw.qweight.view(torch.float8_e4m3fn)
        out[prefix + "weight_scale"] = scale
        scheme.update({"num_bits": 8, "type": "float", "symmetric": True})
    elif fmt == "nvfp4":
        s = scale.float()
        glob = float(2.0 ** torch.floor(torch.log2(448.0 / s.max())))  # a power of two: s * glob stays exact
        out[prefix + "weight_packed"] = qw.qweight
        out[prefix + "weight_scale"] = (s * glob).to(torch.float8_e4m3fn)
        out[prefix + "weight_global_scale"] = torch.tensor([glob], dtype=torch.float32)
        scheme.update({"num_bits": 4, "type": "float", "symmetric": True, "strategy": "tensor_group"})
    elif fmt == "mxfp4":
        exponent = torch.log2(scale.float()).round().to(torch.int64) + 127
        out[prefix + "weight_packed"] = qw.qweight
        out[prefix + "weight_scale"] = exponent.clamp(0, 254).to(torch.uint8)
        scheme.update({"num_bits": 4, "type": "float", "symmetric": True, "scale_dtype": "e8m0"})
    else:
        raise ConfigError(f"no compressed-tensors scheme for format {fmt!r}")
    if scheme["strategy"] != "channel":
        scheme["group_size"] = qw.group
    return out, scheme


def export_compressed_tensors(model, path: str | Path) -> Path:
    """Write ``model``'s target (an EfficientModel or CausalLM whose projections the ``quant`` technique replaced)
    as a compressed-tensors folder; returns the folder."""
    from ..backends.exporters import refuse_online_rotation

    refuse_online_rotation(getattr(model, "model", model), "compressed-tensors")
    from safetensors.torch import save_file

    lm = getattr(model, "model", model)
    c = lm.config
    if c.is_moe:
        raise ConfigError("the compressed-tensors export covers dense models")
    hf = lm.hf_state_dict()
    tensors: dict[str, torch.Tensor] = {}
    schemes: dict[str, dict[str, Any]] = {}
    quantized = set()
    formats = set()
    splits = {"wqkv": [("self_attn.q_proj", c.q_size), ("self_attn.k_proj", c.kv_size),
                       ("self_attn.v_proj", c.kv_size)],
              "wo": [("self_attn.o_proj", c.hidden_size)],
              "w_gate_up": [("mlp.gate_proj", c.intermediate_size), ("mlp.up_proj", c.intermediate_size)],
              "w_down": [("mlp.down_proj", c.hidden_size)]}
    for i, layer in enumerate(lm.layers):
        for attr, parts in splits.items():
            qw = getattr(layer, attr)
            if not isinstance(qw, QWeight):
                continue
            formats.add(qw.fmt)
            start = 0
            for name, rows in parts:
                module = f"model.layers.{i}.{name}"
                entries, scheme = _linear_entries(qw.rows(start, start + rows), module + ".")
                tensors.update(entries)
                schemes[module] = scheme
                quantized.add(module)
                start += rows
    if not quantized:
        raise ConfigError("the model has no quantized projections to export (apply the quant technique first)")
    for name, t in hf.items():
        if not (name.endswith(".weight") and name[: -len(".weight")] in quantized):
            tensors[name] = t.detach().to(lm.dtype)
    kinds = {json.dumps(s, sort_keys=True) for s in schemes.values()}
    if len(kinds) != 1 or len(formats) != 1:
        raise ConfigError("the quantized projections use several schemes; export one format and group size")
    scheme = schemes[next(iter(schemes))]
    fmt = formats.pop()
    linears = [f"model.layers.{i}.{name}" for i in range(c.num_layers) for parts in splits.values()
               for name, _ in parts]
    config = c.to_hf().to_dict()
    config["quantization_config"] = {
        "quant_method": "compressed-tensors", "format": _CT_FORMAT[fmt], "quantization_status": "compressed",
        "config_groups": {"group_0": {"targets": ["Linear"], "weights": scheme, "input_activations": None,
                                      "output_activations": None}},
        "ignore": ["lm_head"] + [m for m in linears if m not in quantized],
    }
    out = Path(path)
    out.mkdir(parents=True, exist_ok=True)
    (out / "config.json").write_text(json.dumps(config, indent=2, default=str) + "\n")
    save_file({k: v.contiguous().cpu() for k, v in tensors.items()}, str(out / "model.safetensors"),
              metadata={"format": "pt"})
    return out


def read_compressed_tensors(path: str | Path) -> tuple[dict[str, Any], dict[str, torch.Tensor]]:
    """``(config, dense Hugging Face state dict)`` of a folder written by :func:`export_compressed_tensors`."""
    from safetensors.torch import load_file

    from ..ops.quant import E2M1_VALUES

    folder = Path(path)
    config = json.loads((folder / "config.json").read_text())
    qc = config.get("quantization_config") or {}
    if qc.get("quant_method") != "compressed-tensors":
        raise CheckpointFormatError(f"{folder} is not a compressed-tensors checkpoint")
    fmt = qc["format"]
    scheme = qc["config_groups"]["group_0"]["weights"]
    raw = load_file(str(folder / "model.safetensors"))
    dense: dict[str, torch.Tensor] = {}
    modules = {k.rsplit(".", 1)[0] for k in raw if k.endswith(".weight_scale")}
    for name, t in raw.items():
        if name.rsplit(".", 1)[0] not in modules:
            dense[name] = t
    table = torch.tensor(E2M1_VALUES)
    for m in modules:
        scale = raw[m + ".weight_scale"]
        if fmt == "pack-quantized":
            n, k = (int(v) for v in raw[m + ".weight_shape"])
            q = _unpack_int32(raw[m + ".weight_packed"], int(scheme["num_bits"]), k).float()
        elif fmt == "int-quantized":
            q = raw[m + ".weight"].float()
        elif fmt == "float-quantized":
            q = raw[m + ".weight"].float()
        elif fmt in ("nvfp4-pack-quantized", "mxfp4-pack-quantized"):
            b = raw[m + ".weight_packed"].to(torch.int64)
            codes = torch.stack([b & 0xF, b >> 4], -1).reshape(b.shape[0], -1)
            q = torch.where(codes >= 8, -table[codes & 7], table[codes & 7])
            if fmt == "nvfp4-pack-quantized":
                scale = scale.float() / raw[m + ".weight_global_scale"].float()
            else:
                scale = torch.exp2(scale.float() - 127.0)
        else:
            raise CheckpointFormatError(f"compressed-tensors format {fmt!r} is not read here")
        group = q.shape[1] // scale.shape[1]
        zp = raw.get(m + ".weight_zero_point")
        if zp is not None:
            q = q - zp.float().repeat_interleave(group, 1)
        w = q * scale.float().repeat_interleave(group, 1)
        dense[m + ".weight"] = w.to(torch.bfloat16)
    return config, dense
