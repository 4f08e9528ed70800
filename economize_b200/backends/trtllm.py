"""Export a model as a TensorRT-LLM checkpoint (the input of ``trtllm-build``; economize ``backends/trtllm``):
``config.json`` and one ``rank{r}.safetensors`` per tensor-parallel rank, written without TensorRT-LLM installed.

The Llama block's names: ``attention.qkv`` (rows of q, then k, then v: the engine's own ``wqkv``), ``attention.dense``
(``o_proj``), ``mlp.fc`` (``gate_proj``), ``mlp.gate`` (``up_proj``), ``mlp.proj`` (``down_proj``),
``input_layernorm``, ``post_layernorm``; ``transformer.vocab_embedding``, ``transformer.ln_f``, ``lm_head``.
Symmetric group-wise int4 projections (zero point 8) are stored as ``W4A16_AWQ`` codes in the layout TensorRT-LLM
reads: ``p.weight`` ``int8 [out / 2, in]`` (signed codes ``q - 8``, row ``2i`` in the low nibble, ``2i + 1`` in the
high one), ``p.weights_scaling_factor`` ``[in / group, out]`` and ``p.prequant_scaling_factor`` ``[in]`` ones; other
formats are written dequantized (TensorRT-LLM's own build quantizes float weights). Tensor parallelism splits q/k/v
heads, gate/up rows and o/down columns per rank.
"""

from __future__ import annotations

import json
from pathlib import Path

import torch

from ..errors import ConfigError
from ..ops.quant import QWeight, unpack

__all__ = ["QUANT_ALGO", "pack_int4_rows", "to_trtllm", "trtllm_config"]

QUANT_ALGO = "W4A16_AWQ"


def pack_int4_rows(signed: torch.Tensor) -> torch.Tensor:
    """Signed int4 codes ``[out, in]`` (-8..7) as ``int8 [out / 2, in]``: even rows in the low nibbles."""
    if signed.shape[0] % 2:
        raise ConfigError(f"W4A16_AWQ packs two rows per byte; got {signed.shape[0]} rows")
    nib = signed.to(torch.int16) & 0xF
    return (nib[0::2] | (nib[1::2] << 4)).to(torch.uint8).view(torch.int8).contiguous()


def _awq_form(qw) -> tuple[torch.Tensor, torch.Tensor] | None:
    """(signed codes [N, K], scales [N, K / g]) when ``qw`` is symmetric group-wise int4, else None."""
    if not isinstance(qw, QWeight) or qw.fmt != "int4" or qw.zeros is None or qw.group not in (64, 128):
        return None
    if not bool((qw.zeros.float() == 136.0).all()):  # stored as 128 + z: symmetric grids have z = 8
        return None
    return unpack(qw.qweight.cpu(), "int4") - 8, qw.scales.float().cpu().t()


def trtllm_config(c, dtype: torch.dtype, tp: int, group: int | None) -> dict:
    """``config.json`` of a Llama-block model (the keys ``trtllm-build`` reads)."""
    rope = dict(c.rope_scaling) if c.rope_scaling else None
    cfg = {
        "architecture": "LlamaForCausalLM", "dtype": str(dtype).removeprefix("torch."),
        "logits_dtype": "float32", "vocab_size": c.vocab_size, "max_position_embeddings": c.max_position_embeddings,
        "hidden_size": c.hidden_size, "num_hidden_layers": c.num_layers, "num_attention_heads": c.num_heads,
        "num_key_value_heads": c.num_kv_heads, "head_size": c.head_dim, "intermediate_size": c.intermediate_size,
        "hidden_act": "silu", "norm_epsilon": c.rms_norm_eps, "position_embedding_type": "rope_gpt_neox",
        "rotary_base": c.rope_theta, "rotary_scaling": rope, "tie_word_embeddings": c.tie_word_embeddings,
        "mapping": {"world_size": tp, "tp_size": tp, "pp_size": 1},
        "quantization": {"quant_algo": QUANT_ALGO if group else None, "group_size": group or 128,
                         "has_zero_point": False, "pre_quant_scale": bool(group)},
    }
    return cfg


_LINEARS = {"wqkv": "attention.qkv", "wo": "attention.dense", "w_down": "mlp.proj"}


def to_trtllm(model, folder: str | Path, tp: int = 1, dtype: torch.dtype = torch.bfloat16) -> Path:
    """Write ``model`` (a dense Llama-block engine model, possibly with int4 ``QWeight`` projections) as a
    TensorRT-LLM checkpoint for ``tp`` ranks; returns the folder."""
    from safetensors.torch import save_file

    target = getattr(model, "model", model)
    from .exporters import refuse_online_rotation

    refuse_online_rotation(target, "TensorRT-LLM")
    c = target.config
    if c.is_moe or c.post_norm or c.sandwich_norm or c.hidden_act != "silu" or c.qk_norm or c.attention_bias:
        raise ConfigError("the TensorRT-LLM writer covers the plain Llama block")
    if c.num_heads % tp or c.num_kv_heads % tp or c.intermediate_size % tp:
        raise ConfigError(f"heads and FFN width must split over {tp} ranks")
    folder = Path(folder)
    folder.mkdir(parents=True, exist_ok=True)
    d = c.head_dim
    groups = set()

    def rows_of(name: str, r: int) -> torch.Tensor:
        """Row indices of rank r's shard of a column-parallel projection."""
        if name == "wqkv":
            hq, hk = c.num_heads // tp, c.num_kv_heads // tp
            q = torch.arange(r * hq * d, (r + 1) * hq * d)
            k = c.q_size + torch.arange(r * hk * d, (r + 1) * hk * d)
            return torch.cat([q, k, k + c.kv_size])
        f = c.intermediate_size // tp
        return torch.cat([torch.arange(r * f, (r + 1) * f), c.intermediate_size + torch.arange(r * f, (r + 1) * f)])

    for r in range(tp):
        out: dict[str, torch.Tensor] = {}
        v = c.vocab_size
        out["transformer.vocab_embedding.weight"] = target.embed.detach().to(dtype).cpu()
        out["transformer.ln_f.weight"] = target.norm.detach().to(dtype).cpu()
        out["lm_head.weight"] = target.head_weight.detach().to(dtype).cpu()
        for i, layer in enumerate(target.layers):
            p = f"transformer.layers.{i}."
            out[p + "input_layernorm.weight"] = layer.attn_norm.detach().to(dtype).cpu()
            out[p + "post_layernorm.weight"] = layer.mlp_norm.detach().to(dtype).cpu()
            for name in ("wqkv", "w_gate_up", "wo", "w_down"):
                w = getattr(layer, name)
                awq = _awq_form(w)
                if name in ("wqkv", "w_gate_up"):
                    rows, cols = rows_of(name, r), slice(None)
                else:
                    k_per = w.shape[1] // tp
                    rows, cols = slice(None), slice(r * k_per, (r + 1) * k_per)
                if awq is not None:
                    codes, scales = awq
                    groups.add(w.group)
                    codes = codes[rows][:, cols]
                    scales = scales[rows][:, cols if cols == slice(None) else
                                          slice(cols.start // w.group, cols.stop // w.group)]
                    parts = [(codes, scales)]
                else:
                    dense = (w.dequantize() if not isinstance(w, torch.Tensor) else w.detach()).float().cpu()
                    parts = [(dense[rows][:, cols], None)]
                tensors = {}
                if name == "w_gate_up":  # gate rows first, then up rows: mlp.fc and mlp.gate
                    data, sc = parts[0]
                    half = data.shape[0] // 2
                    tensors["mlp.fc"] = (data[:half], None if sc is None else sc[:half])
                    tensors["mlp.gate"] = (data[half:], None if sc is None else sc[half:])
                else:
                    tensors[_LINEARS[name]] = parts[0]
                for tname, (data, sc) in tensors.items():
                    if sc is None:
                        out[p + tname + ".weight"] = data.to(dtype).contiguous()
                    else:
                        out[p + tname + ".weight"] = pack_int4_rows(data)
                        out[p + tname + ".weights_scaling_factor"] = sc.t().to(dtype).contiguous()
                        out[p + tname + ".prequant_scaling_factor"] = torch.ones(data.shape[1], dtype=dtype)
        save_file({k: v.contiguous() for k, v in out.items()}, str(folder / f"rank{r}.safetensors"))
    if len(groups) > 1:
        raise ConfigError(f"a TensorRT-LLM checkpoint has one group size; this model mixes {sorted(groups)}")
    cfg = trtllm_config(c, dtype, tp, next(iter(groups)) if groups else None)
    (folder / "config.json").write_text(json.dumps(cfg, indent=2))
    return folder
