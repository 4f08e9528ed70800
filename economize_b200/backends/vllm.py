"""Exporters for vLLM's draft models (economize ``backends/vllm/eagle3/export.py:1-197``,
``backends/vllm/medusa/export.py``; the layouts are the public checkpoint formats vLLM reads, so the tensor names
and config keys below must be exactly these).

* ``vllm/eagle3``: the layout of the published EAGLE-3 heads: a one-layer Llama ``config.json`` with
  ``draft_vocab_size``, ``target_hidden_size`` and ``eagle_aux_hidden_state_layer_ids``, and the tensors
  ``fc.weight``, ``midlayer.*``, ``norm.weight``, ``lm_head.weight``, ``d2t``, ``t2d`` (no embedding: vLLM shares
  the target's). ``format="speculators"`` writes the same fields in the ``speculators`` layout
  (``Eagle3Speculator``, layer config under ``transformer_layer_config``, verifier under ``speculators_config``).
  A ``head="shared"`` drafter exports the model's final norm and no ``lm_head``/``d2t``/``t2d`` (vLLM then shares
  the target's LM head); a full draft vocabulary drops ``d2t``/``t2d``, which vLLM allocates only for a reduced one.
* ``vllm/eagle``: EAGLE-1/2 heads in the layout of the published EAGLE checkpoints: ``fc.weight``/``fc.bias`` over
  ``[embedding; feature]`` and ``layers.0.*`` (no input norm on that layer).
* ``vllm/medusa``: ``head="own"`` Medusa heads as vLLM's ``MedusaModel``: ``blocks.{h}.layers.{l}`` residual
  blocks on the post-norm state and ``lm_heads.{h}``.
"""

from __future__ import annotations

from typing import Any

import torch

from ..errors import ConfigError
from .exporters import DrafterExporter, register_exporter

__all__ = ["EagleVllmExporter", "Eagle3VllmExporter", "MedusaVllmExporter", "draft_layer_tensors"]


def draft_layer_tensors(layer, prefix: str) -> dict[str, torch.Tensor]:
    """A fused draft layer's tensors under Llama names (``q/k/v_proj``, ``gate/up_proj`` split)."""
    q_n, kv_n = layer.heads * layer.head_dim, layer.kv_heads * layer.head_dim
    q, k, v = layer.wqkv.detach().split([q_n, kv_n, kv_n], 0)
    gate, up = layer.w_gate_up.detach().chunk(2, 0)
    out = {f"{prefix}self_attn.q_proj.weight": q, f"{prefix}self_attn.k_proj.weight": k,
           f"{prefix}self_attn.v_proj.weight": v, f"{prefix}self_attn.o_proj.weight": layer.wo.detach(),
           f"{prefix}post_attention_layernorm.weight": layer.post_norm.detach(),
           f"{prefix}mlp.gate_proj.weight": gate, f"{prefix}mlp.up_proj.weight": up,
           f"{prefix}mlp.down_proj.weight": layer.w_down.detach()}
    if layer.bqkv is not None:
        bq, bk, bv = layer.bqkv.detach().split([q_n, kv_n, kv_n], 0)
        out.update({f"{prefix}self_attn.q_proj.bias": bq, f"{prefix}self_attn.k_proj.bias": bk,
                    f"{prefix}self_attn.v_proj.bias": bv,
                    # vLLM gives o_proj a bias whenever attention_bias is set; the draft layer has none
                    f"{prefix}self_attn.o_proj.bias": torch.zeros_like(layer.wo[:, 0])})
    return out


def _layer_config(technique, layer, *, intermediate: int) -> dict[str, Any]:
    c = technique.model.config
    rope_theta = float(technique.config.rope_theta or c.rope_theta)
    rope = dict(technique.config.rope_scaling or (c.rope_scaling if not technique.config.rope_theta else None)
                or {})
    rope.setdefault("rope_type", rope.pop("type", "default"))
    rope["rope_theta"] = rope_theta
    return {
        "architectures": ["LlamaForCausalLM"], "model_type": "llama", "num_hidden_layers": 1,
        "hidden_size": int(c.hidden_size), "intermediate_size": int(intermediate),
        "num_attention_heads": int(layer.heads), "num_key_value_heads": int(layer.kv_heads),
        "head_dim": int(layer.head_dim), "hidden_act": "silu", "attention_bias": layer.bqkv is not None,
        "mlp_bias": False, "rms_norm_eps": float(layer.eps), "vocab_size": int(c.vocab_size),
        "max_position_embeddings": int(c.max_position_embeddings), "rope_theta": rope_theta,
        "rope_scaling": None if rope == {"rope_type": "default", "rope_theta": rope_theta} else rope,
        "rope_parameters": rope, "tie_word_embeddings": False,
        "torch_dtype": str(layer.wqkv.dtype).removeprefix("torch."),
    }


@register_exporter("vllm", "eagle3")
class Eagle3VllmExporter(DrafterExporter):
    """EAGLE-3 heads as vLLM's EAGLE-3 draft model (``speculative_config={"method": "eagle3", "model": <folder>}``;
    ``format="speculators"`` for ``vllm serve <folder>``)."""

    def config(self, technique, *, format: str = "eagle3", num_speculative_tokens: int = 4,
               verifier: str | None = None) -> dict[str, Any]:
        layer = technique.layer
        cfg = _layer_config(technique, layer, intermediate=layer.w_down.shape[1])
        cfg.update({"target_hidden_size": int(technique.model.config.hidden_size),
                    "draft_vocab_size": int(technique.draft_vocab), "use_aux_hidden_state": True,
                    "norm_before_residual": bool(technique.config.norm_before_residual),
                    "eagle_aux_hidden_state_layer_ids": [int(i) for i in technique.aux_layers]})
        if format == "eagle3":
            return cfg
        if format != "speculators":
            raise ConfigError(f"unknown export format {format!r}: expected 'eagle3' or 'speculators'")
        if not verifier:
            raise ConfigError("the speculators format names its verifier: pass verifier='<target id or path>'")
        top = {k: cfg[k] for k in ("draft_vocab_size", "target_hidden_size", "norm_before_residual",
                                   "eagle_aux_hidden_state_layer_ids", "torch_dtype")}
        return {"architectures": ["Eagle3Speculator"], "speculators_model_type": "eagle3",
                "transformer_layer_config": cfg,
                "speculators_config": {
                    "algorithm": "eagle3", "default_proposal_method": "greedy",
                    "proposal_methods": [{"proposal_type": "greedy", "speculative_tokens": num_speculative_tokens}],
                    "verifier": {"name_or_path": verifier, "architectures": ["LlamaForCausalLM"]}},
                **top}

    def tensors(self, technique) -> dict[str, torch.Tensor]:
        out = {"fc.weight": technique.fc.detach(),
               "midlayer.input_layernorm.weight": technique.input_norm.detach(),
               "midlayer.hidden_norm.weight": technique.hidden_norm.detach(),
               **draft_layer_tensors(technique.layer, "midlayer.")}
        model = technique.model
        if technique.shared_head:
            out["norm.weight"] = model.norm.detach().to(technique.fc.dtype)
        else:
            out["norm.weight"] = technique.norm.detach()
            out["lm_head.weight"] = technique.lm_head.detach()
            if technique.draft_vocab < model.config.vocab_size:
                out["d2t"] = technique.d2t.detach()
                out["t2d"] = technique.t2d.detach()
        return out


@register_exporter("vllm", "eagle")
class EagleVllmExporter(DrafterExporter):
    """EAGLE-1/2 heads as vLLM's EAGLE draft model (``speculative_config={"method": "eagle", ...}``)."""

    def config(self, technique, **options: Any) -> dict[str, Any]:
        if options:
            raise ConfigError(f"vllm/eagle takes no options, got {sorted(options)}")
        layer = technique.layer
        cfg = _layer_config(technique, layer, intermediate=layer.w_down.shape[1])
        cfg["fc_bias"] = technique.fc_bias is not None
        return cfg

    def tensors(self, technique) -> dict[str, torch.Tensor]:
        out = {"fc.weight": technique.fc.detach(), **draft_layer_tensors(technique.layer, "layers.0.")}
        if technique.fc_bias is not None:
            out["fc.bias"] = technique.fc_bias.detach()
        return out


@register_exporter("vllm", "medusa")
class MedusaVllmExporter(DrafterExporter):
    """``head="own"`` Medusa heads as vLLM's ``MedusaModel``. vLLM has no head that applies the model's final norm
    after its blocks (``head="shared"``), so those are refused."""

    def _own(self, technique):
        if technique.config.head != "own":
            raise ConfigError("vLLM's Medusa runs its blocks on the post-norm state with one projection per head; "
                              "export a head='own' Medusa technique")
        return technique

    def config(self, technique, **options: Any) -> dict[str, Any]:
        if options:
            raise ConfigError(f"vllm/medusa takes no options, got {sorted(options)}")
        t = self._own(technique)
        c = t.model.config
        return {"architectures": ["MedusaModel"], "model_type": "medusa", "hidden_size": int(c.hidden_size),
                "vocab_size": int(c.vocab_size), "num_heads": len(t.heads),
                "num_hidden_layers": int(t.config.num_layers), "medusa_fc_bias": True,
                "truncated_vocab_size": int(c.vocab_size),
                "torch_dtype": str(t.heads[0].proj.weight.dtype).removeprefix("torch.")}

    def tensors(self, technique) -> dict[str, torch.Tensor]:
        t = self._own(technique)
        out = {}
        for h, head in enumerate(t.heads):
            for j, block in enumerate(head.blocks):
                out[f"blocks.{h}.layers.{j}.weight"] = block.linear.weight.detach()
                out[f"blocks.{h}.layers.{j}.bias"] = block.linear.bias.detach()
            out[f"lm_heads.{h}.weight"] = head.proj.weight.detach()
        return out
