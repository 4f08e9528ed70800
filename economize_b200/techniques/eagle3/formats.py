"""EAGLE-3 checkpoint layouts.

* economize / reference layout (``fc.weight``, ``layer.self_attn.q_proj.weight`` ..., ``norm.weight``,
  ``lm_head.weight``, ``d2t``, ``t2d``): what economize's ``Eagle3Technique`` holds and saves.
* official layout (SafeAILab / SpecForge, ``midlayer.*``) and vLLM ``speculators`` (``layers.0.*``).

The engine fuses q/k/v and gate/up; these functions split and join them. Conversions only rename and
concatenate; no values change.
"""

from __future__ import annotations

import torch

__all__ = ["from_official_state", "from_reference_state", "to_official_state", "to_reference_state"]

_LAYER_PREFIXES = ("layer.", "midlayer.", "layers.0.")


def to_reference_state(tech) -> dict[str, torch.Tensor]:
    """The technique's tensors under economize's ``Eagle3Technique`` names (``layer.*``)."""
    layer = tech.layer
    q, k, v = layer.wqkv.detach().split([layer.heads * layer.head_dim, layer.kv_heads * layer.head_dim,
                                         layer.kv_heads * layer.head_dim], 0)
    gate, up = layer.w_gate_up.detach().chunk(2, 0)
    out = {
        "d2t": tech.d2t.detach(), "t2d": tech.t2d.detach(), "fc.weight": tech.fc.detach(),
        "layer.input_layernorm.weight": tech.input_norm.detach(),
        "layer.hidden_norm.weight": tech.hidden_norm.detach(),
        "layer.post_attention_layernorm.weight": layer.post_norm.detach(),
        "layer.self_attn.q_proj.weight": q, "layer.self_attn.k_proj.weight": k, "layer.self_attn.v_proj.weight": v,
        "layer.self_attn.o_proj.weight": layer.wo.detach(),
        "layer.mlp.gate_proj.weight": gate, "layer.mlp.up_proj.weight": up,
        "layer.mlp.down_proj.weight": layer.w_down.detach(),
    }
    if layer.bqkv is not None:
        bq, bk, bv = layer.bqkv.detach().split([q.shape[0], k.shape[0], v.shape[0]], 0)
        out.update({"layer.self_attn.q_proj.bias": bq, "layer.self_attn.k_proj.bias": bk,
                    "layer.self_attn.v_proj.bias": bv})
    if not tech.shared_head:
        out["norm.weight"] = tech.norm.detach()
        out["lm_head.weight"] = tech.lm_head.detach()
    return {k: v.contiguous() for k, v in out.items()}


def from_reference_state(tech, state: dict[str, torch.Tensor]) -> None:
    """Load economize-named (or official ``midlayer.*`` / ``layers.0.*``) tensors into the technique."""
    norm = {}
    for key, value in state.items():
        for prefix in _LAYER_PREFIXES:
            if key.startswith(prefix):
                key = "layer." + key[len(prefix):]
                break
        norm[key] = value
    layer = tech.layer
    with torch.no_grad():
        def put(dst: torch.Tensor, src: torch.Tensor) -> None:
            dst.copy_(src.to(dst.device, dst.dtype))

        put(tech.fc, norm["fc.weight"])
        put(tech.input_norm, norm["layer.input_layernorm.weight"])
        put(tech.hidden_norm, norm["layer.hidden_norm.weight"])
        put(layer.post_norm, norm["layer.post_attention_layernorm.weight"])
        put(layer.wqkv, torch.cat([norm[f"layer.self_attn.{n}_proj.weight"] for n in "qkv"], 0))
        if layer.bqkv is not None and "layer.self_attn.q_proj.bias" in norm:
            put(layer.bqkv, torch.cat([norm[f"layer.self_attn.{n}_proj.bias"] for n in "qkv"], 0))
        put(layer.wo, norm["layer.self_attn.o_proj.weight"])
        put(layer.w_gate_up, torch.cat([norm["layer.mlp.gate_proj.weight"], norm["layer.mlp.up_proj.weight"]], 0))
        put(layer.w_down, norm["layer.mlp.down_proj.weight"])
        if not tech.shared_head:
            put(tech.norm, norm["norm.weight"])
            put(tech.lm_head, norm["lm_head.weight"])
        if "d2t" in norm:
            put(tech.d2t, norm["d2t"])
        if "t2d" in norm:
            put(tech.t2d, norm["t2d"].bool())
        elif "d2t" in norm:
            tech.t2d.zero_()
            ids = torch.arange(tech.d2t.numel(), device=tech.d2t.device) + tech.d2t
            tech.t2d[ids] = True


def to_official_state(tech) -> dict[str, torch.Tensor]:
    """The official SafeAILab layout (``midlayer.*``)."""
    return {("midlayer." + k[len("layer."):] if k.startswith("layer.") else k): v
            for k, v in to_reference_state(tech).items()}


def from_official_state(tech, state: dict[str, torch.Tensor]) -> None:
    from_reference_state(tech, state)
