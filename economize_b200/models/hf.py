"""Conversion between Hugging Face state dicts and the engine's fused parameter layout.

Gemma's RMSNorm weights ``w`` (the norm scales by ``1 + w``) are stored as ``1 + w`` here, so every family runs the
same norm kernel; sandwich blocks (Gemma-2/3) map four norms per block.

Names follow ``transformers`` 5 (``model.layers.{i}.self_attn.q_proj.weight`` ..., Mixtral experts as fused
``mlp.experts.gate_up_proj [E, 2F, H]`` / ``down_proj [E, H, F]``; the older per-expert ``block_sparse_moe.experts.
{e}.w1/w2/w3`` layout is read too). gpt-oss stores its experts input-major with gate and up interleaved
(``gate_up_proj [E, H, 2F]``, gate in the even columns; ``down_proj [E, F, H]``) and its router as
``mlp.router.{weight, bias}``; they are transposed and de-interleaved into the fused ``[gate; up]`` rows here.
"""

from __future__ import annotations

import torch

from ..errors import CheckpointFormatError

__all__ = ["export_hf_state", "load_hf_state"]


def _take(state: dict[str, torch.Tensor], key: str) -> torch.Tensor:
    if key not in state:
        raise CheckpointFormatError(f"missing weight {key!r}")
    return state[key]


def _norm_in(config, w: torch.Tensor) -> torch.Tensor:
    """A checkpoint's RMSNorm weight as this model stores it (Gemma checkpoints store ``w`` of ``1 + w``)."""
    return w.float() + 1.0 if config.norm_unit_offset else w


def _norm_out(config, w: torch.Tensor) -> torch.Tensor:
    return (w.detach().float() - 1.0).to(w.dtype) if config.norm_unit_offset else w.detach()


@torch.no_grad()
def load_hf_state(model, state: dict[str, torch.Tensor]) -> None:
    """Copy a Hugging Face state dict into ``model`` (a :class:`~economize_b200.models.CausalLM`)."""
    c = model.config
    model.embed.copy_(_take(state, "model.embed_tokens.weight"))
    model.norm.copy_(_norm_in(c, _take(state, "model.norm.weight")))
    if model.lm_head is not None:
        model.lm_head.copy_(state.get("lm_head.weight", state["model.embed_tokens.weight"]))
    for i, layer in enumerate(model.layers):
        p = f"model.layers.{i}."
        a = p + "self_attn."
        if a + "qkv_proj.weight" in state:  # fused checkpoints (phi3): [q; k; v] rows already
            layer.wqkv.copy_(state[a + "qkv_proj.weight"])
        else:
            layer.wqkv.copy_(torch.cat([_take(state, a + f"{n}_proj.weight") for n in "qkv"], 0))
        if layer.bqkv is not None:
            layer.bqkv.copy_(torch.cat([_take(state, a + f"{n}_proj.bias") for n in "qkv"], 0))
        layer.wo.copy_(_take(state, a + "o_proj.weight"))
        if layer.bo is not None:
            layer.bo.copy_(_take(state, a + "o_proj.bias"))
        if layer.q_norm is not None:
            layer.q_norm.copy_(_norm_in(c, _take(state, a + "q_norm.weight")))
            layer.k_norm.copy_(_norm_in(c, _take(state, a + "k_norm.weight")))
        for ours, theirs in _norm_names(c):
            getattr(layer, ours).copy_(_norm_in(c, _take(state, p + theirs + ".weight")))
        if layer.sinks is not None and a + "sinks" in state:
            layer.sinks.copy_(state[a + "sinks"])
        if c.is_moe and c.model_type == "gpt_oss":
            x = p + "mlp.experts."
            layer.router.copy_(_take(state, p + "mlp.router.weight"))
            layer.router_bias.copy_(_take(state, p + "mlp.router.bias"))
            gu = _take(state, x + "gate_up_proj").transpose(1, 2)  # [E, 2F, H], gate rows even
            layer.w_gate_up.copy_(torch.cat([gu[:, 0::2], gu[:, 1::2]], 1))
            b = _take(state, x + "gate_up_proj_bias")
            layer.b_gate_up.copy_(torch.cat([b[:, 0::2], b[:, 1::2]], 1))
            layer.w_down.copy_(_take(state, x + "down_proj").transpose(1, 2))
            layer.b_down.copy_(_take(state, x + "down_proj_bias"))
        elif c.is_moe and c.model_type in ("granitemoe", "granitemoeshared"):
            m = p + "block_sparse_moe."
            layer.router.copy_(_take(state, m + "router.layer.weight"))
            layer.w_gate_up.copy_(_take(state, m + "input_linear.weight"))  # [E, 2F, H], gate half first
            layer.w_down.copy_(_take(state, m + "output_linear.weight"))
            if layer.w_shared_gate_up is not None:
                layer.w_shared_gate_up.copy_(_take(state, p + "shared_mlp.input_linear.weight"))
                layer.w_shared_down.copy_(_take(state, p + "shared_mlp.output_linear.weight"))
        elif c.is_moe:
            if p + "mlp.experts.gate_up_proj" in state:
                layer.router.copy_(_take(state, p + "mlp.gate.weight"))
                layer.w_gate_up.copy_(state[p + "mlp.experts.gate_up_proj"])
                layer.w_down.copy_(_take(state, p + "mlp.experts.down_proj"))
                if layer.w_shared_gate_up is not None:  # qwen2_moe
                    x = p + "mlp.shared_expert."
                    layer.w_shared_gate_up.copy_(torch.cat([_take(state, x + "gate_proj.weight"),
                                                            _take(state, x + "up_proj.weight")], 0))
                    layer.w_shared_down.copy_(_take(state, x + "down_proj.weight"))
                    layer.shared_gate.copy_(_take(state, p + "mlp.shared_expert_gate.weight"))
            else:
                m = p + "block_sparse_moe."
                layer.router.copy_(_take(state, m + "gate.weight"))
                for e in range(c.num_experts):
                    x = m + f"experts.{e}."
                    layer.w_gate_up[e].copy_(torch.cat([_take(state, x + "w1.weight"),
                                                        _take(state, x + "w3.weight")], 0))
                    layer.w_down[e].copy_(_take(state, x + "w2.weight"))
        else:
            m = p + "mlp."
            if m + "gate_up_proj.weight" in state:  # fused checkpoints (phi3): [gate; up]
                layer.w_gate_up.copy_(state[m + "gate_up_proj.weight"])
            else:
                layer.w_gate_up.copy_(torch.cat([_take(state, m + "gate_proj.weight"),
                                                 _take(state, m + "up_proj.weight")], 0))
            layer.w_down.copy_(_take(state, m + "down_proj.weight"))


def _norm_names(config) -> list[tuple[str, str]]:
    """(this model's parameter, the checkpoint's name) of a block's norms."""
    if config.sandwich_norm:  # gemma2 / gemma3: a norm before and after each branch
        return [("attn_norm", "input_layernorm"), ("attn_post_norm", "post_attention_layernorm"),
                ("mlp_norm", "pre_feedforward_layernorm"), ("mlp_post_norm", "post_feedforward_layernorm")]
    if config.post_norm:  # olmo2 / olmo3: the norms follow the branches (attn_norm / mlp_norm hold them)
        return [("attn_norm", "post_attention_layernorm"), ("mlp_norm", "post_feedforward_layernorm")]
    return [("attn_norm", "input_layernorm"), ("mlp_norm", "post_attention_layernorm")]


@torch.no_grad()
def export_hf_state(model, copy: bool = True) -> dict[str, torch.Tensor]:
    """The Hugging Face state dict of ``model`` (split projections, ``transformers`` 5 names); quantized projections
    are dequantized. ``copy=False`` returns views where possible."""
    from ..ops.quant import QWeight

    c = model.config

    def full(t):
        if isinstance(t, QWeight) or (not isinstance(t, torch.Tensor) and hasattr(t, "dequantize")):
            return t.dequantize()
        return t.detach()

    out = {"model.embed_tokens.weight": model.embed.detach(), "model.norm.weight": _norm_out(c, model.norm)}
    if model.lm_head is not None:
        out["lm_head.weight"] = model.lm_head.detach()
    for i, layer in enumerate(model.layers):
        p = f"model.layers.{i}."
        if c.model_type == "phi3":
            out[p + "self_attn.qkv_proj.weight"] = full(layer.wqkv)
        else:
            q, k, v = full(layer.wqkv).split([c.q_size, c.kv_size, c.kv_size], 0)
            for n, w in zip("qkv", (q, k, v)):
                out[p + f"self_attn.{n}_proj.weight"] = w
        if layer.bqkv is not None:
            for n, w in zip("qkv", layer.bqkv.detach().split([c.q_size, c.kv_size, c.kv_size], 0)):
                out[p + f"self_attn.{n}_proj.bias"] = w
        out[p + "self_attn.o_proj.weight"] = full(layer.wo)
        if layer.bo is not None:
            out[p + "self_attn.o_proj.bias"] = layer.bo.detach()
        if layer.q_norm is not None:
            out[p + "self_attn.q_norm.weight"] = _norm_out(c, layer.q_norm)
            out[p + "self_attn.k_norm.weight"] = _norm_out(c, layer.k_norm)
        for ours, theirs in _norm_names(c):
            out[p + theirs + ".weight"] = _norm_out(c, getattr(layer, ours))
        if layer.sinks is not None:
            out[p + "self_attn.sinks"] = layer.sinks.detach()
        if c.is_moe and c.model_type == "gpt_oss":
            x = p + "mlp.experts."
            out[p + "mlp.router.weight"] = layer.router.detach()
            out[p + "mlp.router.bias"] = layer.router_bias.detach()
            g, u = full(layer.w_gate_up).chunk(2, 1)  # [E, F, H] each
            out[x + "gate_up_proj"] = torch.stack([g, u], 2).reshape(g.shape[0], -1, g.shape[2]).transpose(1, 2)
            bg, bu = layer.b_gate_up.detach().chunk(2, 1)
            out[x + "gate_up_proj_bias"] = torch.stack([bg, bu], 2).reshape(bg.shape[0], -1)
            out[x + "down_proj"] = full(layer.w_down).transpose(1, 2)
            out[x + "down_proj_bias"] = layer.b_down.detach()
        elif c.is_moe and c.model_type in ("granitemoe", "granitemoeshared"):
            m = p + "block_sparse_moe."
            out[m + "router.layer.weight"] = layer.router.detach()
            out[m + "input_linear.weight"] = full(layer.w_gate_up)
            out[m + "output_linear.weight"] = full(layer.w_down)
            if layer.w_shared_gate_up is not None:
                out[p + "shared_mlp.input_linear.weight"] = full(layer.w_shared_gate_up)
                out[p + "shared_mlp.output_linear.weight"] = full(layer.w_shared_down)
        elif c.is_moe:
            out[p + "mlp.gate.weight"] = layer.router.detach()
            out[p + "mlp.experts.gate_up_proj"] = full(layer.w_gate_up)
            out[p + "mlp.experts.down_proj"] = full(layer.w_down)
            if layer.w_shared_gate_up is not None:
                g, u = full(layer.w_shared_gate_up).chunk(2, 0)
                out[p + "mlp.shared_expert.gate_proj.weight"] = g
                out[p + "mlp.shared_expert.up_proj.weight"] = u
                out[p + "mlp.shared_expert.down_proj.weight"] = full(layer.w_shared_down)
                out[p + "mlp.shared_expert_gate.weight"] = layer.shared_gate.detach()
        elif c.model_type == "phi3":
            out[p + "mlp.gate_up_proj.weight"] = full(layer.w_gate_up)
            out[p + "mlp.down_proj.weight"] = _unrotated_down(layer, full(layer.w_down))
        else:
            g, u = full(layer.w_gate_up).chunk(2, 0)
            out[p + "mlp.gate_proj.weight"] = g
            out[p + "mlp.up_proj.weight"] = u
            out[p + "mlp.down_proj.weight"] = _unrotated_down(layer, full(layer.w_down))
    return {k: v.clone() for k, v in out.items()} if copy else out


def _unrotated_down(layer, weight: torch.Tensor) -> torch.Tensor:
    """``w_down`` as a model without the online Hadamard rotation needs it: the rotate technique stores ``W H`` and
    rotates the input online; ``H`` (block-diagonal normalized Sylvester) is its own inverse, so ``W = (W H) H``."""
    block = getattr(layer, "down_hadamard", 0)
    if not block:
        return weight
    from ..ops import reference

    return reference.hadamard(weight.float(), block).to(weight.dtype)
