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


# ---- the official checkpoint layout as a registered format ------------------------------------------------------
def _flat(config: dict) -> dict:
    layer = config.get("transformer_layer_config")
    if not isinstance(layer, dict):
        return config
    return {**layer, **{k: v for k, v in config.items() if k != "transformer_layer_config" and v is not None}}


def config_from_official(config: dict):
    """The :class:`Eagle3Config` of an official / SpecForge / vLLM-speculators EAGLE-3 ``config.json``."""
    from ...errors import CheckpointFormatError
    from .config import Eagle3Config

    config = _flat(config)
    eagle = dict(config.get("eagle_config") or {})
    for flag in ("norm_before_fc", "fc_norm", "norm_output", "input_norm"):
        if config.get(flag) or eagle.get(flag):
            raise CheckpointFormatError(f"the EAGLE-3 option {flag!r} is not supported")
    hidden = int(config["hidden_size"])
    target = config.get("target_hidden_size")
    if target is not None and int(target) != hidden:
        raise CheckpointFormatError(f"a draft width {hidden} other than the model's ({target}) is not supported")
    heads = int(config["num_attention_heads"])
    vocab, draft_vocab = config.get("vocab_size"), config.get("draft_vocab_size")
    aux = eagle.get("eagle_aux_hidden_state_layer_ids") or config.get("eagle_aux_hidden_state_layer_ids")
    return Eagle3Config(
        aux_layers=tuple(int(i) for i in aux) if aux else None,
        head="own",
        draft_vocab=int(draft_vocab) if draft_vocab is not None and vocab is not None and draft_vocab < vocab else None,
        intermediate_size=int(config["intermediate_size"]),
        num_heads=heads,
        num_kv_heads=int(config.get("num_key_value_heads") or heads),
        head_dim=int(config.get("head_dim") or hidden // heads),
        attention_bias=bool(config.get("attention_bias", False)),
        rope_theta=float(config.get("rope_theta", 10000.0)),
        rope_scaling=config.get("rope_scaling"),
        rms_norm_eps=float(config.get("rms_norm_eps", 1e-6)),
        norm_before_residual=bool(config.get("norm_before_residual", eagle.get("norm_before_residual", False))),
    )


class Eagle3Format:
    """Official EAGLE-3 heads (SafeAILab, SpecForge, vLLM speculators): ``config.json`` + ``model.safetensors``
    (or ``pytorch_model.bin``) with ``midlayer.*`` / ``layers.0.*``, ``fc``, ``norm``, ``lm_head``, ``d2t``, ``t2d``."""

    files = ("model.safetensors", "pytorch_model.bin")

    def detect(self, path) -> bool:
        import json
        from pathlib import Path

        path = Path(path)
        cfg = path / "config.json"
        if not cfg.is_file() or not any((path / f).is_file() for f in self.files):
            return False
        data = json.loads(cfg.read_text())
        arch = " ".join(data.get("architectures") or [])
        return "draft_vocab_size" in _flat(data) or "Eagle3" in arch or "eagle3" in str(data.get("speculators_model_type", ""))

    def read(self, path):
        import json
        from pathlib import Path

        from ...core.serialization import Checkpoint

        path = Path(path)
        config = json.loads((path / "config.json").read_text())
        if (path / "model.safetensors").is_file():
            from safetensors.torch import load_file

            state = load_file(str(path / "model.safetensors"))
        else:
            state = torch.load(path / "pytorch_model.bin", map_location="cpu", weights_only=True)
        state = {k: v for k, v in state.items() if not k.startswith("embed_tokens")}
        renamed = {}
        for key, value in state.items():
            for prefix in ("midlayer.", "layers.0."):
                if key.startswith(prefix):
                    key = "layer." + key[len(prefix):]
            renamed[key] = value
        cfg = config_from_official(config)
        base = config.get("base_model_name_or_path") or ((config.get("speculators_config") or {}).get("verifier")
                                                         or {}).get("name_or_path")
        return Checkpoint([cfg], {"eagle3": renamed}, None, base, {"base_model": base})


def _register() -> None:
    from ...core.serialization import FORMATS

    if "eagle3" not in FORMATS:
        FORMATS.register("eagle3", Eagle3Format())


_register()
