"""PEFT interoperability (economize ``integrations/peft.py:1-310``).

* The LoRA of a technique in the PEFT adapter format. A technique whose parameters include low-rank adapters lists
  them by Hugging Face module name in ``lora_targets()`` (``EarlyExitConfig(adaptation="lora")``: the draft path's
  ``lm_head``). :func:`save_lora` writes them as ``adapter_config.json`` + ``adapter_model.safetensors``, loadable
  with ``PeftModel.from_pretrained(base, path)``; :func:`load_lora` reads such a folder back (also adapters trained
  with PEFT on the same modules).
* A PEFT adapter as part of the base: :func:`merge_adapter` folds a LoRA adapter folder into the target's weights
  (``W += alpha / r * B A`` per module, q/k/v and gate/up into the engine's fused projections), the equivalent of
  ``PeftModel.merge_and_unload()`` before ``economize_b200.apply``.

The file format is PEFT's (``base_model.model.<module>.lora_A.weight [r, in]``, ``lora_B.weight [out, r]``,
``r``, ``lora_alpha``, ``target_modules``), kept as PEFT writes it so that either side reads the other's files; PEFT
itself is not imported.
"""

from __future__ import annotations

import json
from pathlib import Path
from typing import Any

import torch

from ..errors import CheckpointFormatError, ConfigError

__all__ = ["load_lora", "lora_modules", "merge_adapter", "save_lora"]

_PREFIX = "base_model.model."


def lora_modules(model, technique: str | None = None) -> dict[str, Any]:
    """``{Hugging Face module name: LoRAWeight}`` of the LoRA-capable technique of ``model`` (``technique`` names it
    when several are attached)."""
    techniques = getattr(model, "techniques", None)
    if techniques is None:
        raise ConfigError("lora_modules takes an EfficientModel")
    capable = {n: techniques[n] for n in techniques.keys() if callable(getattr(techniques[n], "lora_targets", None))}
    capable = {n: t for n, t in capable.items() if t.lora_targets()}
    if technique is not None:
        if technique not in capable:
            raise ConfigError(f"technique {technique!r} has no LoRA adapters; LoRA-capable: {sorted(capable)}")
        return capable[technique].lora_targets()
    if len(capable) != 1:
        raise ConfigError(f"expected one technique with LoRA adapters, found {sorted(capable)}; pass technique=")
    return next(iter(capable.values())).lora_targets()


def save_lora(model, path: str | Path, technique: str | None = None, base_model: str | None = None) -> Path:
    """Write the technique's adapters as a PEFT LoRA adapter folder; returns the folder."""
    from safetensors.torch import save_file

    mods = lora_modules(model, technique)
    ranks = {int(w.a.shape[0]) for w in mods.values()}
    scales = {float(w.scale) for w in mods.values()}
    if len(ranks) != 1 or len(scales) != 1:
        raise ConfigError("PEFT's adapter config holds one rank and alpha; the adapters differ")
    r, scale = ranks.pop(), scales.pop()
    config = {"peft_type": "LORA", "task_type": "CAUSAL_LM", "r": r, "lora_alpha": scale * r, "lora_dropout": 0.0,
              "bias": "none", "fan_in_fan_out": False, "use_rslora": False,
              "target_modules": sorted({name.rsplit(".", 1)[-1] for name in mods}),
              "base_model_name_or_path": base_model, "inference_mode": True}
    tensors = {}
    for name, w in mods.items():
        tensors[f"{_PREFIX}{name}.lora_A.weight"] = w.a.detach().float().cpu().contiguous()
        tensors[f"{_PREFIX}{name}.lora_B.weight"] = w.b.detach().float().cpu().contiguous()
    out = Path(path)
    out.mkdir(parents=True, exist_ok=True)
    (out / "adapter_config.json").write_text(json.dumps(config, indent=2) + "\n")
    save_file(tensors, str(out / "adapter_model.safetensors"), metadata={"format": "pt"})
    return out


def _read_adapter(path: str | Path) -> tuple[dict[str, Any], dict[str, tuple[torch.Tensor, torch.Tensor]], float]:
    from safetensors.torch import load_file

    folder = Path(path)
    cfg_file, weights = folder / "adapter_config.json", folder / "adapter_model.safetensors"
    if not cfg_file.is_file() or not weights.is_file():
        raise CheckpointFormatError(f"{folder} is not a PEFT adapter folder (adapter_config.json and "
                                    "adapter_model.safetensors)")
    config = json.loads(cfg_file.read_text())
    if config.get("peft_type", "LORA") != "LORA":
        raise CheckpointFormatError(f"only LoRA adapters are read, got peft_type={config.get('peft_type')!r}")
    if config.get("use_dora") or config.get("fan_in_fan_out"):
        raise CheckpointFormatError("DoRA and fan_in_fan_out adapters are not supported")
    r = int(config["r"])
    alpha = float(config.get("lora_alpha", r))
    scale = alpha / (r ** 0.5) if config.get("use_rslora") else alpha / r
    state = load_file(str(weights))
    pairs: dict[str, list] = {}
    for key, t in state.items():
        name = key[len(_PREFIX):] if key.startswith(_PREFIX) else key
        for part, slot in ((".lora_A.weight", 0), (".lora_B.weight", 1)):
            if name.endswith(part):
                pairs.setdefault(name[: -len(part)], [None, None])[slot] = t
    bad = [m for m, (a, b) in pairs.items() if a is None or b is None]
    if bad:
        raise CheckpointFormatError(f"modules {bad} lack lora_A or lora_B")
    return config, {m: (a, b) for m, (a, b) in pairs.items()}, scale


@torch.no_grad()
def load_lora(model, path: str | Path, technique: str | None = None) -> None:
    """Load a PEFT LoRA adapter into the technique's adapters (same modules, rank and scale)."""
    mods = lora_modules(model, technique)
    _, pairs, scale = _read_adapter(path)
    missing = sorted(set(mods) - set(pairs))
    extra = sorted(set(pairs) - set(mods))
    if missing or extra:
        raise CheckpointFormatError(f"adapter modules differ: missing {missing}, unexpected {extra}")
    for name, w in mods.items():
        a, b = pairs[name]
        if tuple(a.shape) != tuple(w.a.shape) or tuple(b.shape) != tuple(w.b.shape):
            raise CheckpointFormatError(f"{name}: adapter shapes {tuple(a.shape)}/{tuple(b.shape)} differ from "
                                        f"{tuple(w.a.shape)}/{tuple(w.b.shape)}")
        w.a.copy_(a.to(w.a))
        w.b.copy_(b.to(w.b))
        w.scale = scale


@torch.no_grad()
def merge_adapter(model, path: str | Path) -> list[str]:
    """Fold a PEFT LoRA adapter of the target's decoder projections (and ``lm_head``) into its weights; returns the
    merged module names. Quantized projections are refused (merge before quantizing)."""
    lm = getattr(model, "model", model)
    c = lm.config
    _, pairs, scale = _read_adapter(path)
    slices = {"self_attn.q_proj": ("wqkv", 0, c.q_size), "self_attn.k_proj": ("wqkv", c.q_size, c.kv_size),
              "self_attn.v_proj": ("wqkv", c.q_size + c.kv_size, c.kv_size),
              "self_attn.o_proj": ("wo", 0, c.hidden_size),
              "mlp.gate_proj": ("w_gate_up", 0, c.intermediate_size),
              "mlp.up_proj": ("w_gate_up", c.intermediate_size, c.intermediate_size),
              "mlp.down_proj": ("w_down", 0, c.hidden_size)}
    merged = []
    for name, (a, b) in sorted(pairs.items()):
        delta = (b.double() @ a.double() * scale).float()
        if name in ("lm_head", "model.lm_head"):
            target, rows = lm.lm_head, slice(0, None)
            if target is None:
                raise ConfigError("the model ties its LM head to the embedding; an lm_head adapter cannot be merged")
        else:
            parts = name.split(".")
            if len(parts) < 5 or parts[0] != "model" or parts[1] != "layers":
                raise CheckpointFormatError(f"adapter module {name!r} is not a decoder projection or lm_head")
            layer = lm.layers[int(parts[2])]
            key = ".".join(parts[3:])
            if key not in slices:
                raise CheckpointFormatError(f"adapter module {name!r} is not a decoder projection")
            attr, start, size = slices[key]
            target, rows = getattr(layer, attr), slice(start, start + size)
        if not isinstance(target, torch.Tensor):
            raise ConfigError(f"{name}: the projection is not a dense tensor (quantized?); merge before quantizing")
        if tuple(delta.shape) != tuple(target[rows].shape):
            raise CheckpointFormatError(f"{name}: update {tuple(delta.shape)} does not match {tuple(target[rows].shape)}")
        target[rows] += delta.to(target.dtype)
        merged.append(name)
    return merged
