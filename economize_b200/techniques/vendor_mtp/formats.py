"""Reading and writing the MTP modules shipped inside model checkpoints (economize
``techniques/vendor_mtp/formats.py``: ``state_from_vendor``, ``state_to_vendor``, ``mtp_settings``,
``VendorMTPFormat``).

The module's decoder block is this engine's draft layer: a pre-norm attention block (q/k/v projections, optionally
biased, fused into one GEMM) with a SwiGLU MLP. Vendor blocks of that shape load (MiMo's Qwen2 block, and dense
modules in any registered layout); blocks with multi-head latent attention, q/k norms, gated attention outputs or
routed experts (the DeepSeek-V3, GLM-4.5 and Qwen3-Next modules as released) are refused with the names that do
not fit, instead of being loaded partially. FP8 weights with block scales (``weight_scale_inv``, the DeepSeek-V3
and GLM-4.5 releases) are dequantized on load.
"""

from __future__ import annotations

import json
from collections.abc import Mapping
from pathlib import Path

import torch

from ...errors import CheckpointFormatError
from .families import MTP_FAMILIES, MTPFamily, family_for

__all__ = ["VendorMTPFormat", "dequantize_fp8_blocks", "mtp_settings", "state_from_vendor", "state_to_vendor"]

#: vendor block leaves -> this technique's parameter (the block's own norms and unfused projections)
_BLOCK = {"input_layernorm.weight": "input_norm", "post_attention_layernorm.weight": "layer.post_norm",
          "self_attn.o_proj.weight": "layer.wo", "mlp.down_proj.weight": "layer.w_down"}
#: vendor leaves fused into one parameter, in the fused order
_FUSED = {"layer.wqkv": ("self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight"),
          "layer.bqkv": ("self_attn.q_proj.bias", "self_attn.k_proj.bias", "self_attn.v_proj.bias"),
          "layer.w_gate_up": ("mlp.gate_proj.weight", "mlp.up_proj.weight")}


def dequantize_fp8_blocks(tensors: Mapping[str, torch.Tensor], block: tuple[int, int] = (128, 128)
                          ) -> dict[str, torch.Tensor]:
    """Replace every fp8 ``*.weight`` that has a ``*.weight_scale_inv`` companion by ``weight * scale`` (one scale
    per ``block`` tile, the DeepSeek-V3 release format), in bf16; the scales are dropped."""
    out: dict[str, torch.Tensor] = {}
    for key, value in tensors.items():
        if key.endswith(".weight_scale_inv"):
            continue
        scale = tensors.get(key + "_scale_inv") if key.endswith(".weight") else None
        if scale is not None:
            rows, cols = value.shape
            s = scale.float().repeat_interleave(block[0], 0)[:rows].repeat_interleave(block[1], 1)[:, :cols]
            value = (value.float() * s).to(torch.bfloat16)
        elif value.dtype in (torch.float8_e4m3fn, torch.float8_e5m2):
            raise CheckpointFormatError(f"{key} is fp8 without a weight_scale_inv companion")
        out[key] = value
    return out


def _family(name: str) -> MTPFamily:
    if name not in MTP_FAMILIES:
        raise CheckpointFormatError(f"unknown MTP family {name!r}; registered: {MTP_FAMILIES.names()}")
    return MTP_FAMILIES.get(name)


def _module_state(leaves: Mapping[str, torch.Tensor], family: str, spec: MTPFamily) -> dict[str, torch.Tensor]:
    """One module's technique state from its vendor leaves (block and own parameters)."""
    own = {v + ".weight": k for k, v in spec.own_names.items()}
    state: dict[str, torch.Tensor] = {}
    used: set[str] = set()
    for leaf, value in leaves.items():
        if leaf.startswith(spec.skipped):
            used.add(leaf)
        elif leaf in own:
            state[own[leaf]] = value
            used.add(leaf)
        elif leaf in _BLOCK:
            state[_BLOCK[leaf]] = value
            used.add(leaf)
    for ours, parts in _FUSED.items():
        present = [p for p in parts if p in leaves]
        if not present:
            continue
        if len(present) != len(parts):
            raise CheckpointFormatError(f"{family} MTP block: {sorted(set(parts) - set(present))} missing")
        state[ours] = torch.cat([leaves[p] for p in parts], 0)
        used.update(parts)
    foreign = sorted(set(leaves) - used)
    if foreign:
        raise CheckpointFormatError(
            f"the {family} MTP block has tensors this engine's draft layer (pre-norm attention with fused q/k/v and "
            f"a SwiGLU MLP) cannot hold: {foreign[:6]}{' ...' if len(foreign) > 6 else ''}")
    return state


def state_from_vendor(tensors: Mapping[str, torch.Tensor], family: str, num_layers: int,
                      fp8_block: tuple[int, int] = (128, 128)) -> list[dict[str, torch.Tensor]]:
    """The technique state of every MTP module in a checkpoint's tensors (other tensors are ignored).

    Raises:
        CheckpointFormatError: Unknown family, no module tensors, or a block this engine cannot hold.
    """
    spec = _family(family)
    owned = dequantize_fp8_blocks({k: v for k, v in tensors.items() if spec.owns(k, num_layers)}, fp8_block)
    modules: dict[int, dict[str, torch.Tensor]] = {}
    shared: dict[str, torch.Tensor] = {}
    for key, value in owned.items():
        where = spec.locate(key, num_layers)
        if where is not None:
            modules.setdefault(where[0], {})[where[1]] = value
        else:
            shared[spec.shared_leaf(key)] = value
    if not modules:
        raise CheckpointFormatError(f"no {family} MTP module tensors found")
    if sorted(modules) != list(range(len(modules))):
        raise CheckpointFormatError(f"{family} MTP modules {sorted(modules)} are not numbered 0..{len(modules) - 1}")
    return [_module_state({**shared, **modules[i]}, family, spec) for i in range(len(modules))]


def state_to_vendor(states: list[Mapping[str, torch.Tensor]], family: str, num_layers: int,
                    heads: tuple[int, int, int]) -> dict[str, torch.Tensor]:
    """Vendor tensors of module states (inverse of :func:`state_from_vendor`); ``heads`` = (query heads, KV heads,
    head dim) splits the fused projections.

    Raises:
        CheckpointFormatError: The family shares module parameters (Qwen) but the modules' values differ.
    """
    spec = _family(family)
    hq, hkv, hd = heads
    out: dict[str, torch.Tensor] = {}
    block_names = {v: k for k, v in _BLOCK.items()}
    for i, state in enumerate(states):
        base = spec.module_prefix(i, num_layers)
        for ours, value in state.items():
            value = value.detach()
            if ours in spec.own_names:
                name = (spec.shared_prefix or base) + spec.own_names[ours] + ".weight"
                if name in out and not torch.equal(out[name], value):
                    raise CheckpointFormatError(f"the {family} layout shares {name!r}, but the modules differ")
                out[name] = value
            elif ours in block_names:
                out[base + block_names[ours]] = value
            elif ours in ("layer.wqkv", "layer.bqkv"):
                for leaf, part in zip(_FUSED[ours], value.split([hq * hd, hkv * hd, hkv * hd], 0)):
                    out[base + leaf] = part
            elif ours == "layer.w_gate_up":
                for leaf, part in zip(_FUSED[ours], value.chunk(2, 0)):
                    out[base + leaf] = part
    return out


def _text(raw: Mapping) -> Mapping:
    text = raw.get("text_config")
    return {**raw, **text} if isinstance(text, dict) else raw


def mtp_settings(raw: Mapping) -> tuple[str | None, int, int]:
    """``(family, num_layers, modules)`` of a ``config.json`` (``modules`` 0: no MTP; ``family`` None: no
    registered family lists its ``model_type``)."""
    cfg = _text(raw)
    modules = int(cfg.get("num_nextn_predict_layers") or cfg.get("mtp_num_hidden_layers") or 0)
    return family_for(str(cfg.get("model_type", ""))), int(cfg.get("num_hidden_layers", 0) or 0), modules


def _fp8_block(raw: Mapping) -> tuple[int, int]:
    q = _text(raw).get("quantization_config") or {}
    b = q.get("weight_block_size") if isinstance(q, dict) else None
    return (int(b[0]), int(b[1])) if isinstance(b, list) and len(b) == 2 else (128, 128)


class VendorMTPFormat:
    """A model directory whose ``config.json`` declares MTP modules (``num_nextn_predict_layers`` or
    ``mtp_num_hidden_layers``) and whose safetensors hold them; read as a ``vendor_mtp`` technique."""

    @staticmethod
    def _config(path: Path) -> dict | None:
        try:
            raw = json.loads((path / "config.json").read_text())
        except (OSError, ValueError):
            return None
        return raw if isinstance(raw, dict) else None

    @staticmethod
    def _files(path: Path) -> list[Path]:
        index = path / "model.safetensors.index.json"
        if index.is_file():
            names = set(json.loads(index.read_text()).get("weight_map", {}).values())
            return [path / n for n in sorted(names)]
        return sorted(path.glob("*.safetensors"))

    def detect(self, path: Path) -> bool:
        raw = self._config(Path(path))
        return raw is not None and mtp_settings(raw)[2] > 0 and bool(self._files(Path(path)))

    def read(self, path: Path):
        from safetensors import safe_open

        from ...core.serialization import Checkpoint
        from . import VendorMTPConfig

        path = Path(path)
        raw = self._config(path)
        if raw is None:
            raise CheckpointFormatError(f"{path} has no readable config.json")
        family, num_layers, modules = mtp_settings(raw)
        if modules < 1:
            raise CheckpointFormatError(f"{path / 'config.json'} declares no MTP module")
        if family is None:
            raise CheckpointFormatError(f"{path / 'config.json'}: no registered MTP family lists model_type "
                                        f"{_text(raw).get('model_type')!r}; registered: {MTP_FAMILIES.names()}")
        spec = MTP_FAMILIES.get(family)
        tensors: dict[str, torch.Tensor] = {}
        for file in self._files(path):
            with safe_open(str(file), framework="pt") as handle:
                for key in handle.keys():  # noqa: SIM118 (the handle is not iterable)
                    if spec.owns(key, num_layers):
                        tensors[key] = handle.get_tensor(key)
        states = state_from_vendor(tensors, family, num_layers, _fp8_block(raw))
        if len(states) != modules:
            raise CheckpointFormatError(f"config.json declares {modules} MTP modules, the weights hold {len(states)}")
        if modules > 1:
            raise CheckpointFormatError(f"{modules} chained MTP modules: this engine drafts with one module")
        return Checkpoint([VendorMTPConfig(family=family)], {"vendor_mtp": states[0]}, None,
                          raw.get("_name_or_path") or None, {"source": str(path)})


def _register() -> None:
    from ...core.serialization import FORMATS

    if "vendor_mtp" not in FORMATS:
        FORMATS.register("vendor_mtp", VendorMTPFormat())


_register()
