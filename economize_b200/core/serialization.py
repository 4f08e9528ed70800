"""Technique checkpoints: ``save`` / ``read_checkpoint`` / ``attach`` / ``load`` / ``from_pretrained``.

The on-disk layout is economize's (``src/economize/core/serialization.py:83-580``): a folder with
``economize_config.json`` (schema version, the technique configurations as ``{"technique", "config"}`` entries, the
decoding options, the base model id and a teacher fingerprint) and ``economize_model.safetensors`` holding only the
techniques' tensors as ``<technique>.<name>``. Tensor names are economize's (each technique converts from its fused
engine layout), so checkpoints move between the two libraries. Further readable layouts (official EAGLE-3 heads,
Medusa heads, ...) register in :data:`FORMATS`; detection must be unambiguous.
"""

from __future__ import annotations

import hashlib
import json
import warnings
from abc import ABC, abstractmethod
from collections.abc import Mapping
from dataclasses import dataclass, field
from pathlib import Path
from typing import TYPE_CHECKING, Any

import torch
from torch import nn

from .._version import API_LEVEL, __version__
from ..decoding.config import DecodeConfig
from ..errors import CheckpointFormatError, ConfigError, TeacherMismatchWarning
from ..registry import Registry
from .technique import TECHNIQUES, TechniqueConfig

if TYPE_CHECKING:
    from .model import EfficientModel

__all__ = ["CONFIG_FILE", "FORMATS", "SCHEMA_VERSION", "WEIGHTS_FILE", "Checkpoint", "CheckpointFormat", "attach",
           "from_pretrained", "load", "nested_config", "nested_dict", "read_checkpoint", "save",
           "teacher_fingerprint"]

CONFIG_FILE = "economize_config.json"
WEIGHTS_FILE = "economize_model.safetensors"
SCHEMA_VERSION = 1


def nested_dict(config: TechniqueConfig) -> dict[str, Any]:
    return {"technique": config.technique, "config": config.to_dict()}


def nested_config(data: Mapping[str, Any] | TechniqueConfig) -> TechniqueConfig:
    if isinstance(data, TechniqueConfig):
        return data
    if set(data) != {"technique", "config"}:
        raise ConfigError(f"a technique entry needs the keys 'technique' and 'config', got {sorted(data)}")
    return TECHNIQUES.get(str(data["technique"])).config_class.from_dict(dict(data["config"]))


@dataclass
class Checkpoint:
    """What a format reads: configurations, tensors per technique (economize names), decoding, metadata."""

    configs: list[TechniqueConfig]
    states: dict[str, dict[str, torch.Tensor]]
    decoding: DecodeConfig | None = None
    base_model: str | None = None
    meta: dict[str, Any] = field(default_factory=dict)


class CheckpointFormat(ABC):
    @abstractmethod
    def detect(self, path: Path) -> bool:
        """Whether ``path`` holds a checkpoint of this format."""

    @abstractmethod
    def read(self, path: Path) -> Checkpoint:
        """Read the checkpoint at ``path``."""


FORMATS: Registry[CheckpointFormat] = Registry("checkpoint format", "economize_b200.formats")


def _migrate(meta: dict[str, Any]) -> dict[str, Any]:
    version = int(meta.get("schema_version", 0))
    if version > SCHEMA_VERSION:
        raise CheckpointFormatError(f"checkpoint schema version {version} is newer than this release reads "
                                    f"({SCHEMA_VERSION})")
    meta = dict(meta)
    meta["schema_version"] = SCHEMA_VERSION  # version 0 (no field) has the layout of version 1
    return meta


class EconomizeFormat(CheckpointFormat):
    config_file = CONFIG_FILE
    weights_file = WEIGHTS_FILE

    def detect(self, path: Path) -> bool:
        return (path / self.config_file).is_file()

    def read(self, path: Path) -> Checkpoint:
        from safetensors.torch import load_file

        meta = _migrate(json.loads((path / self.config_file).read_text()))
        entries = meta["techniques"]
        configs = [nested_config(e) for e in entries]
        states: dict[str, dict[str, torch.Tensor]] = {str(e["technique"]): {} for e in entries}
        weights = path / self.weights_file
        if weights.exists():
            for key, value in load_file(str(weights)).items():
                name, _, rest = key.partition(".")
                if name not in states:
                    raise CheckpointFormatError(f"tensor {key!r} belongs to no technique in {self.config_file}")
                states[name][rest] = value
        decoding = DecodeConfig.from_dict(meta["decoding"]) if meta.get("decoding") else None
        return Checkpoint(configs, states, decoding, meta.get("base_model"), meta)


class LegacyEffkitFormat(EconomizeFormat):
    """Checkpoints written under the library's earlier name (same layout, other file names)."""

    config_file = "effkit_config.json"
    weights_file = "effkit_model.safetensors"


FORMATS.register("economize", EconomizeFormat())
FORMATS.register("effkit", LegacyEffkitFormat())


def teacher_fingerprint(model: nn.Module, samples: int = 64) -> str:
    """SHA-256 over the base model's parameter names, shapes and ``samples`` evenly spaced values of each (in
    Hugging Face names, so a fused engine model and its ``transformers`` twin agree)."""
    from ..models.llama import CausalLM

    if isinstance(model, CausalLM):
        tensors = model.hf_state_dict(copy=False)
    else:
        tensors = {k: v for k, v in model.state_dict().items()}
    h = hashlib.sha256()
    for name in sorted(tensors):
        t = tensors[name].detach()
        h.update(name.encode())
        h.update(str(tuple(t.shape)).encode())
        flat = t.reshape(-1)
        if flat.numel():
            idx = torch.linspace(0, flat.numel() - 1, min(samples, flat.numel()), device=flat.device).long()
            h.update(flat[idx].float().cpu().numpy().tobytes())
    return h.hexdigest()


def save(model: EfficientModel, path: str | Path, *, extra_meta: Mapping[str, Any] | None = None) -> None:
    """Write the techniques' configurations and tensors (never the base weights) in economize's layout."""
    from safetensors.torch import save_file

    path = Path(path)
    base = model.base_model
    meta: dict[str, Any] = {
        "schema_version": SCHEMA_VERSION,
        "economize_version": API_LEVEL,
        "economize_b200_version": __version__,
        "base_model": getattr(getattr(base, "config", None), "_name_or_path", None),
        "teacher_fingerprint": model.teacher_digest or teacher_fingerprint(model.model),
        "techniques": [nested_dict(t.config) for t in model.techniques.values()],
        "decoding": model.decoding.to_dict(),
    }
    meta.update(extra_meta or {})
    tensors = {f"{t.name}.{k}": v.detach().cpu().contiguous().clone()
               for t in model.techniques.values() for k, v in t.export_state().items()}
    path.mkdir(parents=True, exist_ok=True)
    (path / CONFIG_FILE).write_text(json.dumps(meta, indent=2) + "\n")
    save_file(tensors, str(path / WEIGHTS_FILE))


def read_checkpoint(path: str | Path, format: str | None = None) -> Checkpoint:
    """Read a checkpoint, detecting its format unless ``format`` names one (exactly one format must match)."""
    path = Path(path)
    if format is not None:
        return FORMATS.get(format).read(path)
    matches = [n for n in FORMATS.names() if FORMATS.get(n).detect(path)]
    if len(matches) > 1:
        raise CheckpointFormatError(f"{path} matches several checkpoint formats {matches}; pass format=")
    if not matches:
        raise CheckpointFormatError(f"no registered checkpoint format recognizes {path}; formats: {FORMATS.names()}")
    return FORMATS.get(matches[0]).read(path)


def attach(model: nn.Module, checkpoint: Checkpoint, decoding: DecodeConfig | None = None, *,
           calibration: Any = None, check_teacher: bool = True) -> EfficientModel:
    """Apply the checkpoint's techniques to ``model``, loading their tensors before they attach."""
    from .model import build_model

    result = build_model(model, checkpoint.configs, decoding=decoding or checkpoint.decoding,
                         calibration=calibration, states=checkpoint.states)
    recorded = checkpoint.meta.get("teacher_fingerprint")
    if check_teacher and recorded and checkpoint.meta.get("economize_b200_version"):
        if (result.teacher_digest or teacher_fingerprint(result.model)) != recorded:
            warnings.warn("the base model's weights differ from those the checkpoint was saved with",
                          TeacherMismatchWarning, stacklevel=2)
    return result


def load(model: nn.Module, path: str | Path, *, format: str | None = None, decoding: DecodeConfig | None = None,
         calibration: Any = None, check_teacher: bool = True) -> EfficientModel:
    """Attach the techniques stored at ``path`` (any registered format) to ``model``."""
    return attach(model, read_checkpoint(path, format), decoding, calibration=calibration,
                  check_teacher=check_teacher)


def from_pretrained(path: str | Path, base_model: str | nn.Module | None = None, *, format: str | None = None,
                    decoding: DecodeConfig | None = None, calibration: Any = None, check_teacher: bool = True,
                    **model_kwargs: Any) -> EfficientModel:
    """Load the base model the checkpoint names (or ``base_model``: a path, Hub id or module) with
    ``transformers`` and attach the techniques."""
    checkpoint = read_checkpoint(path, format)
    if isinstance(base_model, nn.Module):
        base = base_model
    else:
        name = base_model or checkpoint.base_model or checkpoint.meta.get("base_model")
        if not name:
            raise CheckpointFormatError("the checkpoint names no base model; pass base_model=")
        import transformers

        base = transformers.AutoModelForCausalLM.from_pretrained(name, **model_kwargs)
    return attach(base, checkpoint, decoding, calibration=calibration, check_teacher=check_teacher)
