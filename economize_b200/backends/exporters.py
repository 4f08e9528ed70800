"""Drafter exporters: one drafter technique written as the folder one serving engine loads (economize
``backends/exporters.py:1-213``).

An exporter names the tensors and the ``config.json`` an engine expects for one technique; :func:`export_drafter`
writes them (``model.safetensors`` in the technique's dtype, ``d2t``/``t2d`` as int64/bool). Exporters are kept per
``"<backend>/<technique>"`` in :data:`EXPORTERS`, so a new engine or a new drafter is one registered class::

    @register_exporter("my_engine", "eagle3")
    class MyExporter(DrafterExporter):
        def config(self, technique, **options): ...
        def tensors(self, technique): ...
"""

from __future__ import annotations

import json
from pathlib import Path
from typing import Any

import torch

from ..errors import ConfigError, EconomizeError
from ..registry import Registry

__all__ = ["EXPORTERS", "DrafterExporter", "UnsupportedBackendError", "export_drafter", "exporter_for",
           "register_exporter"]


class UnsupportedBackendError(EconomizeError, NotImplementedError):
    """No exporter writes this technique for this backend."""


class DrafterExporter:
    """Base of an exporter: :meth:`config` and :meth:`tensors` of one technique instance."""

    technique_name: str = ""

    def config(self, technique: Any, **options: Any) -> dict[str, Any]:
        raise NotImplementedError

    def tensors(self, technique: Any) -> dict[str, torch.Tensor]:
        raise NotImplementedError

    def metadata(self) -> dict[str, str]:
        return {"format": "pt", "exporter": f"economize_b200/{self.technique_name}"}

    def export(self, technique: Any, path: str | Path, **options: Any) -> Path:
        from safetensors.torch import save_file

        out = Path(path)
        out.mkdir(parents=True, exist_ok=True)
        config = self.config(technique, **options)
        tensors = {k: v.detach().to("cpu").contiguous() for k, v in self.tensors(technique).items()}
        (out / "config.json").write_text(json.dumps(config, indent=2, sort_keys=True) + "\n")
        save_file(tensors, str(out / "model.safetensors"), metadata=self.metadata())
        return out


EXPORTERS: Registry[type[DrafterExporter]] = Registry("drafter exporter", "economize_b200.exporters")


def register_exporter(backend: str, technique: str, *, override: bool = False):
    """Class decorator: register an exporter under ``"<backend>/<technique>"``."""
    def add(cls: type[DrafterExporter]) -> type[DrafterExporter]:
        cls.technique_name = technique
        EXPORTERS.register(f"{backend}/{technique}", cls, override=override)
        return cls
    return add


def _techniques(model: Any) -> dict[str, Any]:
    techniques = getattr(model, "techniques", None)
    if techniques is None:
        raise ConfigError("export_drafter takes an EfficientModel (the result of economize_b200.apply)")
    return {name: techniques[name] for name in techniques.keys()}


def exporter_for(model: Any, backend: str, technique: str | None = None) -> tuple[DrafterExporter, Any]:
    """The exporter and the technique instance for ``model`` on ``backend`` (``technique``: which drafter, needed
    only when the model has several)."""
    techniques = _techniques(model)
    if technique is None:
        drafters = [n for n in techniques if f"{backend}/{n}" in EXPORTERS.names()]
        if not drafters:
            raise UnsupportedBackendError(f"no exporter for backend {backend!r} covers the model's techniques "
                                          f"{sorted(techniques)}; registered: {sorted(EXPORTERS.names())}")
        if len(drafters) > 1:
            raise ConfigError(f"the model has several exportable drafters {drafters}; pass technique=")
        technique = drafters[0]
    if technique not in techniques:
        raise ConfigError(f"the model has no technique {technique!r}; it has {sorted(techniques)}")
    key = f"{backend}/{technique}"
    if key not in EXPORTERS.names():
        raise UnsupportedBackendError(f"no exporter {key!r}; registered: {sorted(EXPORTERS.names())}")
    return EXPORTERS.get(key)(), techniques[technique]


def export_drafter(model: Any, path: str | Path, *, backend: str, technique: str | None = None,
                   **options: Any) -> Path:
    """Write ``model``'s drafter as the draft-model folder ``backend`` loads; returns the folder."""
    exporter, instance = exporter_for(model, backend, technique)
    return exporter.export(instance, path, **options)


def refuse_online_rotation(target, fmt: str) -> None:
    """Refuse to write a model whose down projections expect an online Hadamard rotation of their input (the
    ``rotate`` technique's ``online`` option): ``fmt`` files carry no such transform, so they would compute another
    function."""
    if any(getattr(layer, "down_hadamard", 0) for layer in target.layers):
        raise ConfigError(f"{fmt} files carry no online Hadamard rotation; export the model before rotate, or rotate "
                          "with online=()")
