"""All-or-nothing attach: what ``apply`` undoes when a technique fails part way (economize ``core/recipe.py:207-227``
and ``techniques/_weights/transaction.py``).

``apply`` attaches techniques one by one. When one raises, every technique attached before it is detached in reverse
order and the engine model returns to the state it had before the first attach, so the caller's model is not left
half-transformed. Two kinds of state are recorded before a weight-rewriting technique attaches:

* structure, always and cheaply: every module's parameter, buffer and submodule tables, its other attributes
  (weight objects a technique installs in place of a parameter, layer lists, flags), every parameter's ``.data``
  tensor and the model config. Restoring them undoes techniques that replace tensors or modules;
* contents, for the tensors a technique mutates in place (``Technique.inplace_targets``: AWQ / SmoothQuant scale
  folding, pruning masks written into a weight): copies in host memory, taken only when they fit a quarter of the
  host's available memory. Otherwise the error notes that those tensors may have changed and the model must be
  reloaded.

The failing error propagates unchanged, with notes (``BaseException.add_note``) on anything that could not be
undone.
"""

from __future__ import annotations

import copy
from dataclasses import dataclass, field

import torch
from torch import nn

__all__ = ["AttachTransaction", "StructureSnapshot"]

_TABLES = ("_parameters", "_buffers", "_modules")


@dataclass
class StructureSnapshot:
    """References to everything a tensor- or module-replacing transform changes (no tensor is copied)."""

    modules: list[tuple[nn.Module, dict[str, object], dict[str, dict]]] = field(default_factory=list)
    data: list[tuple[nn.Parameter, torch.Tensor]] = field(default_factory=list)
    config: object = None

    @classmethod
    def take(cls, model: nn.Module) -> StructureSnapshot:
        snap = cls()
        for module in model.modules():
            plain = {k: v for k, v in vars(module).items() if k not in _TABLES}
            tables = {name: dict(getattr(module, name)) for name in _TABLES}
            snap.modules.append((module, plain, tables))
        snap.data = [(p, p.data) for p in model.parameters()]
        config = getattr(model, "config", None)
        snap.config = copy.copy(config) if config is not None else None
        return snap

    def restore(self, model: nn.Module) -> None:
        for module, plain, tables in self.modules:
            for key in [k for k in vars(module) if k not in _TABLES and k not in plain]:
                delattr(module, key)  # attributes a transform added
            vars(module).update(plain)
            for name, table in tables.items():
                current = getattr(module, name)
                current.clear()
                current.update(table)
        for p, data in self.data:
            p.data = data
        if self.config is not None and getattr(model, "config", None) is not None:
            vars(model.config).update(vars(self.config))


@dataclass
class _ContentSnapshot:
    saved: list[tuple[torch.Tensor, torch.Tensor]] = field(default_factory=list)
    skipped: int = 0

    @classmethod
    def take(cls, tensors: list[torch.Tensor]) -> _ContentSnapshot:
        snap = cls()
        unique = list({id(t): t for t in tensors if isinstance(t, torch.Tensor)}.values())
        need = sum(t.numel() * t.element_size() for t in unique)
        if need > _host_budget():
            snap.skipped = len(unique)
            return snap
        snap.saved = [(t, t.detach().to("cpu", copy=True)) for t in unique]
        return snap

    def restore(self) -> None:
        with torch.no_grad():
            for t, host in self.saved:
                t.copy_(host.to(t.device))


def _host_budget() -> int:
    """A quarter of the host memory available now (bytes); unlimited when it cannot be read."""
    try:
        import psutil

        return int(psutil.virtual_memory().available // 4)
    except Exception:  # noqa: BLE001 - without psutil the copies are taken
        return 1 << 62


class AttachTransaction:
    """The undo log of one ``apply`` call on an engine model."""

    def __init__(self, model: nn.Module) -> None:
        self.model = model
        self.attached: list = []
        self._structure: StructureSnapshot | None = None
        self._contents: list[_ContentSnapshot] = []

    def before_weights(self, technique) -> None:
        """Record the model's state before a weight-rewriting ``technique`` attaches."""
        if self._structure is None:
            self._structure = StructureSnapshot.take(self.model)
        self._contents.append(_ContentSnapshot.take(list(technique.inplace_targets())))

    def attached_ok(self, technique) -> None:
        self.attached.append(technique)

    def roll_back(self, failed, error: BaseException) -> None:
        """Detach what was attached (newest first) and restore the recorded model state; notes on ``error`` say
        what could not be undone."""
        from .technique import Capability

        for technique in reversed(self.attached):
            if Capability.WEIGHTS in technique.capabilities:
                continue  # undone by the snapshots below
            try:
                technique.detach()
            except Exception as detach_error:  # noqa: BLE001 - the original error stays the one raised
                error.add_note(f"economize_b200: detaching {technique.name!r} during the roll-back failed: "
                               f"{detach_error!r}")
        skipped = sum(c.skipped for c in self._contents)
        for contents in reversed(self._contents):
            contents.restore()
        if self._structure is not None:
            self._structure.restore(self.model)
        if skipped:
            error.add_note(f"economize_b200: {skipped} tensor(s) that a weight transform changes in place were too "
                           "large to copy to host memory before it ran and may have changed; reload the model")
        name = getattr(failed, "name", None)
        if name is not None:
            error.add_note(f"economize_b200: attaching {name!r} failed; every technique attached before it was "
                           "detached and the model restored")
