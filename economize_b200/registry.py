"""Named registries with plugin discovery through entry points (behaviour of ``src/economize/registry.py:43-150``).

Every variation point of the framework (techniques, verifiers, draft policies, checkpoint formats, GEMM and
attention kernels) is a :class:`Registry`. A lookup miss scans the registry's entry-point group once, so a plugin
package can add entries without touching this code.
"""

from __future__ import annotations

import importlib
import logging
import pkgutil
from collections.abc import Callable, Iterable, Iterator
from importlib import metadata
from typing import Generic, TypeVar

from .errors import DuplicateNameError, UnknownNameError

__all__ = ["Registry", "import_submodules"]

T = TypeVar("T")
log = logging.getLogger(__name__)


class Registry(Generic[T]):
    """A mapping from names to objects of one kind.

    Args:
        kind: What the entries are, for messages ("technique", "verifier", ...).
        entry_point_group: Entry-point group searched on the first miss (``None``: no plugins).
    """

    def __init__(self, kind: str, entry_point_group: str | None = None) -> None:
        self.kind = kind
        self.entry_point_group = entry_point_group
        #: sources that failed to load (name -> reason); shown in the error of an unknown name
        self.unavailable: dict[str, str] = {}
        self._items: dict[str, T] = {}
        self._scanned = entry_point_group is None

    def register(self, name: str, obj: T | None = None, *, override: bool = False):
        """Register ``obj`` as ``name``; without ``obj`` return a decorator that does so."""

        def put(value: T) -> T:
            old = self._items.get(name)
            if old is not None and old is not value and not override:
                raise DuplicateNameError(f"{self.kind} {name!r} already registered ({old!r}); use override=True")
            self._items[name] = value
            return value

        if obj is None:
            return put
        return put(obj)

    def unregister(self, name: str) -> T:
        self._scan()
        if name not in self._items:
            raise self._missing(name)
        return self._items.pop(name)

    def get(self, name: str) -> T:
        if name not in self._items:
            self._scan()
        if name not in self._items:
            raise self._missing(name)
        return self._items[name]

    def names(self) -> list[str]:
        self._scan()
        return sorted(self._items)

    def items(self) -> list[tuple[str, T]]:
        return [(n, self._items[n]) for n in self.names()]

    def __contains__(self, name: object) -> bool:
        if name not in self._items:
            self._scan()
        return name in self._items

    def __iter__(self) -> Iterator[str]:
        return iter(self.names())

    def __len__(self) -> int:
        return len(self.names())

    def __repr__(self) -> str:
        return f"Registry({self.kind!r}, {sorted(self._items)})"

    def _missing(self, name: str) -> UnknownNameError:
        known = ", ".join(map(repr, sorted(self._items))) or "none"
        text = f"unknown {self.kind} {name!r}; registered: {known}"
        if self.unavailable:
            text += "; failed to load: " + "; ".join(f"{k}: {v}" for k, v in sorted(self.unavailable.items()))
        return UnknownNameError(text)

    def _scan(self) -> None:
        if self._scanned:
            return
        self._scanned = True
        for ep in metadata.entry_points(group=self.entry_point_group):
            if ep.name in self._items:
                continue
            try:
                self.register(ep.name, ep.load())
            except Exception as err:  # a broken plugin must not break the package
                log.warning("could not load %s plugin %r: %s", self.kind, ep.name, err)
                self.unavailable[ep.name] = f"{type(err).__name__}: {err}"


def import_submodules(package: str, path: Iterable[str], *, unavailable: dict[str, str] | None = None) -> list[str]:
    """Import every public subpackage of ``package`` so it registers its entries; failures are recorded in
    ``unavailable`` (when given) instead of raised."""
    done = []
    for info in pkgutil.iter_modules(path):
        if not info.ispkg or info.name.startswith("_"):
            continue
        try:
            importlib.import_module(f"{package}.{info.name}")
        except Exception as err:
            if unavailable is None:
                raise
            unavailable[info.name] = f"{type(err).__name__}: {err}"
            log.warning("%s.%s skipped: %s", package, info.name, err)
        else:
            done.append(info.name)
    return done
