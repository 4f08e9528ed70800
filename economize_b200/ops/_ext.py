"""Loader of the compiled sm_100a extension ``economize_b200._C``.

The extension is built in-tree (``python setup.py build_ext --inplace``, or ``__graft_entry__.build()``). CUDA
tensors always go to it: :func:`require` raises :class:`~economize_b200.errors.KernelUnavailableError` when it is
missing instead of falling back to PyTorch, so a GPU run can never pass on a silent eager path. CPU tensors use the
PyTorch implementations in :mod:`economize_b200.ops.reference` (the numerics oracle of the kernel tests).
With ``ECZ_CHECK=1`` in the environment the bounds-checked build ``economize_b200._C_check`` is loaded instead.
"""

from __future__ import annotations

import importlib
import os
from types import ModuleType

from ..errors import KernelUnavailableError

__all__ = ["available", "load_error", "require"]

_module: ModuleType | None = None
_error: str | None = None


def _load() -> ModuleType | None:
    global _module, _error
    if _module is not None or _error is not None:
        return _module
    try:
        import torch  # noqa: F401  (the extension links against libtorch)

        _module = importlib.import_module(module_name())
    except Exception as err:  # ImportError, or an undefined symbol of a stale build
        _error = f"{type(err).__name__}: {err}"
    return _module


def module_name() -> str:
    """``economize_b200._C``, or the bounds-checked build ``economize_b200._C_check`` when ``ECZ_CHECK=1``."""
    return "economize_b200._C_check" if os.environ.get("ECZ_CHECK") == "1" else "economize_b200._C"


def available() -> bool:
    """Whether the compiled extension imports."""
    return _load() is not None


def load_error() -> str | None:
    _load()
    return _error


def require() -> ModuleType:
    """The extension module; raises when it is missing (a CUDA tensor must never take a fallback path)."""
    module = _load()
    if module is None:
        raise KernelUnavailableError(f"{module_name()} is not built or failed to load ({_error})")
    return module
