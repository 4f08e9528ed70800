"""Field checks shared by the configuration dataclasses (behaviour of ``src/economize/validation.py``)."""

from __future__ import annotations

import math
import warnings
from collections.abc import Collection, Iterable, Mapping

from .errors import ConfigError, UnknownFieldWarning

__all__ = [
    "check_choice",
    "check_indices",
    "check_non_negative",
    "check_positive",
    "check_probability",
    "check_unit_interval",
    "is_positive_int",
    "known_fields",
]


def is_positive_int(value: object) -> bool:
    return isinstance(value, int) and not isinstance(value, bool) and value > 0


def check_positive(name: str, value: object) -> None:
    """Raise :class:`ConfigError` unless ``value`` is a number > 0 (booleans are not numbers here)."""
    if isinstance(value, bool) or not isinstance(value, (int, float)) or not value > 0 or not math.isfinite(value):
        raise ConfigError(f"{name} must be positive, got {value!r}")


def check_non_negative(name: str, value: object) -> None:
    if isinstance(value, bool) or not isinstance(value, (int, float)) or not value >= 0 or not math.isfinite(value):
        raise ConfigError(f"{name} must be non-negative, got {value!r}")


def check_unit_interval(name: str, value: object, *, closed_low: bool = False, closed_high: bool = False) -> None:
    """``value`` in (0, 1), with either end included on request."""
    if isinstance(value, bool) or not isinstance(value, (int, float)):
        raise ConfigError(f"{name} must be a number in the unit interval, got {value!r}")
    low_ok = value >= 0 if closed_low else value > 0
    high_ok = value <= 1 if closed_high else value < 1
    if not (low_ok and high_ok):
        lo, hi = "[" if closed_low else "(", "]" if closed_high else ")"
        raise ConfigError(f"{name} must lie in {lo}0, 1{hi}, got {value!r}")


def check_probability(name: str, value: object) -> None:
    check_unit_interval(name, value, closed_low=True, closed_high=True)


def check_choice(name: str, value: object, choices: Collection[object]) -> None:
    if value not in choices:
        raise ConfigError(f"{name} must be one of {sorted(map(str, choices))}, got {value!r}")


def check_indices(name: str, values: Iterable[int], *, allow_empty: bool = True) -> None:
    values = list(values)
    if not values and not allow_empty:
        raise ConfigError(f"{name} must not be empty")
    if any(isinstance(v, bool) or not isinstance(v, int) or v < 0 for v in values):
        raise ConfigError(f"{name} must hold non-negative integers, got {values!r}")
    if len(set(values)) != len(values):
        raise ConfigError(f"{name} holds repeated entries: {values!r}")


def known_fields(owner: str, data: Mapping[str, object], known: set[str]) -> dict[str, object]:
    """The entries of ``data`` whose key is in ``known``; the others are dropped with an
    :class:`~economize_b200.errors.UnknownFieldWarning` (a config saved by a newer release)."""
    unknown = sorted(set(data) - known)
    if unknown:
        warnings.warn(f"{owner}: ignoring unknown fields {unknown}", UnknownFieldWarning, stacklevel=3)
    return {k: v for k, v in data.items() if k in known}
