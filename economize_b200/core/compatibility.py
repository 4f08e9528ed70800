"""Which techniques combine: ``compatible``, ``incompatibility``, ``compatibility_matrix`` (economize
``src/economize/core/compatibility.py:45-143``), decided from the technique classes alone (no model needed)."""

from __future__ import annotations

from collections.abc import Iterable

from .technique import TECHNIQUES, Capability, Family, Technique, TechniqueConfig

__all__ = ["compatibility_matrix", "compatible", "incompatibility", "listed_techniques"]

TechniqueRef = str | TechniqueConfig | type[Technique]


def _cls(ref: TechniqueRef) -> type[Technique]:
    if isinstance(ref, str):
        return TECHNIQUES.get(ref)
    if isinstance(ref, TechniqueConfig):
        return TECHNIQUES.get(ref.technique)
    return ref


def incompatibility(a: TechniqueRef, b: TechniqueRef) -> str | None:
    """Why ``a`` and ``b`` cannot be attached together, or ``None`` when they can."""
    ca, cb = _cls(a), _cls(b)
    na, nb = ca.config_class.technique, cb.config_class.technique
    if na == nb:
        return f"{na} cannot be applied twice"
    if Capability.DRAFTER in ca.capabilities and Capability.DRAFTER in cb.capabilities:
        return f"{na} and {nb} both draft tokens (one drafting technique per model)"
    if ca.family == cb.family and ca.family in (Family.QUANTIZATION, Family.KV_COMPRESSION):
        return f"{na} and {nb} are both {ca.family.value} techniques"
    for x, y in ((ca, cb), (cb, ca)):
        excluded = getattr(x, "excludes", ())
        if y.config_class.technique in excluded:
            return f"{x.config_class.technique} excludes {y.config_class.technique}"
    return None


def compatible(a: TechniqueRef, b: TechniqueRef) -> bool:
    return incompatibility(a, b) is None


def listed_techniques() -> list[str]:
    return TECHNIQUES.names()


def compatibility_matrix(techniques: Iterable[TechniqueRef] | None = None) -> dict[str, dict[str, str | None]]:
    """``{a: {b: reason or None}}`` for every pair of ``techniques`` (default: all registered)."""
    names = [(_cls(t).config_class.technique if not isinstance(t, str) else t)
             for t in (techniques if techniques is not None else TECHNIQUES.names())]
    return {a: {b: (None if a == b else incompatibility(a, b)) for b in names} for a in names}
