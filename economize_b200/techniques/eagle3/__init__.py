"""EAGLE-3 drafting (``Eagle3Config``): fused low/mid/high target features + one draft decoder layer."""

from .config import EAGLE3_HEADS, Eagle3Config, default_aux_layers
from .technique import Eagle3Drafter, Eagle3Technique
from . import formats  # noqa: E402,F401  (registers the official EAGLE-3 checkpoint format)

__all__ = ["EAGLE3_HEADS", "Eagle3Config", "Eagle3Drafter", "Eagle3Technique", "default_aux_layers"]
