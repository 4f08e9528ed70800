"""Shared pieces of the one-layer draft decoders (EAGLE-1/2, EAGLE-3)."""

from .config import DraftLayerConfig
from .layer import DraftLayer

__all__ = ["DraftLayer", "DraftLayerConfig"]
