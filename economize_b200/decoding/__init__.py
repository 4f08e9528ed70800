"""Decoding: options, the device-resident speculative engine, tree utilities, selectors."""

from .config import DecodeConfig
from .engine import DecodeResult, GenerationStats, SpecEngine
from .selectors import GreedySelector, TokenSelector, TopPSampler
from .tree import TreeOptions, select_candidates

__all__ = ["DecodeConfig", "DecodeResult", "GenerationStats", "GreedySelector", "SpecEngine", "TokenSelector",
           "TopPSampler", "TreeOptions", "select_candidates"]
