"""Pruning: ``prune`` (magnitude / Wanda / SparseGPT masks, unstructured or N:M; 2:4 weights stored compressed
for the sparse weight-streaming GEMM) and ``depth_prune`` (ShortGPT / SLEB block removal). Economize:
``techniques/prune`` (``config.py:28-160``, ``wanda.py``, ``sparsegpt.py``, ``depth.py``)."""

from .config import DepthPruneConfig, PruneConfig
from .methods import magnitude_scores, nm_mask, sparsegpt, unstructured_mask, wanda_scores
from .technique import DepthPruneTechnique, PruneTechnique

__all__ = ["DepthPruneConfig", "DepthPruneTechnique", "PruneConfig", "PruneTechnique", "magnitude_scores", "nm_mask",
           "sparsegpt", "unstructured_mask", "wanda_scores"]
