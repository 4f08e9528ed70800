"""The persistent datastore of the retrieval drafters (``rest``; economize ``techniques/retrieval``): a suffix array
over records of tokens, built once and memory-mapped when loaded.

    python -m economize_b200.techniques.retrieval build store/ --tokens train.bin --dtype uint32 --spans spans.npy
    python -m economize_b200.techniques.retrieval info store/

From Python: :meth:`SuffixIndex.build` over any token sequences, :meth:`SuffixIndex.save`, then
``RestConfig(datastore="store/")``. The package registers no technique.
"""

from __future__ import annotations

import numpy as np

from .index import FORMAT, SEPARATOR, SuffixIndex, suffix_array

__all__ = ["FORMAT", "SEPARATOR", "SuffixIndex", "build_from_spans", "suffix_array"]


def build_from_spans(tokens: np.ndarray, spans: np.ndarray, depth: int = 64) -> SuffixIndex:
    """Index the records ``tokens[start:end]`` of every row ``(start, end)`` of ``spans``."""
    return SuffixIndex.build((np.asarray(tokens[int(s):int(e)]) for s, e in spans), depth)
