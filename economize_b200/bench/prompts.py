"""Benchmark prompt sets (economize ``bench/prompts.py:99-161``).

* ``"synthetic"``: uniform-random token ids of a fixed length (the headline benchmark's prompts: no dataset needed);
* ``"smoke"``: a few short built-in English prompts;
* a path to a local JSON-lines file in one of the common layouts: Spec-Bench / MT-Bench (``{"turns": [...]}``, the
  first turn is used), GSM8K (``{"question": ...}``), HumanEval (``{"prompt": ...}``), or ``{"text": ...}``.

Text prompts are tokenized with the given tokenizer (``encode``); the datasets themselves are not bundled or fetched.
"""

from __future__ import annotations

import json
from pathlib import Path

import torch

from ..errors import ConfigError

__all__ = ["SMOKE_PROMPTS", "load_prompts"]

SMOKE_PROMPTS = (
    "Explain why the sky is blue in two sentences.",
    "Write a Python function that returns the n-th Fibonacci number.",
    "List three differences between a list and a tuple in Python.",
    "Summarize the plot of a detective story in one paragraph.",
)

_TEXT_KEYS = ("turns", "question", "prompt", "text")


def _text_of(record: dict) -> str:
    for key in _TEXT_KEYS:
        if key in record:
            value = record[key]
            return value[0] if isinstance(value, list) else str(value)
    raise ConfigError(f"a prompt record needs one of {_TEXT_KEYS}, got keys {sorted(record)}")


def load_prompts(source: str | Path, n: int, *, tokenizer=None, length: int = 512, vocab_size: int | None = None,
                 seed: int = 0) -> list[torch.Tensor]:
    """``n`` prompts as 1-D int64 token tensors from ``source`` (see the module docstring)."""
    if n < 1:
        raise ConfigError("n must be positive")
    if source == "synthetic":
        if vocab_size is None:
            raise ConfigError("synthetic prompts need vocab_size")
        g = torch.Generator().manual_seed(seed)
        return [torch.randint(0, vocab_size, (length,), generator=g) for _ in range(n)]
    if source == "smoke":
        texts = [SMOKE_PROMPTS[i % len(SMOKE_PROMPTS)] for i in range(n)]
    else:
        path = Path(source)
        if not path.is_file():
            raise ConfigError(f"no prompt set {str(source)!r}: use 'synthetic', 'smoke' or a JSON-lines file")
        records = [json.loads(line) for line in path.read_text().splitlines() if line.strip()]
        if not records:
            raise ConfigError(f"{path} holds no prompts")
        texts = [_text_of(records[i % len(records)]) for i in range(n)]
    if tokenizer is None:
        raise ConfigError("text prompts need a tokenizer")
    out = []
    for text in texts:
        try:
            ids = tokenizer.encode(text, add_special_tokens=False)
        except TypeError:
            ids = tokenizer.encode(text)
        out.append(torch.tensor(list(ids), dtype=torch.long))
    return out
