"""Distillation from a larger teacher (DistillSpec-style; economize ``train/teacher.py:100-171``).

A drafter is usually distilled from the model it drafts for; :func:`larger_teacher` lets the distributions come
from another model with the same tokenizer instead (a larger sibling, or the unquantized original of a quantized
target). The drafter's inputs (the captured block outputs) still come from the model it is attached to, since those
are what it reads at decode time; only the next-token distributions it is trained towards change.
"""

from __future__ import annotations

from collections.abc import Callable

import torch
from torch import nn

from ..errors import ConfigError
from ..runtime.cache import StepBatch

__all__ = ["TeacherLogits", "larger_teacher"]

#: ``tokens [B, S] -> logits [B, S, V]`` (fp32): the teacher's next-token logits at every position
TeacherLogits = Callable[[torch.Tensor], torch.Tensor]


def larger_teacher(teacher_model: nn.Module, vocab_size: int | None = None) -> TeacherLogits:
    """The next-token logits of ``teacher_model`` as a function of token rows, truncated to the first
    ``vocab_size`` entries when given (a teacher whose vocabulary extends the student's with padding rows).

    ``teacher_model`` is this package's :class:`~economize_b200.models.llama.CausalLM` (one prompt pass through its
    own cache) or any module whose call returns logits or an object with ``.logits`` (a ``transformers`` model). It
    runs without gradients on its own device; the logits come back on the tokens' device."""
    if not isinstance(teacher_model, nn.Module):
        raise ConfigError(f"a larger teacher is a module, got {type(teacher_model).__name__}")

    @torch.no_grad()
    def logits(tokens: torch.Tensor) -> torch.Tensor:
        device = next(teacher_model.parameters()).device
        ids = tokens.to(device)
        if hasattr(teacher_model, "forward_step") and hasattr(teacher_model, "new_cache"):
            batch, length = ids.shape
            cache = teacher_model.new_cache(batch, ((length + 127) // 128) * 128)
            lengths = torch.full((batch,), length, dtype=torch.int32, device=device)
            hidden, _ = teacher_model.forward_step(ids, StepBatch.prefill(lengths, length), cache)
            out = teacher_model.logits(hidden)
        else:
            out = teacher_model(ids)
            out = getattr(out, "logits", out)
        if vocab_size is not None:
            if out.shape[-1] < vocab_size:
                raise ConfigError(f"the teacher's vocabulary ({out.shape[-1]}) is smaller than the student's "
                                  f"({vocab_size})")
            out = out[..., :vocab_size]
        return out.float().to(tokens.device)

    return logits
