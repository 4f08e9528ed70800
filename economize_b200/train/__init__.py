"""Training of technique parameters (drafters): ``fit``, ``TrainConfig``, objectives, checkpoints, data."""

from __future__ import annotations

import logging

from .checkpoint import RunCheckpointer
from .config import TrainConfig
from .data import TensorSource, greedy_continuations
from .loop import TrainResult, fit
from .objective import OBJECTIVES, Eagle3TTT, Objective, OptimDefaults, default_objective, teacher_pass
from .teacher import larger_teacher

__all__ = ["larger_teacher", "OBJECTIVES", "Eagle3TTT", "Objective", "OptimDefaults", "RunCheckpointer", "TensorSource",
           "TrainConfig", "TrainResult", "default_objective", "fit", "fit_eagle3_on_greedy", "greedy_continuations",
           "teacher_pass"]


def fit_eagle3_on_greedy(model, steps: int = 200, n_rows: int = 64, prompt_len: int = 256, new_tokens: int = 128,
                         batch_size: int = 8, seed: int = 0, **overrides) -> TrainResult:
    """Train an attached EAGLE-3 head on the target's own greedy continuations of uniform-random prompts."""
    data = greedy_continuations(model, n_rows, prompt_len, new_tokens, seed=seed)
    result = fit(model, data, steps=steps, batch_size=batch_size, seed=seed, log_every=max(1, steps // 10),
                 **overrides)
    logging.getLogger("economize_b200.train").info("eagle3 training done: %s", result.final)
    return result
