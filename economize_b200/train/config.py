"""Settings of a training run (fields of economize's ``TrainConfig``, ``src/economize/train/loop.py:98-190``)."""

from __future__ import annotations

from dataclasses import asdict, dataclass
from pathlib import Path

from ..validation import check_choice, check_positive

__all__ = ["TrainConfig"]


@dataclass
class TrainConfig:
    steps: int = 1000
    batch_size: int = 8
    seq_len: int = 1024
    grad_accum: int = 1
    lr: float | None = None
    weight_decay: float | None = None
    betas: tuple[float, float] | None = None
    warmup_steps: int | None = None
    schedule: str | None = None
    min_lr_ratio: float | None = None
    grad_clip: float | None = None
    autocast: str | None = "bfloat16"
    nonfinite: str = "raise"
    log_every: int = 50
    eval_every: int | None = None
    save_every: int | None = None
    keep_checkpoints: int = 2
    output_dir: str | Path | None = None
    resume: bool | str | Path = False
    seed: int | None = None
    offload_optimizer: bool = False  # AdamW master weights and moments in host memory (train/offload.py)

    def __post_init__(self) -> None:
        check_positive("steps", self.steps)
        check_positive("grad_accum", self.grad_accum)
        check_positive("batch_size", self.batch_size)
        check_choice("nonfinite", self.nonfinite, ("raise", "skip", "warn"))
        if self.schedule is not None:
            check_choice("schedule", self.schedule, ("cosine", "linear", "constant"))

    def to_dict(self) -> dict:
        out = asdict(self)
        out["output_dir"] = None if self.output_dir is None else str(self.output_dir)
        out["resume"] = str(self.resume) if isinstance(self.resume, Path) else self.resume
        return out
