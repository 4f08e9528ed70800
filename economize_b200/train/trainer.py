"""Hugging Face ``Trainer`` integration (economize ``train/trainer.py``: ``EffTrainer``, ``EffCollator``).

:class:`EffTrainer` trains the technique parameters of an :class:`~economize_b200.EfficientModel` with the
``transformers`` training loop: the objective (the technique's default or a registered name) is wrapped as the
trainer's module (:class:`ObjectiveModule`, whose parameters are the technique's own tensors, not copies), batches
of ``input_ids`` come from :class:`EffCollator`, and the loss is the objective's. ``transformers``' Trainer needs
the ``accelerate`` package; without it :class:`EffTrainer` raises a ConfigError and :func:`economize_b200.train.fit`
is the loop to use.
"""

from __future__ import annotations

from typing import Any

import torch
from torch import nn

from ..errors import ConfigError

__all__ = ["EffCollator", "EffTrainer", "ObjectiveModule"]


class ObjectiveModule(nn.Module):
    """The objective as a module: ``forward(input_ids)`` returns ``{"loss": ..., **metrics}``."""

    def __init__(self, objective) -> None:
        super().__init__()
        self.trained = nn.ParameterList(objective.parameters())
        self._objective = [objective]

    def forward(self, input_ids: torch.Tensor, **_: Any) -> dict[str, Any]:
        loss, metrics = self._objective[0].loss(input_ids)
        return {**{k: torch.tensor(v) for k, v in metrics.items()}, "loss": loss}


class EffCollator:
    """Stacks ``input_ids`` of the dataset's examples (tensors, lists, or dicts with ``input_ids``)."""

    def __call__(self, features: list[Any]) -> dict[str, torch.Tensor]:
        rows = [f["input_ids"] if isinstance(f, dict) else f for f in features]
        return {"input_ids": torch.stack([torch.as_tensor(r, dtype=torch.long) for r in rows])}


def _trainer_base():
    try:
        import accelerate  # noqa: F401
        from transformers import Trainer
    except ImportError as err:
        raise ConfigError("EffTrainer runs transformers' Trainer, which needs the accelerate package; use "
                          "economize_b200.train.fit instead") from err
    return Trainer


def EffTrainer(model, args=None, train_dataset=None, objective=None, **kwargs):  # noqa: N802 (a class factory)
    """A ``transformers.Trainer`` over ``model``'s technique parameters (see the module docstring)."""
    from .loop import _objective

    base = _trainer_base()
    obj = _objective(model, objective)

    class _EffTrainer(base):
        def compute_loss(self, module, inputs, return_outputs=False, num_items_in_batch=None):
            out = module(**inputs)
            return (out["loss"], out) if return_outputs else out["loss"]

    if args is None:
        from transformers import TrainingArguments

        args = TrainingArguments(output_dir="economize_trainer", report_to=[], remove_unused_columns=False)
    return _EffTrainer(model=ObjectiveModule(obj), args=args, train_dataset=train_dataset,
                       data_collator=kwargs.pop("data_collator", EffCollator()), **kwargs)
