"""Training objectives: what ``fit`` optimizes for a technique (economize ``train/objective.py``, ``OBJECTIVES``).

An objective names the parameters it trains and turns a batch of token rows into a loss. The teacher pass (the
frozen target over the rows, with the block outputs the drafter reads) runs on the engine's kernels without
gradients; the student runs in plain PyTorch with autograd.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

from .. import ops
from ..core.technique import Capability
from ..errors import ConfigError
from ..registry import Registry
from ..runtime.cache import StepBatch

__all__ = ["OBJECTIVES", "Eagle3TTT", "Objective", "OptimDefaults", "default_objective", "teacher_pass"]


@dataclass(frozen=True)
class OptimDefaults:
    lr: float = 3e-4
    weight_decay: float = 0.0
    betas: tuple[float, float] = (0.9, 0.95)
    warmup_steps: int = 20
    schedule: str = "cosine"
    min_lr_ratio: float = 0.1
    grad_clip: float | None = 0.5


class Objective:
    name = ""
    defaults = OptimDefaults()

    def __init__(self, model) -> None:
        self.model = model

    def parameters(self) -> list[torch.nn.Parameter]:
        raise NotImplementedError

    def loss(self, tokens: torch.Tensor) -> tuple[torch.Tensor, dict[str, float]]:
        raise NotImplementedError


OBJECTIVES: Registry[type[Objective]] = Registry("training objective", "economize_b200.objectives")


@torch.no_grad()
def teacher_pass(model, tokens: torch.Tensor, capture: tuple[int, ...]) -> tuple[dict[int, torch.Tensor], torch.Tensor]:
    """Captured block outputs and the target's greedy next token at every position of ``tokens [B, S]``."""
    target = model.model
    batch, length = tokens.shape
    cache = target.new_cache(batch, ((length + 127) // 128) * 128)
    lengths = torch.full((batch,), length, dtype=torch.int32, device=tokens.device)
    hidden, aux = target.forward_step(tokens, StepBatch.prefill(lengths, length), cache, capture)
    labels = ops.argmax(target.logits(hidden))
    return aux, labels


@OBJECTIVES.register("eagle3_ttt")
class Eagle3TTT(Objective):
    """EAGLE-3 training-time test: cross-entropy of every unrolled draft step against the target's greedy next
    token, mapped into the draft vocabulary (tokens outside it are ignored); step ``j`` weighs ``decay**(j-1)``."""

    name = "eagle3_ttt"
    defaults = OptimDefaults(lr=1e-3, warmup_steps=10)

    def __init__(self, model, steps: int | None = None, decay: float = 0.8) -> None:
        super().__init__(model)
        tech = model.techniques["eagle3"] if "eagle3" in model.techniques else None
        if tech is None:
            raise ConfigError("eagle3_ttt needs an attached eagle3 technique")
        self.tech = tech
        self.steps = steps or tech.config.train_steps
        self.decay = decay

    def parameters(self) -> list[torch.nn.Parameter]:
        return [p for p in self.tech.parameters() if p.requires_grad]

    def loss(self, tokens: torch.Tensor) -> tuple[torch.Tensor, dict[str, float]]:
        from ..techniques.eagle3.train import unrolled_logits

        tech = self.tech
        aux, labels = teacher_pass(self.model, tokens, tech.aux_layers)
        aux = {k: v.detach() for k, v in aux.items()}
        # target id -> draft id (-100 outside the draft vocabulary)
        d2t = tech.d2t
        draft_of = torch.full((tech.t2d.numel(),), -100, dtype=torch.long, device=tokens.device)
        ids = torch.arange(d2t.numel(), device=tokens.device)
        draft_of[ids + d2t] = ids
        target_ids = draft_of[labels]
        outs = unrolled_logits(tech, aux, tokens, self.steps)
        positions = torch.arange(tokens.shape[1], device=tokens.device)
        total, weight, metrics = 0.0, 0.0, {}
        for j, logits in enumerate(outs, start=1):
            mask = (positions >= j)[None].expand_as(target_ids)
            tgt = torch.where(mask, target_ids, torch.full_like(target_ids, -100))
            ce = torch.nn.functional.cross_entropy(logits.reshape(-1, logits.shape[-1]), tgt.reshape(-1),
                                                   ignore_index=-100)
            w = self.decay ** (j - 1)
            total = total + w * ce
            weight += w
            with torch.no_grad():
                valid = tgt >= 0
                acc = ((logits.argmax(-1) == tgt) & valid).sum() / valid.sum().clamp_min(1)
            metrics[f"acc{j}"] = float(acc)
        loss = total / weight
        metrics["loss"] = float(loss.detach())
        return loss, metrics


def default_objective(model) -> Objective:
    """The objective of the model's trainable technique (its drafter)."""
    for tech in model.techniques.values():
        if Capability.DRAFTER in tech.capabilities and tech.name == "eagle3":
            return Eagle3TTT(model)
        if tech.name == "medusa":
            return MedusaCE(model)
        name = getattr(tech, "objective_name", None)
        if name is not None:
            return OBJECTIVES.get(name)(model)
    raise ConfigError("no attached technique has a default training objective")


@OBJECTIVES.register("medusa_ce")
class MedusaCE(Objective):
    """Medusa-1 self-distillation: head ``j`` at position ``t`` learns the target's greedy token ``j + 1`` places
    after the LM head's (cross-entropy, head ``j`` weighed ``decay**j``)."""

    name = "medusa_ce"
    defaults = OptimDefaults(lr=1e-3, warmup_steps=10)

    def __init__(self, model, decay: float = 0.8) -> None:
        super().__init__(model)
        if "medusa" not in model.techniques:
            raise ConfigError("medusa_ce needs an attached medusa technique")
        self.tech = model.techniques["medusa"]
        self.decay = decay

    def parameters(self) -> list[torch.nn.Parameter]:
        return [p for p in self.tech.parameters() if p.requires_grad]

    def loss(self, tokens: torch.Tensor) -> tuple[torch.Tensor, dict[str, float]]:
        import torch.nn.functional as F

        tech = self.tech
        key = -1 if tech.config.head == "own" else self.model.model.config.num_layers
        aux, labels = teacher_pass(self.model, tokens, (key,))
        states = aux[key].detach()
        total, weight, metrics = 0.0, 0.0, {}
        for j, head in enumerate(tech.heads):
            x = states.to(head.blocks[0].linear.weight.dtype) if len(head.blocks) else states
            for block in head.blocks:
                x = x + F.silu(F.linear(x, block.linear.weight, block.linear.bias))
            if head.proj is not None:
                logits = F.linear(x, head.proj.weight).float()
            else:
                m = self.model.model
                from ..ops.reference import rmsnorm

                logits = F.linear(rmsnorm(x, m.norm, m.config.rms_norm_eps)[0], m.head_weight).float()
            shift = j + 1
            if labels.shape[1] <= shift:
                break
            target = labels[:, shift:]
            ce = F.cross_entropy(logits[:, :-shift].reshape(-1, logits.shape[-1]), target.reshape(-1))
            w = self.decay ** j
            total = total + w * ce
            weight += w
            metrics[f"ce{j + 1}"] = float(ce.detach())
        loss = total / max(weight, 1e-9)
        metrics["loss"] = float(loss.detach())
        return loss, metrics
