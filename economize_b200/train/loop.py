"""``fit``: the training loop for technique parameters (economize ``train/loop.py:250-581``).

AdamW over the objective's parameters (kept in float32 while training, cast back to the model's dtype at the end),
linear warmup + cosine/linear/constant decay, gradient accumulation, clipping, bf16 autocast, a non-finite policy,
atomic checkpoints with resume, and data-parallel gradient averaging when ``torch.distributed`` is initialized.
"""

from __future__ import annotations

import logging
import math
import random
from dataclasses import dataclass, field
from typing import Any

import torch

from ..errors import ConfigError, NonFiniteLossError
from .checkpoint import RunCheckpointer
from .config import TrainConfig
from .data import TensorSource
from .objective import OBJECTIVES, Objective, default_objective

__all__ = ["TrainResult", "fit", "make_scheduler"]

log = logging.getLogger("economize_b200.train")


@dataclass
class TrainResult:
    steps: int = 0
    history: list[dict[str, float]] = field(default_factory=list)
    skipped: int = 0

    @property
    def final(self) -> dict[str, float]:
        return self.history[-1] if self.history else {}


def make_scheduler(optimizer: torch.optim.Optimizer, steps: int, warmup: int, schedule: str, min_ratio: float):
    def factor(step: int) -> float:
        if step < warmup:
            return (step + 1) / max(1, warmup)
        t = (step - warmup) / max(1, steps - warmup)
        if schedule == "constant":
            return 1.0
        if schedule == "linear":
            return max(min_ratio, 1.0 - t * (1 - min_ratio))
        return min_ratio + (1 - min_ratio) * 0.5 * (1 + math.cos(math.pi * min(1.0, t)))

    return torch.optim.lr_scheduler.LambdaLR(optimizer, factor)


def _objective(model, objective: Objective | str | None) -> Objective:
    if objective is None:
        return default_objective(model)
    if isinstance(objective, str):
        return OBJECTIVES.get(objective)(model)
    return objective


def fit(model, data: Any, objective: Objective | str | None = None, config: TrainConfig | None = None,
        **overrides: Any) -> TrainResult:
    """Train the technique parameters of ``model`` (an :class:`~economize_b200.EfficientModel`).

    Args:
        data: A ``[N, S]`` token tensor, or an object with ``next()`` returning ``[B, S]`` batches.
        objective: An :class:`Objective`, a registered name, or ``None`` for the technique's default.
        config: A :class:`TrainConfig`; keyword ``overrides`` replace its fields.
    """
    cfg = config or TrainConfig()
    if overrides:
        cfg = TrainConfig(**{**cfg.__dict__, **overrides})
    if cfg.seed is not None:
        torch.manual_seed(cfg.seed)
        random.seed(cfg.seed)
    obj = _objective(model, objective)
    dist_on = torch.distributed.is_available() and torch.distributed.is_initialized()
    rank = torch.distributed.get_rank() if dist_on else 0
    # data parallelism: every rank draws its own batches (the seed is offset by the rank)
    source = TensorSource(data, cfg.batch_size, seed=(cfg.seed or 0) + 1000003 * rank) \
        if isinstance(data, torch.Tensor) else data
    ckpt = RunCheckpointer(cfg.output_dir, cfg.keep_checkpoints) if cfg.output_dir is not None else None
    params = obj.parameters()
    if not params:
        raise ConfigError("the objective has no trainable parameters")
    modules = {id(p): p for p in params}
    orig_dtype = params[0].dtype
    if dist_on:  # data parallelism: every rank starts from rank 0's parameters (as DDP does)
        with torch.no_grad():
            for p in params:
                torch.distributed.broadcast(p.data, src=0)
    for p in params:  # fp32 master weights while training
        p.data = p.data.float()
    d = obj.defaults
    opt_cls = torch.optim.AdamW
    if cfg.offload_optimizer:
        from .offload import OffloadedAdamW as opt_cls
    opt = opt_cls(params, lr=cfg.lr or d.lr, betas=cfg.betas or d.betas,
                  weight_decay=d.weight_decay if cfg.weight_decay is None else cfg.weight_decay)
    sched = make_scheduler(opt, cfg.steps, d.warmup_steps if cfg.warmup_steps is None else cfg.warmup_steps,
                           cfg.schedule or d.schedule, d.min_lr_ratio if cfg.min_lr_ratio is None else cfg.min_lr_ratio)
    clip = d.grad_clip if cfg.grad_clip is None else (cfg.grad_clip or None)
    names = {id(p): n for n, p in _named(obj, params)}
    result = TrainResult()
    start = 0
    resume_from = None
    if ckpt is not None and cfg.resume:
        if cfg.resume is True:
            done = ckpt.finished()
            if done is not None:
                weights, state = RunCheckpointer.load(done)
                _load(params, names, weights)
                _restore_dtype(params, orig_dtype)
                return TrainResult(steps=state["step"])
            resume_from = ckpt.latest()
        else:
            resume_from = cfg.resume
    if resume_from is not None:
        weights, state = RunCheckpointer.load(resume_from)
        _load(params, names, weights)
        opt.load_state_dict(state["optimizer"])
        sched.load_state_dict(state["scheduler"])
        if hasattr(source, "restore"):
            source.restore(state["data"])
        torch.set_rng_state(state["torch_rng"])
        start = state["step"]
    dist = torch.distributed.is_available() and torch.distributed.is_initialized()
    amp = {"bfloat16": torch.bfloat16, "float16": torch.float16}.get(str(cfg.autocast).replace("torch.", ""))
    dev_type = params[0].device.type
    for step in range(start, cfg.steps):
        opt.zero_grad(set_to_none=True)
        metrics_acc: dict[str, float] = {}
        bad = False
        for _ in range(cfg.grad_accum):
            batch = source.next()
            with torch.autocast(dev_type, dtype=amp, enabled=amp is not None and dev_type == "cuda"):
                loss, metrics = obj.loss(batch)
            if not torch.isfinite(loss):
                if cfg.nonfinite == "raise":
                    _restore_dtype(params, orig_dtype)
                    raise NonFiniteLossError(f"non-finite loss {float(loss)} at step {step}")
                if cfg.nonfinite == "skip":
                    bad = True
                    continue
                log.warning("non-finite loss at step %d", step)
            (loss / cfg.grad_accum).backward()
            for k, v in metrics.items():
                metrics_acc[k] = metrics_acc.get(k, 0.0) + v / cfg.grad_accum
        if dist:
            world = torch.distributed.get_world_size()
            for p in params:
                if p.grad is not None:
                    torch.distributed.all_reduce(p.grad)
                    p.grad /= world
        if bad:
            opt.zero_grad(set_to_none=True)
            result.skipped += 1
        else:
            if clip:
                torch.nn.utils.clip_grad_norm_(params, clip)
            opt.step()
        sched.step()
        metrics_acc["step"] = step + 1
        metrics_acc["lr"] = sched.get_last_lr()[0]
        result.history.append(metrics_acc)
        result.steps = step + 1
        if (step + 1) % cfg.log_every == 0 or step + 1 == cfg.steps:
            log.info("step %d %s", step + 1, {k: round(v, 4) for k, v in metrics_acc.items()})
        if ckpt is not None and cfg.save_every and (step + 1) % cfg.save_every == 0 and step + 1 < cfg.steps:
            ckpt.save(step + 1, _state(params, names), opt, sched,
                      source.state() if hasattr(source, "state") else {})
    if ckpt is not None:
        ckpt.save(result.steps, _state(params, names), opt, sched,
                  source.state() if hasattr(source, "state") else {}, final=True,
                  result={"step": result.steps, "final": result.final})
    _restore_dtype(params, orig_dtype)
    model.refresh()
    del modules
    return result


def _named(obj: Objective, params: list[torch.nn.Parameter]):
    owner = getattr(obj, "tech", None)
    if owner is not None:
        lookup = {id(p): n for n, p in owner.named_parameters()}
        return [(lookup.get(id(p), f"param{i}"), p) for i, p in enumerate(params)]
    return [(f"param{i}", p) for i, p in enumerate(params)]


def _state(params, names) -> dict[str, torch.Tensor]:
    return {names[id(p)]: p.detach() for p in params}


def _load(params, names, weights) -> None:
    with torch.no_grad():
        for p in params:
            p.data = weights[names[id(p)]].to(p.device, torch.float32)


def _restore_dtype(params, dtype) -> None:
    for p in params:
        p.data = p.data.to(dtype)
        p.grad = None
