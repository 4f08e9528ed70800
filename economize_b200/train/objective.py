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


def dense_linear(x: torch.Tensor, w, b: torch.Tensor | None = None) -> torch.Tensor:
    """``x @ w.T (+ b)`` with autograd for a tensor, a quantized weight (dequantized) or a LoRA-wrapped one (base
    product plus the trainable low-rank update)."""
    import torch.nn.functional as F

    from ..ops.lora import LoRAWeight

    if isinstance(w, LoRAWeight):
        y = dense_linear(x, w.base) + w.delta(x).to(x.dtype)
        return y if b is None else y + b
    if not isinstance(w, torch.Tensor):
        w = w.dequantize(x.dtype)
    return F.linear(x, w, b)


def _check_plain_block(config) -> None:
    """Refuse the block variants :func:`torch_block` does not model (it is the Llama block: pre-norms, per-head q/k
    norms, causal attention over the whole row, a dense SwiGLU MLP)."""
    variants = {"MoE MLPs": config.is_moe, "sandwich norms": config.sandwich_norm, "post norms": config.post_norm,
                "full-width q/k norms": config.qk_norm_full, "NoPE layers": bool(config.nope_layers),
                "sliding windows": any(config.window_of(i) for i in range(config.num_layers)),
                "soft-caps": bool(config.attn_softcap), "sink logits": config.attn_sinks,
                "an output-projection bias": config.o_bias, "a non-SwiGLU activation": config.hidden_act != "silu",
                "scaled attention or residuals": config.attention_multiplier is not None
                or config.residual_multiplier != 1.0, "position-scaled queries": config.query_position_scale is not None}
    found = [name for name, present in variants.items() if present]
    if found:
        raise ConfigError(f"the PyTorch training block models the Llama block; {config.model_type} has "
                          f"{', '.join(found)}")


def torch_block(layer, h: torch.Tensor, config, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """A pre-norm decoder block in plain PyTorch (autograd, causal attention over the whole row): the residual
    stream ``h [B, S, H]`` in, the block's output stream out. Used to train technique-owned blocks and adapters."""
    import torch.nn.functional as F

    from ..ops.reference import rmsnorm

    lin = dense_linear
    _check_plain_block(config)
    eps = config.rms_norm_eps
    batch, length, _ = h.shape
    heads, kv_heads, hd = config.num_heads, config.num_kv_heads, config.head_dim
    x = rmsnorm(h, layer.attn_norm, eps)[0]
    q, k, v = lin(x, layer.wqkv, layer.bqkv).split([heads * hd, kv_heads * hd, kv_heads * hd], -1)
    q = q.reshape(batch, length, heads, hd)
    k = k.reshape(batch, length, kv_heads, hd)
    if layer.q_norm is not None:
        q, k = rmsnorm(q, layer.q_norm, eps)[0], rmsnorm(k, layer.k_norm, eps)[0]
    c, s = cos[:length][None, :, None].to(q.dtype), sin[:length][None, :, None].to(q.dtype)

    def rot(t):
        a, b = t[..., : hd // 2], t[..., hd // 2:]
        return torch.cat([a * c - b * s, b * c + a * s], -1)

    q, k = rot(q).transpose(1, 2), rot(k).transpose(1, 2)
    v = v.reshape(batch, length, kv_heads, hd).transpose(1, 2)
    group = heads // kv_heads
    o = F.scaled_dot_product_attention(q, k.repeat_interleave(group, 1), v.repeat_interleave(group, 1),
                                       is_causal=True)
    h = h + lin(o.transpose(1, 2).reshape(batch, length, heads * hd), layer.wo)
    x = rmsnorm(h, layer.mlp_norm, eps)[0]
    g, u = lin(x, layer.w_gate_up).chunk(2, -1)
    a = F.silu(g) * u
    block = getattr(layer, "down_hadamard", 0)  # the online rotation the rotate technique folded into w_down
    if block:
        from ..ops import reference

        a = reference.hadamard(a, block)
    return h + lin(a, layer.w_down)


@OBJECTIVES.register("recovery_ce")
class RecoveryCE(Objective):
    """Next-token cross-entropy of a pruned target through its recovery adapters (LLM-Pruner's recovery stage;
    economize ``techniques/width_prune/recovery.py``): the whole model runs in plain PyTorch with autograd."""

    def __init__(self, model) -> None:
        super().__init__(model)
        self.tech = next(t for t in model.techniques.values() if getattr(t, "recovery", None) is not None)

    def parameters(self) -> list[torch.nn.Parameter]:
        return list(self.tech.recovery.parameters())

    def loss(self, tokens: torch.Tensor) -> tuple[torch.Tensor, dict[str, float]]:
        import torch.nn.functional as F

        from ..ops.reference import rmsnorm

        target = self.model.model
        c = target.config
        cos, sin = target.rope_tables(tokens.shape[1])
        h = target.embed_tokens(tokens).float()
        for layer in target.layers:
            h = torch_block(layer, h, c, cos, sin)
        logits = F.linear(rmsnorm(h, target.norm.float(), c.rms_norm_eps)[0], target.head_weight.float())
        loss = F.cross_entropy(logits[:, :-1].reshape(-1, logits.shape[-1]).float(), tokens[:, 1:].reshape(-1))
        return loss, {"loss": float(loss.detach())}


@OBJECTIVES.register("kangaroo_distill")
class KangarooDistill(Objective):
    """Kangaroo's adapter training: the adapter blocks read the target's residual stream after ``exit_layer``
    blocks and, through the target's final norm and LM head, learn the target's greedy next token (cross-entropy)."""

    name = "kangaroo_distill"
    defaults = OptimDefaults(lr=5e-4, warmup_steps=10)

    def __init__(self, model) -> None:
        super().__init__(model)
        if "kangaroo" not in model.techniques:
            raise ConfigError("kangaroo_distill needs an attached kangaroo technique")
        self.tech = model.techniques["kangaroo"]

    def parameters(self) -> list[torch.nn.Parameter]:
        return [p for p in self.tech.adapter.parameters() if p.requires_grad]

    def loss(self, tokens: torch.Tensor) -> tuple[torch.Tensor, dict[str, float]]:
        import torch.nn.functional as F

        from ..ops.reference import rmsnorm

        target = self.model.model
        k = self.tech.config.exit_layer
        aux, labels = teacher_pass(self.model, tokens, (k,))
        h = aux[k].detach()
        cos, sin = target.rope_tables(tokens.shape[1])
        for block in self.tech.adapter:
            h = torch_block(block, h, target.config, cos, sin)
        logits = F.linear(rmsnorm(h, target.norm, target.config.rms_norm_eps)[0], target.head_weight).float()
        loss = F.cross_entropy(logits.reshape(-1, logits.shape[-1]), labels.reshape(-1))
        with torch.no_grad():
            acc = (logits.argmax(-1) == labels).float().mean()
        return loss, {"loss": float(loss.detach()), "acc": float(acc)}


# ---- distillation objectives for EAGLE-3 heads -----------------------------------------------------------------
DIVERGENCES = ("kl", "rkl", "js", "tvd", "ce_top1")


def divergence(student_logp: torch.Tensor, teacher_p: torch.Tensor, kind: str) -> torch.Tensor:
    """Per-row divergence between a teacher distribution ``teacher_p`` and a student ``exp(student_logp)``."""
    sp = student_logp.exp()
    tlog = torch.log(teacher_p.clamp_min(1e-12))
    if kind == "kl":
        return (teacher_p * (tlog - student_logp)).sum(-1)
    if kind == "rkl":
        return (sp * (student_logp - tlog)).sum(-1)
    if kind == "js":
        m = 0.5 * (sp + teacher_p)
        logm = torch.log(m.clamp_min(1e-12))
        return 0.5 * (teacher_p * (tlog - logm)).sum(-1) + 0.5 * (sp * (student_logp - logm)).sum(-1)
    if kind == "tvd":
        return 0.5 * (sp - teacher_p).abs().sum(-1)
    if kind == "ce_top1":
        return -student_logp.gather(-1, teacher_p.argmax(-1, keepdim=True))[..., 0]
    raise ConfigError(f"unknown divergence {kind!r}; choose from {DIVERGENCES}")


def _teacher_draft_probs(model, tech, tokens: torch.Tensor, top_k: int | None, teacher=None):
    """Teacher next-token probabilities over the EAGLE-3 draft vocabulary ``[B, S, V_d]`` (restricted to the
    teacher's ``top_k`` tokens when given), plus the captured block outputs. ``teacher``: a function of the tokens
    giving another model's logits (:func:`~economize_b200.train.teacher.larger_teacher`); ``None``: the target's."""
    target = model.model
    batch, length = tokens.shape
    cache = target.new_cache(batch, ((length + 127) // 128) * 128)
    lengths = torch.full((batch,), length, dtype=torch.int32, device=tokens.device)
    with torch.no_grad():
        hidden, aux = target.forward_step(tokens, StepBatch.prefill(lengths, length), cache, tech.aux_layers)
        logits = target.logits(hidden).float() if teacher is None else teacher(tokens)
        ids = torch.arange(tech.d2t.numel(), device=tokens.device) + tech.d2t
        drafted = logits[..., ids]  # the draft vocabulary's logits, draft order
        if top_k is not None:
            kth = logits.topk(top_k, -1).values[..., -1:]
            drafted = drafted.masked_fill(drafted < kth, float("-inf"))
        probs = torch.softmax(drafted, -1).nan_to_num(0.0)
    return {k: v.detach() for k, v in aux.items()}, probs


@OBJECTIVES.register("distill_kl")
class Eagle3Distill(Objective):
    """Unrolled EAGLE-3 steps trained against the target's full next-token distribution (restricted to the draft
    vocabulary) under a divergence (``kl``, ``rkl``, ``js``, ``tvd``, ``ce_top1``); ``teacher``: a larger model
    with the same tokenizer (or its logits function) whose distributions replace the target's."""

    name = "distill_kl"
    defaults = OptimDefaults(lr=1e-3, warmup_steps=10)

    def __init__(self, model, divergence: str = "kl", steps: int | None = None, decay: float = 0.8,
                 top_k: int | None = None, teacher=None) -> None:
        super().__init__(model)
        if "eagle3" not in model.techniques:
            raise ConfigError(f"{self.name} needs an attached eagle3 technique")
        if divergence not in DIVERGENCES:
            raise ConfigError(f"unknown divergence {divergence!r}")
        self.tech = model.techniques["eagle3"]
        self.kind, self.decay, self.top_k = divergence, decay, top_k
        if isinstance(teacher, torch.nn.Module):  # a larger model with the same tokenizer
            from .teacher import larger_teacher

            teacher = larger_teacher(teacher, model.model.config.vocab_size)
        self.teacher = teacher
        self.steps = steps or self.tech.config.train_steps

    def parameters(self) -> list[torch.nn.Parameter]:
        return [p for p in self.tech.parameters() if p.requires_grad]

    def loss(self, tokens: torch.Tensor) -> tuple[torch.Tensor, dict[str, float]]:
        from ..techniques.eagle3.train import unrolled_logits

        aux, probs = _teacher_draft_probs(self.model, self.tech, tokens, self.top_k, self.teacher)
        outs = unrolled_logits(self.tech, aux, tokens, self.steps)
        positions = torch.arange(tokens.shape[1], device=tokens.device)
        total, weight, metrics = 0.0, 0.0, {}
        for j, logits in enumerate(outs, start=1):
            valid = (positions >= j)[None].expand(tokens.shape[0], -1)
            d = divergence(torch.log_softmax(logits.float(), -1), probs, self.kind)
            term = (d * valid).sum() / valid.sum().clamp_min(1)
            w = self.decay ** (j - 1)
            total, weight = total + w * term, weight + w
            metrics[f"div{j}"] = float(term.detach())
        loss = total / weight
        metrics["loss"] = float(loss.detach())
        return loss, metrics


@OBJECTIVES.register("hass")
class HASS(Objective):
    """HASS (Zhang et al., 2024, "Learning Harmonized Representations for Speculative Sampling"): EAGLE-3's
    training-time-test cross-entropy plus ``alpha`` times a KL distillation restricted to the target's top-K tokens
    (harmonized objective distillation), both over the unrolled steps that feed the head its own features
    (harmonized context alignment). Economize: ``techniques/hass``."""

    name = "hass"
    defaults = OptimDefaults(lr=1e-3, warmup_steps=10)

    def __init__(self, model, top_k: int = 10, alpha: float = 1.0, steps: int | None = None) -> None:
        super().__init__(model)
        self.ttt = Eagle3TTT(model, steps)
        self.distill = Eagle3Distill(model, "kl", steps, top_k=top_k)
        self.alpha = alpha

    def parameters(self) -> list[torch.nn.Parameter]:
        return self.ttt.parameters()

    def loss(self, tokens: torch.Tensor) -> tuple[torch.Tensor, dict[str, float]]:
        ce, m1 = self.ttt.loss(tokens)
        kl, m2 = self.distill.loss(tokens)
        loss = ce + self.alpha * kl
        return loss, {**{f"ttt_{k}": v for k, v in m1.items()}, **{f"topk_{k}": v for k, v in m2.items()},
                      "loss": float(loss.detach())}
