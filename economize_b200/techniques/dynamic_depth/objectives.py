"""Training objectives of the dynamic-depth techniques (economize ``techniques/dynamic_depth/objective.py``).

The base model stays frozen; only the gates, routers, adapters, low-rank updates and exit classifiers are trained.
The student pass runs every block in plain PyTorch (:func:`~economize_b200.train.objective.torch_block`, so
autograd reaches the technique's modules on any device) with the policy in training mode, and is scored with the
cross-entropy against the frozen model's greedy next token plus the technique's regulariser:

* ``gateskip``: ``sparsity * mean(gate)``;
* ``mod``: ``aux_weight * BCE(sigmoid(router), top-k membership)``, the causal predictor used at inference;
* ``flexidepth``: ``layer_penalty * mean((sum_l g_l)^2)``;
* ``loradrop``: the mean squared error between each low-rank update and the layer update it replaces;
* ``calm``: no student pass; the exit classifier learns from the frozen states which layers already predict the
  final layer's top token (BCE).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from ...errors import ConfigError
from ...runtime.cache import StepBatch
from ...train.objective import OBJECTIVES, Objective, OptimDefaults, torch_block

__all__ = ["student_pass"]


def student_pass(tech, tokens: torch.Tensor) -> torch.Tensor:
    """Logits ``[B, S, V]`` of the model under ``tech``'s policy in training mode (autograd through the gates)."""
    model = tech.model
    policy = tech.policy
    cfg = model.config
    cos, sin = model.rope_tables(tokens.shape[1])
    b, s = tokens.shape
    batch = StepBatch.prefill(torch.full((b,), s, dtype=torch.int32, device=tokens.device), s)
    policy.training = True
    try:
        h = model.embed_tokens(tokens).float()
        policy.begin_pass(batch, h)
        params = {}
        for i, layer in enumerate(model.layers):
            w = {n: getattr(layer, n) for n in ("attn_norm", "wqkv", "bqkv", "wo", "q_norm", "k_norm", "mlp_norm",
                                                "w_gate_up", "w_down")}
            params[i] = type("L", (), {k: (v.float() if isinstance(v, torch.Tensor) else v) for k, v in w.items()})
            out = torch_block(params[i], h, cfg, cos, sin)
            h = policy.combine(i, h, out, batch).float() if policy.gates(i) else out
        from ...ops.reference import rmsnorm

        hn = rmsnorm(h, model.norm.float(), cfg.rms_norm_eps)[0]
        return F.linear(hn, model.head_weight.float())
    finally:
        policy.training = False


def _teacher_labels(model, tokens: torch.Tensor) -> torch.Tensor:
    from ...train.objective import teacher_pass

    class _Wrap:
        pass

    w = _Wrap()
    w.model = model
    return teacher_pass(w, tokens, ())[1]


class _DepthObjective(Objective):
    technique = ""
    defaults = OptimDefaults(lr=1e-3, warmup_steps=0, grad_clip=1.0)

    def __init__(self, model) -> None:
        super().__init__(model)
        if self.technique not in model.techniques:
            raise ConfigError(f"the {self.name} objective needs an attached {self.technique} technique")
        self.tech = model.techniques[self.technique]

    def parameters(self):
        return [p for p in self.tech.parameters() if p.requires_grad]

    def regulariser(self, log: dict) -> tuple[torch.Tensor, dict[str, float]]:
        return torch.zeros(()), {}

    def loss(self, tokens: torch.Tensor):
        labels = _teacher_labels(self.tech.model, tokens)
        logits = student_pass(self.tech, tokens)
        ce = F.cross_entropy(logits[:, :-1].reshape(-1, logits.shape[-1]).float(), labels[:, :-1].reshape(-1))
        reg, metrics = self.regulariser(self.tech.policy.gate_log)
        loss = ce + reg.to(ce.device)
        metrics.update(ce=float(ce.detach()), loss=float(loss.detach()))
        return loss, metrics


@OBJECTIVES.register("gateskip")
class GateSkipObjective(_DepthObjective):
    name = technique = "gateskip"
    sparsity = 0.01

    def regulariser(self, log):
        gates = torch.stack([g.float().mean() for g in log.values()])
        return self.sparsity * gates.mean(), {"mean_gate": float(gates.mean().detach())}


@OBJECTIVES.register("mod")
class MoDObjective(_DepthObjective):
    name = technique = "mod"
    aux_weight = 0.1

    def regulariser(self, log):
        terms = []
        for key, run in log.items():
            if isinstance(key, tuple):
                r = log[key[0]]
                terms.append(F.binary_cross_entropy_with_logits(r.float(), run.float()))
        aux = torch.stack(terms).mean() if terms else torch.zeros(())
        return self.aux_weight * aux, {"router_bce": float(aux.detach())}


@OBJECTIVES.register("flexidepth")
class FlexiDepthObjective(_DepthObjective):
    name = technique = "flexidepth"
    layer_penalty = 1e-3

    def regulariser(self, log):
        total = torch.stack([g.float() for g in log.values()]).sum(0)  # [B, S] layers used
        pen = total.pow(2).mean()
        return self.layer_penalty * pen, {"layer_penalty": float(pen.detach())}


@OBJECTIVES.register("loradrop")
class LoRADropObjective(_DepthObjective):
    name = technique = "loradrop"

    def regulariser(self, log):
        mse = torch.stack([F.mse_loss(lora, target.detach()) for lora, target in log.values()]).mean()
        return mse, {"imitation_mse": float(mse.detach())}


@OBJECTIVES.register("calm")
class CalmObjective(Objective):
    """BCE of the exit classifier on every layer's state against "this layer's top token equals the last layer's"."""

    name = "calm"
    defaults = OptimDefaults(lr=1e-3, warmup_steps=0, grad_clip=None)
    positive_weight = 1.0

    def __init__(self, model) -> None:
        super().__init__(model)
        tech = model.techniques["calm"] if "calm" in model.techniques else None
        if tech is None or tech.classifier is None:
            raise ConfigError("the calm objective trains the exit classifier of a calm technique with "
                              "confidence='classifier'")
        self.tech = tech

    def parameters(self):
        return list(self.tech.classifier.parameters())

    def loss(self, tokens: torch.Tensor):
        from ... import ops

        model = self.tech.model
        n = model.config.num_layers
        b, s = tokens.shape
        with torch.no_grad():
            cache = model.new_cache(b, ((s + 127) // 128) * 128)
            lengths = torch.full((b,), s, dtype=torch.int32, device=tokens.device)
            _, aux = model.forward_step(tokens, StepBatch.prefill(lengths, s), cache, capture=tuple(range(1, n + 1)))
            final = model.greedy(ops.rmsnorm(aux[n], model.norm, model.config.rms_norm_eps)[0])
        losses = []
        for i in range(1, n):
            with torch.no_grad():
                pred = model.greedy(ops.rmsnorm(aux[i], model.norm, model.config.rms_norm_eps)[0])
                label = (pred == final).float()
            logit = self.tech.classifier.logit(aux[i].detach())
            weight = torch.where(label > 0, self.positive_weight, 1.0)
            losses.append(F.binary_cross_entropy_with_logits(logit, label, weight=weight))
        loss = torch.stack(losses).mean()
        return loss, {"loss": float(loss.detach())}
