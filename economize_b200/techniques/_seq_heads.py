"""Sequentially dependent draft heads on the target's last hidden state (shared package of ``hydra`` and
``redrafter``).

The target state ``h_t`` of the last committed position and the embedding of the token the target chose after it
(the cycle's first token) start every draft; each further step reads the embedding of the token drafted before it.
The heads read out through the target's final norm and LM head. The drafter runs chains and dynamic trees through
the engine (``tree_step`` carries each node's state; the root's extended state lives in a buffer of its own), and
the ``step_distill`` objective trains the heads by teacher forcing against the frozen target's distributions.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn

from .. import ops
from ..core.technique import Capability, Family, Technique
from ..decoding.config import DecodeConfig
from ..errors import ConfigError
from ..runtime.cache import StepBatch
from ..train.objective import OBJECTIVES, Objective, OptimDefaults

__all__ = ["SequentialHeadTechnique", "SequentialHeadDrafter", "StepDistill"]


class SequentialHeadTechnique(Technique):
    """Subclasses define ``start(h, e) -> state`` (the root state from the target state and the first token's
    embedding), ``advance(state, e, depth) -> state`` and ``readout(state, depth) -> pre-norm hidden [.., H]``."""

    capabilities = Capability.DRAFTER
    family = Family.DRAFTER
    lossless = True
    objective_name = "step_distill"

    def embed(self, tokens: torch.Tensor) -> torch.Tensor:
        return self.model.embed_tokens(tokens.clamp_min(0))

    def logits(self, hidden: torch.Tensor) -> torch.Tensor:
        model = self.model
        normed, _ = ops.rmsnorm(hidden.to(model.dtype), model.norm, model.config.rms_norm_eps)
        return model.logits(normed).float()

    def drafter(self):
        return SequentialHeadDrafter(self)

    def max_steps(self) -> int:
        raise NotImplementedError

    def default_decoding(self) -> DecodeConfig:
        return DecodeConfig(cycle_length=min(self.max_steps(), 5) + 1)

    def source_states(self, h: torch.Tensor) -> torch.Tensor:
        """The states the heads start from, given the target's states ``[B, S, H]`` of a whole sequence (causal);
        the identity unless a subclass runs a layer of its own over them (Hydra++'s prefix layer)."""
        return h

    # teacher forcing: logits of step j (0-based) at every position t predict token t + j + 2
    def teacher_forced(self, h: torch.Tensor, tokens: torch.Tensor, steps: int) -> list[torch.Tensor]:
        s = tokens.shape[1]
        h = self.source_states(h)
        out = []
        state = self.start(h[:, : s - 1], self.embed(tokens[:, 1:]))  # position t with token t + 1
        for j in range(steps):
            n = s - 1 - j
            if n <= 1:
                break
            if j > 0:
                state = self.advance(state[:, :n], self.embed(tokens[:, 1 + j: 1 + j + n]), j)
            out.append(self.readout_logits(state[:, :n], j))
        return out

    def readout_logits(self, state: torch.Tensor, depth: int) -> torch.Tensor:
        return self.logits(self.readout(state, depth))


class SequentialHeadDrafter:
    def __init__(self, tech: SequentialHeadTechnique) -> None:
        self.tech = tech
        n = tech.model.config.num_layers
        self.capture_layers = (n,)  # the pre-norm stream after the last block
        self.carry_size = tech.model.config.hidden_size
        self.root_ext: torch.Tensor | None = None

    def begin(self, batch: int, capacity: int) -> None:
        pass

    def draft_depth(self, decode: DecodeConfig) -> int:
        k = max(1, decode.cycle_length - 1)
        if decode.draft_policy_name == "dynamic_tree":
            k = int(decode.draft_policy_options.get("depth", k))
        if k > self.tech.max_steps():
            raise ConfigError(f"{self.tech.name} drafts at most {self.tech.max_steps()} tokens per cycle")
        return k

    def draft_nodes(self, decode: DecodeConfig) -> int:
        return self.draft_depth(decode)

    def fuse(self, aux):
        return aux[self.capture_layers[0]]

    def observe(self, tokens, sources, kv_len, n_valid, root):
        rows = torch.arange(tokens.shape[0], device=tokens.device)
        h = sources[rows, root.long()]
        state = self.tech.start(h, self.tech.embed(tokens[rows, root.long()]))
        if self.root_ext is None or self.root_ext.shape != state.shape:
            self.root_ext = torch.zeros_like(state)
        self.root_ext.copy_(state)
        return self.tech.readout_logits(state, 0), h.to(self.tech.model.dtype)

    def tree_step(self, tokens, states, positions, kv_base, n_forwarded, q_offset, mask):
        batch, width = tokens.shape
        if states.shape[-1] == self.carry_size:  # children of the root: the root's extended state
            states = self.root_ext[:, None].expand(batch, width, self.root_ext.shape[-1])
        depth = self.tech.depth_of(states) + 1
        new = self.tech.advance(states, self.tech.embed(tokens), depth)
        return self.tech.readout_logits(new, depth), new

    def to_target(self, ids):
        return ids


@OBJECTIVES.register("step_distill")
class StepDistill(Objective):
    """KL from the frozen target's next-token distribution at ``t + j + 1`` to draft step ``j`` at ``t`` (teacher
    forcing with the real tokens), summed over steps: the distillation of Hydra++ and ReDrafter."""

    name = "step_distill"
    defaults = OptimDefaults(lr=1e-3, warmup_steps=10)

    def __init__(self, model, steps: int | None = None) -> None:
        super().__init__(model)
        tech = next((t for t in model.techniques.values() if isinstance(t, SequentialHeadTechnique)), None)
        if tech is None:
            raise ConfigError("step_distill trains the heads of an attached hydra or redrafter technique")
        self.tech = tech
        self.steps = steps or tech.max_steps()

    def parameters(self):
        return [p for p in self.tech.parameters() if p.requires_grad]

    def loss(self, tokens: torch.Tensor):
        tech = self.tech
        model = tech.model
        n = model.config.num_layers
        b, s = tokens.shape
        with torch.no_grad():
            cache = model.new_cache(b, ((s + 127) // 128) * 128)
            lengths = torch.full((b,), s, dtype=torch.int32, device=tokens.device)
            hidden, aux = model.forward_step(tokens, StepBatch.prefill(lengths, s), cache, capture=(n,))
            teacher = torch.log_softmax(model.logits(hidden).float(), -1)  # [B, S, V]: predicts t + 1
        outs = tech.teacher_forced(aux[n].detach(), tokens, self.steps)
        total, metrics = 0.0, {}
        for j, logits in enumerate(outs):
            m = logits.shape[1]
            target = teacher[:, j + 1: j + 1 + m]  # the target's distribution after token t + j + 1
            kl = F.kl_div(torch.log_softmax(logits.float(), -1), target, log_target=True, reduction="sum") / (b * m)
            total = total + kl
            with torch.no_grad():
                metrics[f"acc{j + 1}"] = float((logits.argmax(-1) == target.argmax(-1)).float().mean())
        loss = total / max(len(outs), 1)
        metrics["loss"] = float(loss.detach())
        return loss, metrics
