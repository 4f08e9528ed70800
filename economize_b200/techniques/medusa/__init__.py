"""Medusa heads (``medusa``; Cai et al. 2024, economize ``techniques/medusa``).

Head ``j`` maps the target's last hidden state at the last processed token through ``num_layers`` residual blocks
``x + SiLU(W x + b)`` and a vocabulary projection, drafting the token ``j + 1`` places after the LM head's. A
cycle's draft is a static tree over the heads' ranked candidates (``tree``: a name in :data:`MEDUSA_TREES` or
explicit paths; without one, the chain of every head's top candidate). Parameter names are economize's
(``heads.{i}.blocks.{j}.linear``, ``heads.{i}.proj``).
"""

from __future__ import annotations

from collections.abc import Sequence
from dataclasses import dataclass
from typing import ClassVar

import torch
import torch.nn.functional as F
from torch import nn

from ... import ops
from ...core.technique import Capability, Family, Technique, TechniqueConfig, register_technique
from ...decoding.config import DecodeConfig
from ...errors import ConfigError, UnknownNameError
from ...registry import Registry
from ...validation import check_choice, check_positive

__all__ = ["MEDUSA_TREES", "MedusaConfig", "MedusaDrafter", "MedusaTechnique", "normalize_paths"]

Paths = tuple[tuple[int, ...], ...]
MEDUSA_TREES: Registry[Paths] = Registry("Medusa tree", "economize_b200.medusa_trees")

# The 63-node sparse tree "mc_sim_7b_63" published with Medusa (FasterDecoding/Medusa medusa_choices.py), kept
# identical so trees tuned for Medusa checkpoints apply unchanged: path (r1, .., rj) is head j's rank-rj candidate
# under the node (r1, .., r(j-1)).
MEDUSA_TREES.register("mc_sim_7b_63", tuple(tuple(p) for p in (
    (0,), (0, 0), (1,), (0, 1), (2,), (0, 0, 0), (1, 0), (0, 2), (3,), (0, 3), (4,), (0, 4), (2, 0), (0, 5),
    (0, 0, 1), (5,), (0, 6), (6,), (0, 7), (0, 1, 0), (1, 1), (7,), (0, 8), (0, 0, 2), (3, 0), (0, 9), (8,), (9,),
    (1, 0, 0), (0, 2, 0), (1, 2), (0, 0, 3), (4, 0), (2, 1), (0, 0, 4), (0, 0, 5), (0, 0, 0, 0), (0, 1, 1),
    (0, 0, 6), (0, 3, 0), (5, 0), (1, 3), (0, 0, 7), (0, 0, 8), (0, 0, 9), (6, 0), (0, 4, 0), (1, 4), (7, 0),
    (0, 1, 2), (2, 0, 0), (3, 1), (2, 2), (8, 0), (0, 5, 0), (1, 5), (1, 0, 1), (0, 2, 1), (9, 0), (0, 6, 0),
    (0, 0, 0, 1), (1, 6), (0, 7, 0))))


def normalize_paths(paths: Sequence[Sequence[int]]) -> Paths:
    out = tuple(tuple(int(r) for r in p) for p in paths)
    seen = set(out)
    if not out or len(seen) != len(out):
        raise ConfigError("a Medusa tree needs distinct, non-empty paths")
    for p in out:
        if not p or min(p) < 0 or (len(p) > 1 and p[:-1] not in seen):
            raise ConfigError(f"invalid Medusa tree path {p}")
    return out


@dataclass(frozen=True)
class MedusaConfig(TechniqueConfig):
    technique: ClassVar[str] = "medusa"
    num_heads: int = 5
    num_layers: int = 1
    head: str = "own"
    tree: str | Paths | None = None
    param_dtype: str = "model"

    def __post_init__(self) -> None:
        check_positive("num_heads", self.num_heads)
        check_positive("num_layers", self.num_layers)
        check_choice("head", self.head, ("own", "shared"))
        check_choice("param_dtype", self.param_dtype, ("model", "float32", "bfloat16", "float16"))
        if self.tree is not None:
            paths = self.paths
            if max(len(p) for p in paths) > self.num_heads:
                raise ConfigError(f"the Medusa tree is deeper than the {self.num_heads} heads")
            if not isinstance(self.tree, str):
                object.__setattr__(self, "tree", paths)

    @property
    def paths(self) -> Paths | None:
        if self.tree is None:
            return None
        if isinstance(self.tree, str):
            try:
                return MEDUSA_TREES.get(self.tree)
            except UnknownNameError as err:
                raise ConfigError(str(err)) from None
        return normalize_paths(self.tree)


class ResBlock(nn.Module):
    def __init__(self, hidden: int, dtype: torch.dtype, device) -> None:
        super().__init__()
        self.linear = nn.Linear(hidden, hidden, dtype=dtype, device=device)
        nn.init.zeros_(self.linear.weight)


class MedusaHead(nn.Module):
    def __init__(self, hidden: int, vocab: int, layers: int, own: bool, dtype: torch.dtype, device) -> None:
        super().__init__()
        self.blocks = nn.ModuleList(ResBlock(hidden, dtype, device) for _ in range(layers))
        self.proj = nn.Linear(hidden, vocab, bias=False, dtype=dtype, device=device) if own else None

    def hidden(self, x: torch.Tensor) -> torch.Tensor:
        for block in self.blocks:
            x = x + F.silu(ops.linear(x, block.linear.weight, block.linear.bias))
        return x


@register_technique
class MedusaTechnique(Technique):
    config_class = MedusaConfig
    capabilities = Capability.DRAFTER
    family = Family.DRAFTER
    objective_name = "medusa_ce"

    def __init__(self, config: MedusaConfig, model) -> None:
        super().__init__(config, model)
        c = model.config
        dtype = model.dtype if config.param_dtype == "model" else getattr(torch, config.param_dtype)
        own = config.head == "own"
        self.heads = nn.ModuleList(MedusaHead(c.hidden_size, c.vocab_size, config.num_layers, own, dtype,
                                              model.device) for _ in range(config.num_heads))
        if own:
            with torch.no_grad():
                for h in self.heads:
                    h.proj.weight.copy_(model.head_weight.detach().to(dtype))

    def head_logits(self, states: torch.Tensor) -> torch.Tensor:
        """``[..., K, V]`` fp32 logits of every head for target states ``[..., H]`` (post-norm for own heads,
        pre-norm for shared ones)."""
        model = self.model
        out = []
        for h in self.heads:
            x = h.hidden(states.to(h.blocks[0].linear.weight.dtype) if len(h.blocks) else states)
            if h.proj is not None:
                out.append(ops.linear(x, h.proj.weight).float())
            else:
                normed, _ = ops.rmsnorm(x.to(model.dtype), model.norm, model.config.rms_norm_eps)
                out.append(model.logits(normed).float())
        return torch.stack(out, -2)

    def drafter(self) -> MedusaDrafter:
        return MedusaDrafter(self)

    def default_decoding(self) -> DecodeConfig:
        return DecodeConfig(cycle_length=self.config.num_heads + 1)


class MedusaDrafter:
    """Static-tree drafter: ``observe`` ranks every head's candidates at the last processed token, ``propose``
    gathers the tree's tokens from those ranks (one gather, the parents are fixed)."""

    def __init__(self, technique: MedusaTechnique) -> None:
        self.t = technique
        self.own = technique.config.head == "own"
        self.capture_layers = (-1,) if self.own else (technique.model.config.num_layers,)
        self.carry_size = technique.model.config.hidden_size
        self.top: torch.Tensor | None = None
        self.paths: Paths = ()

    def draft_depth(self, decode: DecodeConfig) -> int:
        paths = self.t.config.paths
        if paths is None:
            k = min(self.t.config.num_heads, max(1, decode.cycle_length - 1))
            paths = tuple((0,) * d for d in range(1, k + 1))
        self.paths = paths
        return max(len(p) for p in paths)

    def draft_nodes(self, decode: DecodeConfig) -> int:
        self.draft_depth(decode)
        return len(self.paths)

    @property
    def ranks(self) -> int:
        return 1 + max(max(p) for p in self.paths)

    def begin(self, batch: int, capacity: int) -> None:
        dev = self.t.model.device
        k = self.t.config.num_heads
        if self.top is None or self.top.shape[0] != batch:
            self.top = torch.zeros(batch, k, self.ranks, dtype=torch.int64, device=dev)
        index = {p: i for i, p in enumerate(self.paths)}
        self._gather = torch.tensor([(len(p) - 1) * self.ranks + p[-1] for p in self.paths], device=dev)
        self._parents = torch.tensor([index[p[:-1]] if len(p) > 1 else -1 for p in self.paths], device=dev)

    def fuse(self, aux: dict[int, torch.Tensor]) -> torch.Tensor:
        return aux[self.capture_layers[0]]

    def observe(self, tokens: torch.Tensor, sources: torch.Tensor, kv_len: torch.Tensor, n_valid: torch.Tensor,
                root: torch.Tensor) -> tuple[torch.Tensor | None, torch.Tensor | None]:
        rows = torch.arange(tokens.shape[0], device=tokens.device)
        state = sources[rows, root.long()]  # the target state of the last processed token
        logits = self.t.head_logits(state)  # [B, K, V]
        self.top.copy_(logits.topk(self.ranks, -1).indices)
        return None, None

    def propose(self, history: torch.Tensor, length: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        batch = self.top.shape[0]
        tokens = self.top.reshape(batch, -1)[:, self._gather]
        return tokens, self._parents.expand(batch, -1).contiguous()

    def to_target(self, ids: torch.Tensor) -> torch.Tensor:
        return ids
