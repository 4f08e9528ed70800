"""Hybrid drafting (``hybrid``; economize ``techniques/hybrid``): a model-free primary proposer (the built-in prompt
lookup, or another static proposer such as ``suffix_decoding``) and a model drafter as the fallback. Each cycle the
fallback drafts every row and the primary's proposal replaces it in the rows where the primary found a match (its
first token is valid); the target verifies whatever each row holds in one pass.

In the engine the batch drafts as one captured computation, so the fallback's draft steps run for every row; the
gain is the acceptance of the copied tokens where the lookup matches (long verbatim spans), not skipped draft
compute. With a rejection-sampling verifier the copied tokens count as a deterministic proposal (one-hot draft
distribution), which keeps the verification lossless.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, ClassVar

import torch
import torch.nn.functional as F
from torch import nn

from ...core.technique import Capability, Family, Technique, TechniqueConfig, register_technique, technique_for
from ...decoding.config import DecodeConfig
from ...errors import ConfigError
from ...validation import check_choice, check_positive
from ..lookup import LookupConfig, LookupDrafter

__all__ = ["HybridConfig", "HybridDrafter", "HybridTechnique"]


def _nested(value, name: str):
    from ...core.serialization import nested_config

    if value is None or isinstance(value, TechniqueConfig):
        return value
    if isinstance(value, dict):
        return nested_config(value)
    raise ConfigError(f"{name} must be a technique configuration, got {type(value).__name__}")


@dataclass(frozen=True)
class HybridConfig(TechniqueConfig):
    """Prompt lookup (or ``primary``) with a fallback drafter.

    Attributes:
        fallback: Configuration of the model drafter used where the primary proposes nothing (e.g.
            ``Eagle3Config()``); its state is saved with the hybrid under ``fallback.``.
        max_ngram, min_ngram, max_proposal, match: The built-in lookup (see ``LookupConfig``).
        max_drafts: Most tokens kept from the fallback per row and cycle (default: its full budget).
        primary: A static proposer's configuration in place of the built-in lookup (n-gram fields stay default).
    """

    technique: ClassVar[str] = "hybrid"
    fallback: Any = None
    max_ngram: int = 3
    min_ngram: int = 1
    max_proposal: int | None = None
    max_drafts: int | None = None
    match: str = "earliest"
    primary: Any = None

    def __post_init__(self) -> None:
        object.__setattr__(self, "fallback", _nested(self.fallback, "fallback"))
        object.__setattr__(self, "primary", _nested(self.primary, "primary"))
        if self.fallback is None:
            raise ConfigError("hybrid needs a fallback drafter configuration (e.g. fallback=Eagle3Config())")
        for role, cfg in (("fallback", self.fallback), ("primary", self.primary)):
            if cfg is not None and Capability.DRAFTER not in technique_for(cfg).capabilities:
                raise ConfigError(f"hybrid {role} {cfg.technique!r} is not a drafting technique")
        if self.fallback.technique in ("hybrid", "lookup"):
            raise ConfigError(f"hybrid fallback must be a model drafter, not {self.fallback.technique!r}")
        check_positive("max_ngram", self.max_ngram)
        check_positive("min_ngram", self.min_ngram)
        if self.min_ngram > self.max_ngram:
            raise ConfigError("min_ngram exceeds max_ngram")
        check_choice("match", self.match, ("earliest", "latest"))
        for name in ("max_proposal", "max_drafts"):
            if getattr(self, name) is not None:
                check_positive(name, getattr(self, name))
        if self.primary is not None and (self.max_ngram, self.min_ngram, self.max_proposal, self.match) != \
                (3, 1, None, "earliest"):
            raise ConfigError("the n-gram fields configure the built-in lookup; a hybrid with a primary drafter keeps "
                              "them at their defaults")

    def lookup_config(self) -> LookupConfig:
        return LookupConfig(self.max_ngram, self.min_ngram, self.max_proposal, self.match)

    def to_dict(self) -> dict[str, Any]:
        from ...core.serialization import nested_dict

        out = super().to_dict()
        out["fallback"] = nested_dict(self.fallback)
        out["primary"] = None if self.primary is None else nested_dict(self.primary)
        return out

    def validate(self, model) -> None:
        self.fallback.validate(model)
        if self.primary is not None:
            self.primary.validate(model)


class HybridDrafter:
    """The fallback drafter with the primary's proposals laid over it (:meth:`overlay`, called by the engine after
    drafting); every other call goes to the fallback."""

    def __init__(self, fallback, primary, max_drafts: int | None) -> None:
        self.fallback = fallback
        self.primary = primary
        self.max_drafts = max_drafts
        self.graph_safe = getattr(fallback, "graph_safe", True) and getattr(primary, "graph_safe", True)
        self.depth = 1

    def __getattr__(self, name: str):
        return getattr(self.__dict__["fallback"], name)

    def draft_depth(self, decode: DecodeConfig) -> int:
        self.depth = self.fallback.draft_depth(decode)
        if self.primary.draft_depth(decode) > self.depth:
            raise ConfigError("the hybrid's primary proposes deeper than its fallback drafts; lower its budget")
        return self.depth

    def draft_nodes(self, decode: DecodeConfig) -> int:
        n = self.fallback.draft_nodes(decode)
        if self.primary.draft_nodes(decode) > n:
            raise ConfigError("the hybrid's primary proposes more nodes than its fallback drafts")
        return n

    def overlay(self, history: torch.Tensor, length: torch.Tensor, tokens: torch.Tensor, parents: torch.Tensor,
                q_full: torch.Tensor | None):
        batch, width = tokens.shape
        p_tok, p_par = self.primary.propose(history, length)
        n = p_tok.shape[1]
        if self.max_drafts is not None:  # cap the fallback's drafts (chains: by position; trees: by depth)
            depth = torch.zeros_like(parents)
            for j in range(width):
                par = parents[:, j]
                depth[:, j] = torch.where(par >= 0, depth.gather(1, par.clamp_min(0)[:, None])[:, 0] + 1, 1)
            tokens = tokens.masked_fill(depth > self.max_drafts, -1)
        pad_t = torch.full((batch, width - n), -1, dtype=tokens.dtype, device=tokens.device)
        pad_p = torch.full((batch, width - n), -1, dtype=parents.dtype, device=parents.device)
        p_tok = torch.cat([p_tok.to(tokens.dtype), pad_t], 1)
        p_par = torch.cat([p_par.to(parents.dtype), pad_p], 1)
        hit = (p_tok[:, 0] >= 0)[:, None]
        tokens = torch.where(hit, p_tok, tokens)
        parents = torch.where(hit, p_par, parents)
        if q_full is not None:
            onehot = F.one_hot(p_tok[:, : q_full.shape[1]].clamp_min(0), q_full.shape[-1]).to(q_full.dtype)
            q_full = torch.where(hit[..., None], onehot, q_full)
        return tokens, parents, q_full


@register_technique
class HybridTechnique(Technique):
    """Holds the fallback (and primary) techniques as submodules; the fallback's state is saved under
    ``fallback.``."""

    config_class = HybridConfig
    capabilities = Capability.DRAFTER
    family = Family.DRAFTER
    lossless = True

    def __init__(self, config: HybridConfig, model) -> None:
        super().__init__(config, model)
        self.fallback = technique_for(config.fallback)(config.fallback, model)
        self.primary = technique_for(config.primary)(config.primary, model) if config.primary is not None else None
        self.graph_safe = self.fallback.graph_safe and (self.primary is None or self.primary.graph_safe)

    @property
    def wrapped_drafter(self) -> Technique:
        return self.fallback

    def calibrate(self, calibration) -> None:
        for t in (self.fallback, self.primary):
            if t is not None and hasattr(t, "calibrate"):
                t.calibrate(calibration)

    def attach(self) -> None:
        self.fallback.attach()
        if self.primary is not None:
            self.primary.attach()

    def detach(self) -> None:
        self.fallback.detach()
        if self.primary is not None:
            self.primary.detach()

    def drafter(self):
        primary = self.primary.drafter() if self.primary is not None else LookupDrafter(self.config.lookup_config())
        return HybridDrafter(self.fallback.drafter(), primary, self.config.max_drafts)

    def default_decoding(self) -> DecodeConfig | None:
        return self.fallback.default_decoding()

    def technique_state(self) -> dict[str, torch.Tensor]:
        out = {f"fallback.{k}": v for k, v in self.fallback.technique_state().items()}
        if self.primary is not None:
            out.update({f"primary.{k}": v for k, v in self.primary.technique_state().items()})
        return out

    def export_state(self) -> dict[str, torch.Tensor]:
        out = {f"fallback.{k}": v for k, v in self.fallback.export_state().items()}
        if self.primary is not None:
            out.update({f"primary.{k}": v for k, v in self.primary.export_state().items()})
        return out

    def load_technique_state(self, state: dict[str, torch.Tensor]) -> None:
        fb = {k[len("fallback."):]: v for k, v in state.items() if k.startswith("fallback.")}
        pr = {k[len("primary."):]: v for k, v in state.items() if k.startswith("primary.")}
        rest = sorted(k for k in state if not k.startswith(("fallback.", "primary.")))
        if rest:
            raise ConfigError(f"hybrid: unexpected tensors {rest[:5]}")
        self.fallback.load_technique_state(fb)
        if self.primary is not None and pr:
            self.primary.load_technique_state(pr)
