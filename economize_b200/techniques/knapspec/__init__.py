"""KnapSpec self-drafting (``knapspec``; economize ``techniques/knapspec``): the draft skips attention and MLP
sublayers chosen by a 0/1 knapsack that keeps the most important sublayers within a latency budget.

* Latency model (decode is bound by bytes moved): an attention sublayer costs its projection weights plus the KV
  cache it reads at ``context`` tokens, an MLP sublayer its three projections; costs are in bytes.
* Importance: ``1 - cos`` between the full model's final hidden states and those with only that sublayer skipped,
  on calibration tokens.
* Selection: maximise kept importance subject to ``kept cost <= budget * total cost`` (dynamic programming over
  costs quantised to ``resolution`` units); the first and last ``keep_edges`` blocks are always kept whole.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import ClassVar

import torch

from ...core.technique import TechniqueConfig, register_technique
from ...errors import ConfigError
from .._self_draft import SelfDraftTechnique, layer_view
from ..layer_skip import _final_states

__all__ = ["KnapSpecConfig", "KnapSpecTechnique", "knapsack_keep", "sublayer_costs"]


@dataclass(frozen=True)
class KnapSpecConfig(TechniqueConfig):
    technique: ClassVar[str] = "knapspec"
    budget: float = 0.5
    context: int = 2048
    keep_edges: int = 1
    resolution: int = 2000

    def __post_init__(self) -> None:
        if not 0.0 < self.budget < 1.0:
            raise ConfigError(f"budget must lie in (0, 1), got {self.budget}")
        if self.context < 1 or self.resolution < 10:
            raise ConfigError("context must be >= 1 and resolution >= 10")


def sublayer_costs(config, context: int) -> tuple[float, float]:
    """Bytes one decode token moves through an attention and an MLP sublayer (bf16)."""
    h = config.hidden_size
    attn = 2 * (h * (config.q_size + 2 * config.kv_size) + config.q_size * h) + 2 * 2 * context * config.kv_size
    mlp = 2 * 3 * h * config.intermediate_size
    return float(attn), float(mlp)


def knapsack_keep(values: list[float], costs: list[float], capacity: float, resolution: int) -> list[bool]:
    """0/1 knapsack: which items to keep to maximise value within ``capacity`` (costs quantised)."""
    unit = max(capacity, 1e-9) / resolution
    w = [max(1, int(round(c / unit))) for c in costs]
    cap = resolution
    best = [[0.0] * (cap + 1) for _ in range(len(values) + 1)]
    for i, (v, wi) in enumerate(zip(values, w), start=1):
        row, prev = best[i], best[i - 1]
        for c in range(cap + 1):
            row[c] = prev[c]
            if wi <= c and prev[c - wi] + v > row[c]:
                row[c] = prev[c - wi] + v
    keep = [False] * len(values)
    c = cap
    for i in range(len(values), 0, -1):
        if best[i][c] != best[i - 1][c]:
            keep[i - 1] = True
            c -= w[i - 1]
    return keep


@register_technique
class KnapSpecTechnique(SelfDraftTechnique):
    config_class = KnapSpecConfig

    @torch.no_grad()
    def view_layers(self) -> list[tuple[int, bool, bool]]:
        cfg: KnapSpecConfig = self.config
        model = self.model
        n = model.config.num_layers
        batches = self.calibration_batches()
        ref = _final_states(model, batches)
        attn_cost, mlp_cost = sublayer_costs(model.config, cfg.context)
        items, values, costs = [], [], []
        for i in range(cfg.keep_edges, n - cfg.keep_edges):
            for kind in ("attn", "mlp"):
                spec = [(j, j == i and kind == "attn", j == i and kind == "mlp") for j in range(n)]
                h = _final_states(layer_view(model, spec), batches)
                drop = 1.0 - float(torch.nn.functional.cosine_similarity(h, ref, dim=-1).mean())
                items.append((i, kind))
                values.append(max(drop, 0.0))
                costs.append(attn_cost if kind == "attn" else mlp_cost)
        edges = 2 * cfg.keep_edges * (attn_cost + mlp_cost)
        total = n * (attn_cost + mlp_cost)
        capacity = max(cfg.budget * total - edges, 0.0)
        keep = knapsack_keep(values, costs, capacity, cfg.resolution)
        skip_attn = {i for (i, kind), k in zip(items, keep) if kind == "attn" and not k}
        skip_mlp = {i for (i, kind), k in zip(items, keep) if kind == "mlp" and not k}
        self.skipped = {"attn": sorted(skip_attn), "mlp": sorted(skip_mlp)}
        return [(i, i in skip_attn, i in skip_mlp) for i in range(n) if not (i in skip_attn and i in skip_mlp)]
