"""``prune`` and ``depth_prune`` techniques."""

from __future__ import annotations

import dataclasses

import torch
from torch import nn

from ...core.technique import Capability, Family, Technique, register_technique
from ...errors import ConfigError
from ...ops.quant import install
from ...ops.sparse import Sparse24Weight
from ...runtime.cache import StepBatch
from .._self_draft import block_influence
from ..quant.config import PROJECTIONS
from ..quant.methods import collect
from ..quant.technique import _key, _selected
from . import methods
from .config import DepthPruneConfig, PruneConfig, parse_sparsity

__all__ = ["DepthPruneTechnique", "PruneTechnique"]


def _batches(cal) -> list[torch.Tensor]:
    if cal is None:
        return []
    return [cal if cal.dim() == 2 else cal[None]] if isinstance(cal, torch.Tensor) else [torch.as_tensor(c) for c in cal]


@register_technique
class PruneTechnique(Technique):
    config_class = PruneConfig
    capabilities = Capability.WEIGHTS
    family = Family.PRUNING
    lossless = False

    def __init__(self, config: PruneConfig, model) -> None:
        super().__init__(config, model)
        self._calibration = None
        self.weights = nn.ModuleDict()     # compressed 2:4 projections
        self.masks: dict[str, torch.Tensor] = {}  # other projections: keep masks (weights are zeroed in place)

    def calibrate(self, calibration) -> None:
        self._calibration = calibration

    def _targets(self) -> dict[int, list[str]]:
        cfg: PruneConfig = self.config
        layers = [i - 1 for i in cfg.layers] if cfg.layers else range(self.model.config.num_layers)
        return {i: [n for n, hf in PROJECTIONS.items() if _selected(hf, cfg.targets, cfg.exclude)
                    and getattr(self.model.layers[i], n).dim() == 2] for i in layers}

    @torch.no_grad()
    def attach(self) -> None:
        cfg: PruneConfig = self.config
        model = self.model
        frac, nm = parse_sparsity(cfg.sparsity)
        store24 = (cfg.semi_structured is not False) and nm == (2, 4)
        if not self.weights and not self.masks:
            wanted = self._targets()
            stats = None
            if cfg.needs_calibration:
                batches = _batches(self._calibration)
                if not batches:
                    raise ConfigError(f"prune method={cfg.method!r} needs calibration tokens")
                stats = collect(model, batches, wanted, hessian=cfg.method == "sparsegpt",
                                keep_rows=cfg.calibration_tokens)
            for i, names in wanted.items():
                layer = model.layers[i]
                for name in names:
                    w = getattr(layer, name).detach()
                    if cfg.method == "sparsegpt":
                        pruned, keep = methods.sparsegpt(w, stats[(i, name)].hessian, frac, nm, cfg.blocksize,
                                                         cfg.percdamp)
                    else:
                        if cfg.method == "wanda":
                            s = stats[(i, name)]
                            col = (s.h.diagonal() if s.h is not None else None)
                            norm = torch.sqrt(col) if col is not None else torch.sqrt(
                                (s.sample.float() ** 2).sum(0))
                            score = methods.wanda_scores(w, norm)
                        else:
                            score = methods.magnitude_scores(w)
                        keep = methods.nm_mask(score, *nm) if nm else methods.unstructured_mask(score, frac)
                        pruned = w * keep
                    if store24 and w.shape[1] % 64 == 0 and w.shape[0] % 2 == 0:
                        self.weights[_key(i, name)] = Sparse24Weight.from_dense(pruned, keep)
                    else:
                        getattr(layer, name).copy_(pruned)
                        self.masks[_key(i, name)] = keep
        for key, sw in self.weights.items():
            i, name = key.split(":")
            install(model.layers[int(i)], name, sw.to(model.device))

    def inplace_targets(self) -> list[torch.Tensor]:
        """Unstructured and N:M pruning write the masked weights into the existing projections."""
        if not hasattr(self, "_targets"):
            return []
        out = []
        for i, names in self._targets().items():
            layer = self.model.layers[i]
            out += [getattr(layer, n) for n in names if isinstance(getattr(layer, n), torch.Tensor)]
        return out

    def technique_state(self) -> dict[str, torch.Tensor]:
        out = {}
        for key, sw in self.weights.items():
            out[f"weights.{key}.values"] = sw.values
            out[f"weights.{key}.meta"] = sw.meta
        for key, m in self.masks.items():
            out[f"masks.{key}"] = m
        return out

    def load_technique_state(self, state: dict[str, torch.Tensor]) -> None:
        found: dict[str, dict[str, torch.Tensor]] = {}
        for name, t in state.items():
            kind, rest = name.split(".", 1)
            if kind == "weights":
                key, buf = rest.rsplit(".", 1)
                found.setdefault(key, {})[buf] = t
            elif kind == "masks":
                self.masks[rest] = t.bool()
        for key, bufs in found.items():
            self.weights[key] = Sparse24Weight(bufs["values"], bufs["meta"])

    def sparsity(self) -> float:
        """Fraction of zeros over the pruned projections."""
        zeros = total = 0
        for sw in self.weights.values():
            total += sw.out_features * sw.in_features
            zeros += sw.out_features * sw.in_features - int((sw.values != 0).sum())
        for key, m in self.masks.items():
            total += m.numel()
            zeros += int((~m).sum())
        return zeros / max(total, 1)


@register_technique
class DepthPruneTechnique(Technique):
    """Remove decoder blocks (ShortGPT, SLEB); the model's depth changes, so it attaches before every other
    technique is built."""

    config_class = DepthPruneConfig
    capabilities = Capability.WEIGHTS
    family = Family.DEPTH
    lossless = False

    def __init__(self, config: DepthPruneConfig, model) -> None:
        super().__init__(config, model)
        self._calibration = None
        self.removed: list[int] = [i - 1 for i in config.layers]

    def calibrate(self, calibration) -> None:
        self._calibration = calibration

    def conflicts(self, other) -> str | None:
        return None

    def _candidates(self, n: int) -> list[int]:
        cfg = self.config
        first = 1 if cfg.keep_first is None else cfg.keep_first
        last = 1 if cfg.keep_last is None else cfg.keep_last
        return list(range(first, n - last))

    @torch.no_grad()
    def _nll(self, keep: list[int], batches) -> float:
        from .._self_draft import layer_view

        view = layer_view(self.model, keep)
        total, count = 0.0, 0
        for tokens in batches:
            tokens = tokens.to(self.model.device)
            b, length = tokens.shape
            cache = view.new_cache(b, ((length + 127) // 128) * 128)
            lengths = torch.full((b,), length, dtype=torch.int32, device=tokens.device)
            h, _ = view.forward_step(tokens, StepBatch.prefill(lengths, length), cache)
            logits = view.logits(h[:, :-1]).float()
            total += float(torch.nn.functional.cross_entropy(logits.reshape(-1, logits.shape[-1]),
                                                             tokens[:, 1:].reshape(-1), reduction="sum"))
            count += b * (length - 1)
        return total / max(count, 1)

    @torch.no_grad()
    def _choose(self) -> list[int]:
        cfg: DepthPruneConfig = self.config
        n = self.model.config.num_layers
        batches = _batches(self._calibration)
        if not batches:
            raise ConfigError("depth_prune needs calibration tokens (or layers=) to choose the blocks")
        cand = self._candidates(n)
        if cfg.method == "shortgpt":
            bi = block_influence(self.model, batches)
            return sorted(sorted(cand, key=lambda i: float(bi[i]))[: cfg.num_blocks])
        removed: list[int] = []
        for _ in range(cfg.num_blocks):
            best = min((i for i in cand if i not in removed),
                       key=lambda i: self._nll([j for j in range(n) if j not in removed and j != i], batches))
            removed.append(best)
        return sorted(removed)

    @torch.no_grad()
    def attach(self) -> None:
        model = self.model
        if not self.removed:
            self.removed = self._choose()
        keep = [i for i in range(model.config.num_layers) if i not in set(self.removed)]
        model.layers = nn.ModuleList(model.layers[i] for i in keep)
        model.config = dataclasses.replace(model.config, num_layers=len(keep))
        if model.kv_scales is not None:
            model.kv_scales = tuple(s[keep].contiguous() for s in model.kv_scales)
        object.__setattr__(self.config, "layers", tuple(i + 1 for i in self.removed))

    def technique_state(self) -> dict[str, torch.Tensor]:
        return {"removed": torch.tensor(self.removed, dtype=torch.int64)}

    def load_technique_state(self, state: dict[str, torch.Tensor]) -> None:
        self.removed = [int(i) for i in state["removed"].tolist()]
