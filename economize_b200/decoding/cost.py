"""Cost accounting of a generation: one event per model call (economize ``decoding/cost.py``; the kind names, the
event fields and the summary keys are the reference's, so cost logs of both implementations compare).

The engine never stops the GPU to log: a cycle is one CUDA graph replay. It keeps one device word per row and
cycle (the drafts the cycle accepted, ``_State.acc_hist``), and after the generation :meth:`SpecEngine.cost_log`
turns the row's cycle history and the cycle's fixed shape (the draft steps and their widths, the verified tree
size, the drafter's observe pass) into the events below, positions included.
"""

from __future__ import annotations

from collections import Counter
from collections.abc import Iterable, Mapping
from dataclasses import dataclass, field, replace
from typing import Final, TypedDict

__all__ = ["CostEvent", "CostKind", "CostLog", "CostSummary", "LayerFootprint"]


class CostSummary(TypedDict):
    """The aggregate counts of :meth:`CostLog.summary`."""

    exact_calls: int
    exact_tokens: int
    draft_steps: int
    wasted_draft_steps: int
    replay_calls: int
    layer_tokens: int
    module_layer_tokens: dict[str, int]
    sequential_calls: int
    relative_layer_tokens: float


class CostKind:
    """Kinds of call (plain strings, so a technique may add its own)."""

    EXACT: Final = "exact"                  # the unmodified model over one or more tokens
    DRAFT: Final = "draft"                  # one draft step
    DRAFT_WASTED: Final = "draft_wasted"    # a draft step whose proposal was discarded
    REPLAY: Final = "replay"                # exact tokens run again to rebuild recurrent state
    DRAFT_CATCHUP: Final = "draft_catchup"  # a separate draft network over committed tokens before drafting
    DRAFT_OBSERVE: Final = "draft_observe"  # a draft module over committed tokens to update its cache


@dataclass(frozen=True)
class LayerFootprint:
    """The decoder layers one call runs: ``first_layer .. last_layer`` (1-indexed; empty when ``last_layer <
    first_layer``) of the decoded model (``module=None``) or of a separate network named ``module``; ``layers``
    lists them when they are not one range."""

    first_layer: int
    last_layer: int
    module: str | None = None
    layers: tuple[int, ...] | None = None

    @classmethod
    def of(cls, layers: Iterable[int], module: str | None = None) -> LayerFootprint:
        chosen = sorted(set(int(i) for i in layers))
        if not chosen:
            return cls(1, 0, module)
        if chosen == list(range(chosen[0], chosen[-1] + 1)):
            return cls(chosen[0], chosen[-1], module)
        return cls(chosen[0], chosen[-1], module, tuple(chosen))

    @classmethod
    def none(cls, module: str | None = None) -> LayerFootprint:
        return cls(1, 0, module)

    @classmethod
    def all(cls, num_layers: int, module: str | None = None) -> LayerFootprint:
        return cls(1, num_layers, module)


@dataclass(frozen=True)
class CostEvent:
    """One model call: its kind, the tokens it processed in parallel, the position of the first, the layers it
    ran (see :class:`LayerFootprint`) and, for a draft step, its index within the cycle."""

    kind: str
    tokens: int
    position: int
    first_layer: int
    last_layer: int
    step: int | None = None
    module: str | None = None
    layers: tuple[int, ...] | None = None

    @property
    def layer_indices(self) -> tuple[int, ...]:
        if self.layers is not None:
            return self.layers
        return tuple(range(max(1, self.first_layer), self.last_layer + 1))

    @property
    def layer_tokens(self) -> int:
        """Decoder-layer applications: the unit in which calls are compared."""
        return self.tokens * len(self.layer_indices)


@dataclass
class CostLog:
    """The model calls of one row's generation, in order."""

    events: list[CostEvent] = field(default_factory=list)

    def record(self, kind: str, tokens: int, position: int, first_layer: int, last_layer: int,
               step: int | None = None, *, module: str | None = None, layers: tuple[int, ...] | None = None) -> None:
        self.events.append(CostEvent(kind, tokens, position, first_layer, last_layer, step, module, layers))

    def record_footprint(self, kind: str, tokens: int, position: int, footprint: LayerFootprint,
                         step: int | None = None) -> None:
        self.record(kind, tokens, position, footprint.first_layer, footprint.last_layer, step,
                    module=footprint.module, layers=footprint.layers)

    def mark_last_wasted(self) -> None:
        last = self.events[-1]
        self.events[-1] = replace(last, kind=f"{last.kind}_wasted")

    def truncate(self, length: int) -> None:
        del self.events[length:]

    def count(self, kind: str) -> int:
        return sum(e.kind == kind for e in self.events)

    def summary(self, num_layers: int, prompt_tokens: int, generated: int) -> CostSummary:
        """Totals, with the decoded model's layer applications relative to plain decoding of the same output
        (``(prompt_tokens + generated - 1) * num_layers``); separate networks are counted per module."""
        own = [e for e in self.events if e.module is None]
        per_module: Counter[str] = Counter()
        for e in self.events:
            if e.module is not None:
                per_module[e.module] += e.layer_tokens
        layer_tokens = sum(e.layer_tokens for e in own)
        baseline = max(1, (prompt_tokens + generated - 1) * num_layers)
        exact = [e for e in self.events if e.kind == CostKind.EXACT]
        return {"exact_calls": len(exact), "exact_tokens": sum(e.tokens for e in exact),
                "draft_steps": self.count(CostKind.DRAFT), "wasted_draft_steps": self.count(CostKind.DRAFT_WASTED),
                "replay_calls": self.count(CostKind.REPLAY), "layer_tokens": layer_tokens,
                "module_layer_tokens": dict(per_module), "sequential_calls": len(self.events),
                "relative_layer_tokens": layer_tokens / baseline}

    def as_tuples(self, kinds: Mapping[str, str] | None = None) -> list[tuple[str, int, int]]:
        """``(kind, tokens, position)`` per event, kinds renamed by ``kinds`` (to compare with another decoder)."""
        rename = kinds or {}
        return [(rename.get(e.kind, e.kind), e.tokens, e.position) for e in self.events]

    def __len__(self) -> int:
        return len(self.events)
