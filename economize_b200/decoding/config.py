"""User-facing decoding options (fields and semantics of economize's ``DecodeConfig``,
``src/economize/decoding/config.py:19-143``)."""

from __future__ import annotations

from collections.abc import Mapping
from dataclasses import dataclass, field, fields
from typing import Any

from ..errors import ConfigError
from ..validation import check_positive, check_unit_interval, known_fields

__all__ = ["DecodeConfig"]


def _frozen(value: Any) -> Any:
    if isinstance(value, list | tuple):
        return tuple(_frozen(v) for v in value)
    return value


@dataclass(frozen=True)
class DecodeConfig:
    """How a model with a drafting technique generates.

    One cycle runs the exact model once over the tokens not yet verified (yielding one exact token) and lets the
    drafter propose up to ``cycle_length - 1`` further tokens (or a tree under ``draft_policy="dynamic_tree"``).

    Attributes:
        cycle_length: Tokens per cycle; ``1`` is plain decoding.
        lossless: Verify drafts (default) or keep them all (``False``: the ``accept_all`` verifier).
        min_confidence: Stop a chain draft when the drafter's top probability falls below this value.
        verifier: Name of a registered verifier (``greedy``, ``rejection``, ``typical``, ``accept_all``).
        draft_policy: Name of a registered draft policy (``fixed``, ``confidence``, ``dynamic_tree``).
        verifier_options: Keyword options of the verifier.
        cuda_graphs: Record the whole cycle (draft, verify, accept, commit) as one CUDA graph per batch size and
            replay it; the host then only polls the generated lengths.
        sync_interval: Plain decoding reads results back every this many steps.
        record_confidence / record_distributions: Telemetry of the drafter's probabilities (kept for API parity).
        draft_loop_graph: Accepted for compatibility; the engine always graphs the whole cycle when
            ``cuda_graphs`` is on.
        draft_policy_options: Options of the draft policy (``{"depth": 6, "topk": 10, "total_tokens": 60}``).
        prefill_chunk: Prefill prompts in chunks of this many tokens.
        window_cache: Ring caches for sliding-window layers: the cache becomes a page pool and every windowed
            layer keeps a ring of pages covering its window (its memory follows the window, not the context);
            prompts longer than the ring's reserve are prefilled in chunks.
        kv_pages: Keep the KV cache in a pool of 128-slot pages addressed through per-layer page tables (the
            paged layout of serving engines; implied by ``window_cache``).
    """

    cycle_length: int = 4
    lossless: bool | None = None
    min_confidence: float | None = None
    verifier: str | None = None
    draft_policy: str | None = None
    verifier_options: Mapping[str, object] = field(default_factory=dict, hash=False)
    cuda_graphs: bool = False
    sync_interval: int = 8
    record_confidence: bool = False
    record_distributions: bool = False
    draft_loop_graph: bool = False
    draft_policy_options: Mapping[str, object] = field(default_factory=dict, hash=False)
    prefill_chunk: int | None = None
    window_cache: bool = False
    kv_pages: bool = False

    def __post_init__(self) -> None:
        check_positive("cycle_length", self.cycle_length)
        check_positive("sync_interval", self.sync_interval)
        if self.prefill_chunk is not None:
            check_positive("prefill_chunk", self.prefill_chunk)
        if self.min_confidence is not None:
            check_unit_interval("min_confidence", self.min_confidence, closed_high=True)
        for name in ("verifier_options", "draft_policy_options"):
            value = getattr(self, name)
            if not isinstance(value, Mapping):
                raise ConfigError(f"{name} must be a mapping, got {type(value).__name__}")
        object.__setattr__(self, "verifier_options", dict(self.verifier_options))
        object.__setattr__(self, "draft_policy_options",
                           {k: _frozen(v) for k, v in self.draft_policy_options.items()})

    def __hash__(self) -> int:
        skip = ("verifier_options", "draft_policy_options")
        return hash((*(getattr(self, f.name) for f in fields(self) if f.name not in skip),
                     *(tuple(sorted(getattr(self, n).items())) for n in skip)))

    @property
    def verifier_name(self) -> str:
        return self.verifier or ("accept_all" if self.lossless is False else "greedy")

    @property
    def draft_policy_name(self) -> str:
        return self.draft_policy or ("fixed" if self.min_confidence is None else "confidence")

    def to_dict(self) -> dict[str, Any]:
        data = {f.name: getattr(self, f.name) for f in fields(self)}
        data["verifier_options"] = dict(self.verifier_options)
        data["draft_policy_options"] = {k: list(v) if isinstance(v, tuple) else v
                                        for k, v in self.draft_policy_options.items()}
        return data

    @classmethod
    def from_dict(cls, data: Mapping[str, object]) -> DecodeConfig:
        return cls(**known_fields(cls.__name__, data, set(cls.__dataclass_fields__)))
