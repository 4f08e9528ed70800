"""Draft policies: how many tokens a proposal drafts and in which shape (economize
``src/economize/decoding/policies.py`` and ``dynamic_tree.py``).

* ``fixed``: a chain of ``cycle_length - 1`` drafts.
* ``confidence``: a chain that stops where the drafter's top probability falls below ``min_confidence`` (the first
  draft is always made). The engine keeps its shapes fixed: drafts after the stop are invalidated, so they are
  never accepted and the acceptance statistics are those of the shortened chain.
* ``dynamic_tree``: EAGLE-2 dynamic trees (``depth``, ``topk``, ``total_tokens``).
* ``sequoia``: one static tree of the best shape for measured acceptance rates (economize ``decoding/sequoia.py``).
* ``specexec``: SpecExec best-first search over a candidate pool (economize ``decoding/specexec.py``).
"""

from __future__ import annotations

from typing import Any, ClassVar

from ..errors import ConfigError
from ..registry import Registry
from .tree import TreeOptions

__all__ = ["POLICIES", "ConfidencePolicy", "DraftPolicy", "DynamicTreePolicy", "FixedPolicy", "SequoiaPolicy",
           "SpecExecPolicy"]


class DraftPolicy:
    name: ClassVar[str] = ""
    drafts_tree: ClassVar[bool] = False

    def __init__(self, config: Any) -> None:
        self.config = config


POLICIES: Registry[type[DraftPolicy]] = Registry("draft policy", "economize_b200.policies")


@POLICIES.register("fixed")
class FixedPolicy(DraftPolicy):
    name = "fixed"


@POLICIES.register("confidence")
class ConfidencePolicy(DraftPolicy):
    name = "confidence"

    def __init__(self, config: Any) -> None:
        super().__init__(config)
        if config.min_confidence is None:
            raise ConfigError("draft_policy 'confidence' needs DecodeConfig.min_confidence")
        self.min_confidence = float(config.min_confidence)


@POLICIES.register("dynamic_tree")
class DynamicTreePolicy(DraftPolicy):
    name = "dynamic_tree"
    drafts_tree = True

    def __init__(self, config: Any) -> None:
        super().__init__(config)
        self.options = TreeOptions.from_options(config.draft_policy_options, config.cycle_length)


@POLICIES.register("sequoia")
class SequoiaPolicy(DraftPolicy):
    """One static Sequoia tree per cycle (options: ``acceptance`` or ``paths``, ``total_tokens``, ``depth``,
    ``verify_latency``, ``draft_latency``, ``record_acceptance``; :mod:`economize_b200.decoding.sequoia`)."""

    name = "sequoia"
    drafts_tree = True

    def __init__(self, config: Any) -> None:
        from .sequoia import tree_from_options

        super().__init__(config)
        self.tree, self.record = tree_from_options(config.draft_policy_options, config.cycle_length)


@POLICIES.register("specexec")
class SpecExecPolicy(DraftPolicy):
    """SpecExec best-first search (options: ``depth``, ``width``, ``topk``, ``total_tokens``, ``decay``;
    :mod:`economize_b200.decoding.specexec`)."""

    name = "specexec"
    drafts_tree = True

    def __init__(self, config: Any) -> None:
        from .specexec import SearchOptions

        super().__init__(config)
        self.options = SearchOptions.from_options(config.draft_policy_options, config.cycle_length)
