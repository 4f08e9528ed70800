"""Exporters for SGLang's draft models (economize ``backends/sglang/export.py:309``).

SGLang's EAGLE-3 worker (``--speculative-algorithm EAGLE3 --speculative-draft-model-path <folder>``) reads the same
published EAGLE-3 layout as vLLM, with ``architectures=["LlamaForCausalLMEagle3"]``; its EAGLE-1/2 worker reads the
published EAGLE layout with ``architectures=["LlamaForCausalLMEagle"]``. The tensors are those of the vLLM exporters.
"""

from __future__ import annotations

from typing import Any

from ..errors import ConfigError
from .exporters import register_exporter
from .vllm import EagleVllmExporter, Eagle3VllmExporter

__all__ = ["EagleSglangExporter", "Eagle3SglangExporter"]


@register_exporter("sglang", "eagle3")
class Eagle3SglangExporter(Eagle3VllmExporter):
    def config(self, technique, **options: Any) -> dict[str, Any]:
        if options:
            raise ConfigError(f"sglang/eagle3 takes no options, got {sorted(options)}")
        cfg = super().config(technique)
        cfg["architectures"] = ["LlamaForCausalLMEagle3"]
        return cfg


@register_exporter("sglang", "eagle")
class EagleSglangExporter(EagleVllmExporter):
    def config(self, technique, **options: Any) -> dict[str, Any]:
        cfg = super().config(technique, **options)
        cfg["architectures"] = ["LlamaForCausalLMEagle"]
        return cfg
