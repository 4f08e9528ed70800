"""Pipeline placement: a model's decoder layers split over devices in contiguous stages (economize places layers
with Hugging Face's ``device_map`` and its runner moves the hidden states to each layer's device,
``src/economize/runtime/runner.py:164-166``).

:func:`pipeline_split` moves each stage's layers to its device; the embedding, the final norm and the LM head stay
on the first device (the home device, where the engine keeps its state). A pass moves the residual stream to a
stage when it reaches that stage's first layer and back home after the last one; each stage keeps its own KV cache
(``SplitKVCache``). Decoding then runs without CUDA graphs (a graph belongs to one device), as in economize. Use it
for a model that does not fit one device's memory; tensor parallelism (:mod:`.tp`) is the faster split.
"""

from __future__ import annotations

from collections.abc import Sequence

import torch

from ..errors import ConfigError

__all__ = ["pipeline_split", "stage_sizes"]


def stage_sizes(num_layers: int, stages: int) -> list[int]:
    """Layers per stage, as equal as possible (earlier stages take the remainder)."""
    if stages < 1 or stages > num_layers:
        raise ConfigError(f"cannot split {num_layers} layers into {stages} stages")
    base, extra = divmod(num_layers, stages)
    return [base + (1 if s < extra else 0) for s in range(stages)]


@torch.no_grad()
def pipeline_split(model, devices: Sequence[torch.device | str], balance: Sequence[int] | None = None):
    """Place ``model``'s layers (an engine :class:`~economize_b200.models.CausalLM` or an EfficientModel) on
    ``devices`` in order; ``balance`` gives the layers per stage (default: equal). Returns the model."""
    from ..core.model import EfficientModel

    target = model.model if isinstance(model, EfficientModel) else model
    c = target.config
    devices = [torch.device(d) for d in devices]
    sizes = list(balance) if balance is not None else stage_sizes(c.num_layers, len(devices))
    if len(sizes) != len(devices) or sum(sizes) != c.num_layers or min(sizes) < 1:
        raise ConfigError(f"balance {sizes} does not place {c.num_layers} layers on {len(devices)} devices")
    if target.tp is not None and target.tp.size > 1:
        raise ConfigError("pipeline placement of a tensor-parallel model is not supported")
    if target.kv_quantizer is not None or target.kv_evictor is not None or target.prefill_sparsity is not None:
        raise ConfigError("pipeline placement keeps plain per-stage caches (no KIVI, eviction or sparse views)")
    placement = []
    for dev, n in zip(devices, sizes):
        placement += [dev] * n
    for layer, dev in zip(target.layers, placement):
        layer.to(dev)
    target.placement = placement if len(set(placement)) > 1 or placement[0] != target.device else None
    if isinstance(model, EfficientModel):
        model.refresh()
    return model
