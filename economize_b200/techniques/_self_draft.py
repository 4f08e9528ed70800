"""Self-drafting from a sub-network of the target (shared package of ``layer_skip``, ``early_exit``, ``kangaroo`` and
``knapspec``).

A :func:`layer_view` is a :class:`~economize_b200.models.llama.CausalLM` that shares the target's embedding, final
norm, LM head and a chosen list of its decoder layers (optionally skipping the attention or MLP sublayer of some,
or followed by extra technique-owned layers). The view owns nothing but its own KV cache, so drafting with it runs
on the same kernels as the target; the engine drives it like a separate draft model
(:class:`~economize_b200.techniques.draft_model.DraftLMDrafter`). Economize implements these drafters as layer
policies of its runner (``runtime/policy.py:23-79``, ``techniques/layer_skip``, ``techniques/early_exit``).
"""

from __future__ import annotations

import dataclasses
from collections.abc import Sequence

import torch
from torch import nn

from ..core.technique import Capability, Family, Technique
from ..decoding.config import DecodeConfig
from ..errors import ConfigError
from ..models.llama import CausalLM, DecoderLayer
from ..runtime.cache import StepBatch

__all__ = ["LayerRef", "SelfDraftTechnique", "block_influence", "layer_view"]


class LayerRef(nn.Module):
    """A decoder layer seen through a view: the same parameters, optionally without its attention or MLP."""

    def __init__(self, layer: DecoderLayer, skip_attn: bool = False, skip_mlp: bool = False) -> None:
        super().__init__()
        self._target = [layer]  # not a submodule: the target owns it
        self.skip_attn, self.skip_mlp = skip_attn, skip_mlp

    def __getattr__(self, name: str):
        try:
            return super().__getattr__(name)
        except AttributeError:
            return getattr(self.__dict__["_target"][0], name)

    def register_parameter(self, name: str, param: nn.Parameter | None) -> None:
        """A parameter of the view's own that shadows the target's (a draft path's rewritten weight); the base
        class would refuse it because the name resolves to the target's attribute."""
        if param is not None and not isinstance(param, nn.Parameter):
            raise TypeError(f"cannot assign {type(param).__name__} as parameter {name!r}")
        self._parameters[name] = param


def layer_view(target: CausalLM, layers: Sequence[int | tuple[int, bool, bool]],
               extra: Sequence[nn.Module] = ()) -> CausalLM:
    """A :class:`CausalLM` over the target's layers ``layers`` (indices, or ``(index, skip_attn, skip_mlp)``)
    followed by ``extra`` layers, sharing the embedding, final norm and LM head."""
    view = CausalLM.__new__(CausalLM)
    nn.Module.__init__(view)
    refs = []
    for spec in layers:
        i, sa, sm = (spec, False, False) if isinstance(spec, int) else spec
        if not 0 <= i < target.config.num_layers:
            raise ConfigError(f"layer {i} is outside the target's {target.config.num_layers} layers")
        refs.append(LayerRef(target.layers[i], sa, sm))
    order = [spec if isinstance(spec, int) else spec[0] for spec in layers]
    # per-layer attributes keyed by the target's layer index follow the layers into the view's numbering
    view.config = dataclasses.replace(target.config, num_layers=len(refs) + len(extra),
                                      nope_layers=tuple(j for j, i in enumerate(order)
                                                        if i in target.config.nope_layers))
    view.embed = target.embed
    view.layers = nn.ModuleList(refs + list(extra))
    view.norm = target.norm
    view.lm_head = target.lm_head
    view._rope = None
    view.observer = None
    view.kv_dtype = target.kv_dtype
    view.kv_scales = None
    view.kv_evictor = None
    view.kv_quantizer = None
    view.depth_policy = None
    view.prefill_sparsity = None
    view.exact_tail = target.exact_tail
    if target.kv_scales is not None:
        idx = [spec if isinstance(spec, int) else spec[0] for spec in layers]
        ks, vs = target.kv_scales
        ones = torch.ones(len(extra), ks.shape[1], dtype=ks.dtype, device=ks.device)
        view.kv_scales = (torch.cat([ks[idx], ones]), torch.cat([vs[idx], ones]))
    view.tp = target.tp
    view.local = dict(target.local)
    return view


@torch.no_grad()
def block_influence(model: CausalLM, batches: Sequence[torch.Tensor]) -> torch.Tensor:
    """ShortGPT's Block Influence of every layer: ``1 - cos(h_in, h_out)`` of its residual-stream input and output,
    averaged over the calibration tokens (Men et al., 2024). Low values mark layers that change little."""
    n = model.config.num_layers
    total = torch.zeros(n, dtype=torch.float64)
    count = 0
    for tokens in batches:
        tokens = torch.as_tensor(tokens).to(model.device)
        if tokens.dim() == 1:
            tokens = tokens[None]
        b, length = tokens.shape
        cache = model.new_cache(b, ((length + 127) // 128) * 128)
        lengths = torch.full((b,), length, dtype=torch.int32, device=model.device)
        _, aux = model.forward_step(tokens, StepBatch.prefill(lengths, length), cache, capture=tuple(range(n + 1)))
        for i in range(n):
            a, o = aux[i].float().reshape(-1, aux[i].shape[-1]), aux[i + 1].float().reshape(-1, aux[i].shape[-1])
            cos = torch.nn.functional.cosine_similarity(a, o, dim=-1)
            total[i] += float((1 - cos).sum())
        count += b * length
    return (total / max(count, 1)).float()


class SelfDraftTechnique(Technique):
    """Base of the sub-network drafters: subclasses choose the layers in :meth:`view_layers`."""

    capabilities = Capability.DRAFTER
    family = Family.DRAFTER
    lossless = True

    def __init__(self, config, model: CausalLM) -> None:
        super().__init__(config, model)
        self._calibration = None
        self._view: list[CausalLM] = []

    def calibrate(self, calibration) -> None:
        self._calibration = calibration

    def calibration_batches(self) -> list[torch.Tensor]:
        cal = self._calibration
        if cal is None:
            raise ConfigError(f"{self.name} needs calibration tokens for its layer search "
                              "(apply(..., calibration=ids)) or an explicit layer list")
        return [cal] if isinstance(cal, torch.Tensor) else list(cal)

    def view_layers(self) -> list[int | tuple[int, bool, bool]]:
        raise NotImplementedError

    def extra_layers(self) -> list[nn.Module]:
        return []

    def attach(self) -> None:
        self._view = [layer_view(self.model, self.view_layers(), self.extra_layers())]

    @property
    def view(self) -> CausalLM:
        if not self._view:
            self.attach()
        return self._view[0]

    def drafter(self):
        from .draft_model import DraftLMDrafter

        return DraftLMDrafter(self.view, self.model.config.hidden_size)

    def default_decoding(self) -> DecodeConfig:
        return DecodeConfig(cycle_length=4)
