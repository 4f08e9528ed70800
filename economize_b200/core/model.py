"""``EfficientModel`` and ``apply``: the user-facing wrapper of a model with techniques attached.

Same surface as economize (``src/economize/core/model.py:73-386``): ``apply(model, *configs, decoding=)``
attaches techniques in capability order and returns an :class:`EfficientModel` with ``generate``, ``decode``,
``decode_batch``, ``decoder``, ``save_pretrained`` and attribute fall-through to the wrapped model. The difference is
what executes: the wrapper converts a Hugging Face causal LM into the engine's own :class:`CausalLM` (fused weights,
sm_100a kernels) and decodes with :class:`~economize_b200.decoding.engine.SpecEngine`; the Hugging Face module is
kept as ``base_model`` for its config and as an oracle.
"""

from __future__ import annotations

from collections.abc import Sequence
from typing import Any

import torch
from torch import nn

from ..decoding.config import DecodeConfig
from ..decoding.engine import DecodeResult, SpecEngine
from ..errors import ConfigError, EconomizeError, UnsupportedModelError
from ..models.llama import CausalLM
from .technique import CAPABILITY_ORDER, Capability, Simulation, Technique, TechniqueConfig, check_compatible, \
    technique_for

__all__ = ["EfficientModel", "apply", "as_engine_model", "build_model"]

LOSSLESS_COMPATIBLE = Capability.WEIGHTS | Capability.ACTIVATIONS | Capability.DRAFTER


def as_engine_model(model: nn.Module) -> CausalLM:
    """The engine model of ``model``: itself for a :class:`CausalLM`, a converted copy of a HF causal LM."""
    if isinstance(model, CausalLM):
        return model
    if isinstance(model, EfficientModel):
        return model.model
    if hasattr(model, "config") and hasattr(model, "state_dict"):
        return CausalLM.from_hf(model)
    raise UnsupportedModelError(f"cannot execute a {type(model).__name__}: pass a transformers causal LM of a "
                                "supported family or an economize_b200.models.CausalLM")


def _rank(technique: Technique) -> int:
    for i, cap in enumerate(CAPABILITY_ORDER):
        if cap != Capability.NONE and cap in technique.capabilities:
            return i
    return len(CAPABILITY_ORDER)


class EfficientModel(nn.Module):
    """A model with efficiency techniques attached.

    Args:
        model: The engine model the techniques act on.
        techniques: Attached techniques in attach order.
        decoding: Default decoding options.
        base_model: The module the user passed (a HF model), kept for attribute fall-through.
    """

    def __init__(self, model: CausalLM, techniques: Sequence[Technique], decoding: DecodeConfig,
                 base_model: nn.Module | None = None) -> None:
        super().__init__()
        self.model = model
        self.techniques = nn.ModuleDict({t.name: t for t in techniques})
        self._base = [base_model if base_model is not None else model]
        self._decoders: dict[tuple[DecodeConfig, str | None], SpecEngine] = {}
        self.decoding = decoding
        self.source_digests: dict[str, str] | None = None
        #: fingerprint of the base weights taken before weight-rewriting techniques attached (else None)
        self.teacher_digest: str | None = None

    def __getattr__(self, name: str) -> Any:
        try:
            return super().__getattr__(name)
        except AttributeError:
            if name in ("model", "techniques", "_base", "_modules", "_parameters", "_buffers"):
                raise
            return getattr(self._base[0], name)

    @property
    def base_model(self) -> nn.Module:
        return self._base[0]

    def unwrap(self) -> nn.Module:
        return self.base_model

    @property
    def device(self) -> torch.device:
        return self.model.device

    def forward(self, input_ids: torch.Tensor, **kwargs: Any) -> torch.Tensor:
        """Logits ``[B, S, V]`` of a full causal pass of the engine model (no cache reuse)."""
        from ..runtime.cache import StepBatch

        ids = input_ids if input_ids.dim() == 2 else input_ids[None]
        batch, length = ids.shape
        cache = self.model.new_cache(batch, ((length + 127) // 128) * 128)
        lengths = torch.full((batch,), length, dtype=torch.int32, device=ids.device)
        hidden, _ = self.model.forward_step(ids, StepBatch.prefill(lengths, length), cache)
        return self.model.logits(hidden)

    # ---- techniques --------------------------------------------------------------------------------------------
    @property
    def drafting_technique(self) -> Technique | None:
        return next((t for t in self.techniques.values() if Capability.DRAFTER in t.capabilities), None)

    def technique_parameters(self):
        return self.techniques.parameters()

    def simulations(self) -> dict[str, Simulation]:
        return {n: s for n, t in self.techniques.items() if (s := t.simulation()) is not None}

    def lossy_techniques(self, compatible: Capability = Capability.NONE) -> list[str]:
        return [t.name for t in self.techniques.values()
                if not t.lossless and not (t.capabilities and t.capabilities in compatible)]

    def refresh(self) -> None:
        """Drop decoders and graphs (after the weights or devices changed)."""
        self._decoders.clear()

    def detach(self) -> nn.Module:
        rewrites = [t.name for t in self.techniques.values() if Capability.WEIGHTS in t.capabilities]
        if rewrites:
            raise EconomizeError(f"{rewrites} rewrote the weights in place and cannot be detached; reload the model")
        for t in reversed(list(self.techniques.values())):
            t.detach()
        self._decoders.clear()
        return self.base_model

    # ---- decoding ----------------------------------------------------------------------------------------------
    @property
    def decoding(self) -> DecodeConfig:
        return self._decoding

    @decoding.setter
    def decoding(self, config: DecodeConfig) -> None:
        if not isinstance(config, DecodeConfig):
            raise ConfigError(f"decoding must be a DecodeConfig, got {type(config).__name__}")
        self._decoding = config

    def decoder(self, decoding: DecodeConfig | None = None, selector: Any = None) -> SpecEngine:
        """The engine for ``decoding`` (cached per configuration and selector with its CUDA graphs)."""
        config = decoding or self.decoding
        sampling = selector is not None and not getattr(selector, "greedy", True)
        key = (config, repr(selector) if sampling else None)
        engine = self._decoders.get(key)
        if engine is None:
            if config.lossless is True:
                lossy = self.lossy_techniques(LOSSLESS_COMPATIBLE)
                if lossy:
                    raise ConfigError(f"lossless=True contradicts the lossy technique(s) {lossy}")
            technique = self.drafting_technique
            drafter = technique.drafter() if technique is not None and config.cycle_length > 1 else None
            vocab = getattr(technique, "draft_vocab", None)
            engine = SpecEngine(self.model, drafter, config, draft_vocab=vocab, selector=selector if sampling else None)
            self._decoders[key] = engine
        return engine

    @torch.no_grad()
    def decode(self, input_ids: torch.Tensor, max_new_tokens: int, *, decoding: DecodeConfig | None = None,
               stop: int | Sequence[int] | None = None, selector: Any = None) -> DecodeResult:
        if input_ids.dim() == 2 and input_ids.shape[0] == 1:
            input_ids = input_ids[0]
        if input_ids.dim() != 1:
            raise ConfigError(f"decode takes one prompt [P] or [1, P], got {tuple(input_ids.shape)}")
        return self.decode_batch([input_ids], max_new_tokens, decoding=decoding, stop=stop, selector=selector)[0]

    @torch.no_grad()
    def decode_batch(self, prompts: Sequence[torch.Tensor] | torch.Tensor, max_new_tokens: int | Sequence[int], *,
                     decoding: DecodeConfig | None = None, stop: int | Sequence[int] | None = None,
                     selector: Any = None) -> list[DecodeResult]:
        config = decoding or self.decoding
        stops = [stop] if isinstance(stop, int) else (list(stop) if stop is not None else None)
        return self.decoder(config, selector).generate(prompts, max_new_tokens, stops)

    def generate(self, inputs: torch.Tensor | None = None, *, max_new_tokens: int = 20,
                 decoding: DecodeConfig | None = None, input_ids: torch.Tensor | None = None,
                 attention_mask: torch.Tensor | None = None, do_sample: bool = False, temperature: float = 1.0,
                 top_p: float = 1.0, top_k: int = 0, eos_token_id: int | Sequence[int] | None = None,
                 pad_token_id: int | None = None, **unused: Any) -> torch.Tensor:
        """``transformers``-style generate: returns ``[B, P + N]`` (prompt followed by new tokens, right-padded with
        ``pad_token_id``). ``attention_mask`` marks left padding of ragged prompts, which is stripped."""
        from ..decoding.selectors import TopPSampler

        ids = inputs if inputs is not None else input_ids
        if ids is None:
            raise ConfigError("generate needs input_ids")
        if ids.dim() == 1:
            ids = ids[None]
        prompts = []
        for b in range(ids.shape[0]):
            row = ids[b]
            if attention_mask is not None:
                row = row[attention_mask[b].bool()]
            prompts.append(row)
        selector = TopPSampler(temperature=temperature, top_p=top_p, top_k=top_k) if do_sample else None
        results = self.decode_batch(prompts, max_new_tokens, decoding=decoding, stop=eos_token_id,
                                    selector=selector)
        pad = pad_token_id if pad_token_id is not None else 0
        rows = [torch.cat([p.to(r.tokens.device), r.tokens]) for p, r in zip(prompts, results)]
        width = max(r.numel() for r in rows)
        out = torch.full((len(rows), width), pad, dtype=torch.long)
        for b, r in enumerate(rows):
            out[b, : r.numel()] = r.cpu()
        return out.to(ids.device)

    # ---- persistence -------------------------------------------------------------------------------------------
    def save_pretrained(self, path: str, **kwargs: Any) -> None:
        from .serialization import save

        save(self, path, **kwargs)


def build_model(model: nn.Module, configs: Sequence[TechniqueConfig], *, decoding: DecodeConfig | None = None,
                calibration: Any = None, states: dict[str, dict[str, torch.Tensor]] | None = None) -> EfficientModel:
    engine_model = as_engine_model(model)
    digest = None
    if any(Capability.WEIGHTS in technique_for(c).capabilities for c in configs):
        from .serialization import teacher_fingerprint

        digest = teacher_fingerprint(engine_model)

    def build(config):
        t = technique_for(config)(config, engine_model)
        if states and t.name in states:
            t.load_technique_state(states[t.name])
        if hasattr(t, "calibrate") and calibration is not None:
            t.calibrate(calibration)
        return t

    # weight transforms (which may change the depth or the projections) are built and attached first, so the other
    # techniques are built against the transformed model. A failure anywhere rolls the whole call back.
    from .transaction import AttachTransaction

    order = sorted(configs, key=lambda c: _rank(technique_for(c)))
    techniques: list[Technique] = []
    tx = AttachTransaction(engine_model)
    current = None
    try:
        for config in order:
            if Capability.WEIGHTS in technique_for(config).capabilities:
                current = None
                t = build(config)
                current = t
                techniques.append(t)
                check_compatible(techniques)
                tx.before_weights(t)
                t.attach()
                tx.attached_ok(t)
        current = None
        rest = [build(c) for c in order if Capability.WEIGHTS not in technique_for(c).capabilities]
        check_compatible(techniques + rest)
        for t in rest:
            current = t
            t.attach()
            tx.attached_ok(t)
        current = None
        techniques += rest
        for t in techniques:  # drafter transforms (draft_quant, frspec) act once the drafter is attached
            if hasattr(t, "after_drafter"):
                drafter = next((d for d in techniques if Capability.DRAFTER in d.capabilities), None)
                if drafter is None:
                    raise ConfigError(f"{t.name} transforms a drafter, but no drafting technique is applied")
                current = t
                t.after_drafter(drafter)
    except BaseException as error:
        if current is not None and Capability.WEIGHTS not in current.capabilities:
            try:  # a technique that raised part way through its own attach is detached too
                current.detach()
            except Exception:  # noqa: BLE001 - the original error is the one to report
                pass
        tx.roll_back(current, error)
        raise
    if decoding is None:
        decoding = next((d for t in techniques if (d := t.default_decoding()) is not None), None)
    if decoding is None:
        decoding = DecodeConfig(cycle_length=4 if any(Capability.DRAFTER in t.capabilities for t in techniques)
                                else 1)
    result = EfficientModel(engine_model, techniques, decoding, base_model=model)
    result.teacher_digest = digest
    return result


def apply(model: nn.Module, *configs: TechniqueConfig, decoding: DecodeConfig | None = None,
          calibration: Any = None) -> EfficientModel:
    """Attach the techniques of ``configs`` to ``model`` (a ``transformers`` causal LM or a
    :class:`~economize_b200.models.CausalLM`), in capability order.

    Raises:
        IncompatibleTechniquesError: a technique twice, two drafters, or two techniques that exclude each other.
        ConfigError: a configuration does not fit the model.
    """
    return build_model(model, configs, decoding=decoding, calibration=calibration)
