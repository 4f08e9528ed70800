"""A separate draft language model (``draft_model``; economize ``techniques/draft_model``), e.g. Llama-3.2-1B
drafting for Llama-3.1-8B. The draft model runs on the engine's kernels with its own slot KV cache: after every
exact pass it processes the committed columns and the root token, then runs chain steps or EAGLE-2 tree steps."""

from __future__ import annotations

from dataclasses import dataclass, fields
from typing import Any, ClassVar

import torch
from torch import nn

from ...core.technique import Capability, Family, Technique, TechniqueConfig, register_technique
from ...decoding.config import DecodeConfig
from ...errors import ConfigError
from ...models.llama import CausalLM
from ...runtime.cache import KVCache, StepBatch

__all__ = ["DraftLMDrafter", "DraftModelConfig", "DraftModelTechnique", "install_view", "load_draft"]


@dataclass(frozen=True)
class DraftModelConfig(TechniqueConfig):
    """Attributes: ``model`` (a Hugging Face id or path, a ``transformers`` causal LM or an engine
    :class:`CausalLM`), ``revision``, ``dtype`` (``None``: the target's), ``attn_implementation`` (accepted for
    compatibility; the engine's kernels run the model), ``window`` / ``sink`` (``window > 0``: the draft model
    attends to a StreamingLLM view of its own cache, the first ``sink`` prompt tokens plus the ``window`` most
    recent ones, as TriForce's and MagicDec's long-context drafters do; the attention kernel skips the hidden
    128-key chunks)."""

    technique: ClassVar[str] = "draft_model"
    model: Any = None
    revision: str | None = None
    dtype: str | None = None
    attn_implementation: str | None = None
    window: int = 0
    sink: int = 0

    def __post_init__(self) -> None:
        if self.model is None:
            raise ConfigError("draft_model needs model= (an id, a path or a model)")
        if self.window < 0 or self.sink < 0:
            raise ConfigError("draft_model window and sink must be >= 0")

    def to_dict(self) -> dict[str, Any]:
        out = {f.name: getattr(self, f.name) for f in fields(self)}
        if not isinstance(out["model"], str):
            out["model"] = getattr(getattr(self.model, "config", None), "_name_or_path", None) or "<in-memory model>"
        return out


def install_view(draft: CausalLM, config: DraftModelConfig) -> None:
    """With ``config.window > 0`` the draft model attends to a StreamingLLM view of its own cache."""
    if config.window > 0:
        from ..sparse_kv_draft import MagicDecConfig, SparseViewEvictor

        draft.kv_evictor = SparseViewEvictor(MagicDecConfig(sink=config.sink, window=config.window),
                                             draft.config.num_layers)


def load_draft(config: DraftModelConfig, target: CausalLM) -> CausalLM:
    dtype = {None: target.dtype, "float32": torch.float32, "bfloat16": torch.bfloat16,
             "float16": torch.float16}[config.dtype]
    model = config.model
    if isinstance(model, str):
        import transformers

        model = transformers.AutoModelForCausalLM.from_pretrained(model, revision=config.revision, dtype=dtype)
    if isinstance(model, CausalLM):
        draft = model
    elif isinstance(model, nn.Module):
        draft = CausalLM.from_hf(model, dtype=dtype, device=target.device)
    else:
        raise ConfigError(f"draft_model cannot use a {type(model).__name__}")
    if draft.config.vocab_size != target.config.vocab_size:
        raise ConfigError(f"the draft model's vocabulary ({draft.config.vocab_size}) differs from the target's "
                          f"({target.config.vocab_size})")
    return draft


@register_technique
class DraftModelTechnique(Technique):
    config_class = DraftModelConfig
    capabilities = Capability.DRAFTER
    family = Family.DRAFTER

    def __init__(self, config: DraftModelConfig, model: CausalLM) -> None:
        super().__init__(config, model)
        self._draft = [load_draft(config, model)]  # not a submodule: its weights are not the technique's
        install_view(self.draft, config)

    @property
    def draft(self) -> CausalLM:
        return self._draft[0]

    def export_state(self) -> dict[str, torch.Tensor]:
        return {}

    def load_technique_state(self, state: dict[str, torch.Tensor]) -> None:
        if state:
            raise ConfigError("draft_model stores no tensors in checkpoints (its config names the model)")

    def drafter(self) -> DraftLMDrafter:
        return DraftLMDrafter(self.draft, self.model.config.hidden_size)

    def default_decoding(self) -> DecodeConfig:
        return DecodeConfig(cycle_length=5)


class DraftLMDrafter:
    """The engine-side drafter of a draft LM (a :class:`~economize_b200.decoding.drafter.DraftModel`)."""

    capture_layers: tuple[int, ...] = (-1,)  # only for the shapes: the draft model reads tokens, not states
    carry_size = 0

    def __init__(self, draft: CausalLM, target_hidden: int) -> None:
        self.draft = draft
        self.target_hidden = target_hidden
        self.cache: KVCache | None = None

    def begin(self, batch: int, capacity: int) -> None:
        if self.cache is None or self.cache.batch != batch or self.cache.capacity < capacity:
            self.cache = self.draft.new_cache(batch, capacity)
        else:
            self.cache.reset()
        self._prompt_pass = True  # the first observe covers the prompt (KV policies of the draft score it)

    def fuse(self, aux: dict[int, torch.Tensor]) -> torch.Tensor:
        states = aux[-1]
        return torch.zeros(*states.shape[:2], 1, dtype=self.draft.dtype, device=states.device)

    def observe(self, tokens: torch.Tensor, sources: torch.Tensor, kv_len: torch.Tensor, n_valid: torch.Tensor,
                root: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        batch, width = tokens.shape
        dev = tokens.device
        pos = (kv_len[:, None] + torch.arange(width, device=dev, dtype=torch.int32)[None]).to(torch.int32)
        first, self._prompt_pass = getattr(self, "_prompt_pass", False), False
        hidden, _ = self.draft.forward_step(tokens, StepBatch(kv_len, n_valid.to(torch.int32), pos.contiguous(),
                                                              is_prefill=first), self.cache)
        rows = torch.arange(batch, device=dev)
        logits = self.draft.logits(hidden[rows, root.long()]).float()
        return logits, torch.zeros(batch, self.target_hidden, dtype=self.draft.dtype, device=dev)

    def tree_step(self, tokens: torch.Tensor, states: torch.Tensor, positions: torch.Tensor, kv_base: torch.Tensor,
                  n_forwarded: int, q_offset: int, mask: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        batch = tokens.shape[0]
        n_new = torch.full((batch,), n_forwarded, dtype=torch.int32, device=tokens.device)
        hidden, _ = self.draft.forward_step(tokens, StepBatch(kv_base.to(torch.int32), n_new,
                                                              positions.to(torch.int32), mask, q_offset), self.cache)
        return self.draft.logits(hidden).float(), states

    def to_target(self, ids: torch.Tensor) -> torch.Tensor:
        return ids
