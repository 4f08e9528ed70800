"""EAGLE-3 drafting on the engine: the technique (parameters, checkpoint layout) and its device drafter.

Parameter names follow the official checkpoints after fusing projections: ``fc [H, 3H]``, the draft layer
(``midlayer.*`` of SafeAILab / SpecForge with q/k/v and gate/up fused), ``norm``, ``lm_head [V_d, H]``, ``d2t``
and ``t2d``. :mod:`.formats` converts official and vLLM ``speculators`` checkpoints.
"""

from __future__ import annotations

import torch
from torch import nn

from ... import ops
from ...core.technique import Capability, Family, Technique, register_technique
from ...decoding.config import DecodeConfig
from ...models.config import ModelConfig
from ...runtime.cache import KVCache, StepBatch
from .._draft_layer.layer import DraftLayer
from .config import Eagle3Config

__all__ = ["Eagle3Drafter", "Eagle3Technique"]


def _dtype(config: Eagle3Config, model) -> torch.dtype:
    return {"model": model.dtype, "float32": torch.float32, "bfloat16": torch.bfloat16,
            "float16": torch.float16}[config.param_dtype]


@register_technique
class Eagle3Technique(Technique):
    config_class = Eagle3Config
    capabilities = Capability.DRAFTER
    family = Family.DRAFTER
    lossless = True

    def __init__(self, config: Eagle3Config, model) -> None:
        super().__init__(config, model)
        c = model.config
        dtype, dev = _dtype(config, model), model.device
        kw = dict(dtype=dtype, device=dev)
        h = c.hidden_size
        self.aux_layers = config.layers(c.num_layers)
        heads = config.num_heads or c.num_heads
        kv_heads = config.num_kv_heads or (c.num_kv_heads if config.num_heads is None else heads)
        head_dim = config.head_dim or c.head_dim
        self.eps = config.rms_norm_eps or c.rms_norm_eps
        self.fc = nn.Parameter(torch.empty(h, len(self.aux_layers) * h, **kw))
        self.input_norm = nn.Parameter(torch.ones(h, **kw))
        self.hidden_norm = nn.Parameter(torch.ones(h, **kw))
        bias = bool(config.attention_bias) if config.attention_bias is not None else c.attention_bias
        self.layer = DraftLayer(2 * h, h, config.intermediate_size or c.intermediate_size, heads, kv_heads,
                                head_dim, self.eps, bias, dtype, dev)
        rope = ModelConfig.from_dict({**c.to_dict(), "rope_theta": config.rope_theta or c.rope_theta,
                                      "rope_scaling": config.rope_scaling if config.rope_theta else c.rope_scaling})
        self.layer.set_rope(rope)
        self.draft_vocab = config.draft_vocab or c.vocab_size
        self.shared_head = config.head == "shared"
        if not self.shared_head:
            self.norm = nn.Parameter(model.norm.detach().clone().to(dtype))
            self.lm_head = nn.Parameter(model.head_weight.detach()[: self.draft_vocab].clone().to(dtype))
        self.register_buffer("d2t", torch.zeros(self.draft_vocab, dtype=torch.int64, device=dev))
        self.register_buffer("t2d", torch.zeros(c.vocab_size, dtype=torch.bool, device=dev))
        self.t2d[: self.draft_vocab] = True
        self.reset_parameters()

    @torch.no_grad()
    def reset_parameters(self, seed: int | None = None, std: float = 0.02, identity: bool = False) -> None:
        """Random N(0, std) matrices. With ``identity``, start as an early exit of the target instead: ``fc``
        selects the highest fused feature, and the attention and MLP output maps are zero, so the draft layer
        passes that feature through and the (target-initialised) head drafts what the target's head would say on
        it; training then learns the corrections."""
        gen = None
        if seed is not None:
            gen = torch.Generator(device=self.fc.device)
            gen.manual_seed(seed)
        for p in (self.fc, self.layer.wqkv, self.layer.wo, self.layer.w_gate_up, self.layer.w_down):
            p.copy_(torch.randn(p.shape, generator=gen, device=p.device, dtype=torch.float32) * std)
        if identity:
            h = self.fc.shape[0]
            self.fc.zero_()
            self.fc[:, -h:].copy_(torch.eye(h, device=self.fc.device, dtype=self.fc.dtype))
            self.layer.wo.zero_()
            self.layer.w_down.zero_()

    @torch.no_grad()
    def draft_vocab_from(self, tokens: torch.Tensor) -> torch.Tensor:
        """Choose the draft vocabulary as the ``draft_vocab`` most frequent ids of ``tokens`` (EAGLE-3's rule;
        ties and unseen ids fill up in id order) and return the chosen ids."""
        vocab = self.t2d.numel()
        counts = torch.bincount(tokens.reshape(-1).long().to(self.d2t.device), minlength=vocab)[:vocab].float()
        order = torch.argsort(-counts - torch.arange(vocab, device=counts.device) * 1e-9 / vocab)
        ids = order[: self.draft_vocab]
        self.set_draft_vocab(ids)
        return ids

    @torch.no_grad()
    def extend_draft_vocab(self, tokens: torch.Tensor, keep: torch.Tensor) -> int:
        """Make every id of ``tokens`` draftable without disturbing the ids of ``keep`` (the ones the head was
        trained on): missing ids replace draft slots whose id is not in ``keep``; their head rows start from the
        target's. Returns the number of ids added."""
        have = self.t2d.clone()
        missing = torch.unique(tokens.reshape(-1).long().to(have.device))
        missing = missing[~have[missing]]
        if missing.numel() == 0:
            return 0
        ids = torch.arange(self.draft_vocab, device=have.device) + self.d2t
        kept = torch.zeros_like(have)
        kept[torch.unique(keep.reshape(-1).long().to(have.device))] = True
        free = (~kept[ids]).nonzero().flatten()[: missing.numel()]
        missing = missing[: free.numel()]
        new_ids = ids.clone()
        new_ids[free] = missing
        order = torch.argsort(new_ids)
        rows = self.lm_head.detach()[order].clone()
        fresh = torch.isin(new_ids[order], missing)
        rows[fresh] = self.model.head_weight.detach()[new_ids[order][fresh]].to(rows.dtype)
        sorted_ids = new_ids[order]
        self.d2t.copy_(sorted_ids - torch.arange(sorted_ids.numel(), device=sorted_ids.device))
        self.t2d.zero_()
        self.t2d[sorted_ids] = True
        self.lm_head.copy_(rows)
        return int(missing.numel())

    @torch.no_grad()
    def set_draft_vocab(self, token_ids: torch.Tensor) -> None:
        """Restrict the own head to ``token_ids`` (``draft_vocab`` most frequent target tokens, any order)."""
        ids = token_ids.to(self.d2t.device).long().sort().values[: self.draft_vocab]
        self.d2t.copy_(ids - torch.arange(ids.numel(), device=ids.device))
        self.t2d.zero_()
        self.t2d[ids] = True
        self.lm_head.copy_(self.model.head_weight.detach()[ids].to(self.lm_head.dtype))

    def head_weights(self) -> tuple[torch.Tensor, torch.Tensor]:
        if self.shared_head:
            return self.model.norm, self.model.head_weight
        return self.norm, self.lm_head

    def default_decoding(self) -> DecodeConfig:
        return DecodeConfig(cycle_length=4)

    def export_state(self) -> dict[str, torch.Tensor]:
        from .formats import to_reference_state

        return to_reference_state(self)

    def load_technique_state(self, state: dict[str, torch.Tensor]) -> None:
        from .formats import from_reference_state

        from_reference_state(self, state)

    def drafter(self) -> Eagle3Drafter:
        return Eagle3Drafter(self)


class Eagle3Drafter:
    """The device-side EAGLE-3 drafter (the engine's :class:`~economize_b200.decoding.drafter.DraftModel`).

    Its draft cache holds the draft layer's keys/values ``[B, H_kv, slots, D]`` laid out like the target's (slot
    ``p`` = position ``p``). :meth:`observe` rewrites the entries of the committed columns from the exact pass's
    fused states and runs the root step; :meth:`tree_step` runs a frontier of a draft tree.
    """

    def __init__(self, technique: Eagle3Technique) -> None:
        self.t = technique
        self.capture_layers = tuple(technique.aux_layers)
        self.carry_size = technique.model.config.hidden_size
        self.cache: KVCache | None = None

    @property
    def d2t_map(self) -> torch.Tensor:
        """Draft id -> target id offsets (read by the engine's fused top-k)."""
        return self.t.d2t

    def begin(self, batch: int, capacity: int) -> None:
        layer = self.t.layer
        if self.cache is None or self.cache.batch != batch or self.cache.capacity < capacity:
            self.cache = KVCache(1, batch, layer.kv_heads, capacity, layer.head_dim, layer.wqkv.dtype,
                                 layer.wqkv.device)
        else:
            self.cache.reset()

    def fuse(self, aux: dict[int, torch.Tensor]) -> torch.Tensor:
        x = torch.cat([aux[i] for i in self.capture_layers], -1)
        return ops.linear(x.to(self.t.fc.dtype), self.t.fc)

    def _step(self, tokens: torch.Tensor, sources: torch.Tensor, batch: StepBatch) -> torch.Tensor:
        t = self.t
        emb = t.model.embed_tokens(tokens).to(t.fc.dtype)
        x_e, _ = ops.rmsnorm(emb, t.input_norm, t.eps)
        x_h, _ = ops.rmsnorm(sources, t.hidden_norm, t.eps)
        residual = x_h if t.config.norm_before_residual else sources
        mlp, a = t.layer.run(torch.cat([x_e, x_h], -1), residual, self.cache, batch)
        return mlp, a

    def _head(self, mlp: torch.Tensor, a: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        norm, head = self.t.head_weights()
        normed, out = ops.rmsnorm(mlp, norm, self.t.eps, a)
        return ops.linear(normed, head).float(), out

    def observe(self, tokens: torch.Tensor, sources: torch.Tensor, kv_len: torch.Tensor, n_valid: torch.Tensor,
                root: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        batch, width = tokens.shape
        dev = tokens.device
        pos = (kv_len[:, None] + torch.arange(width, device=dev, dtype=torch.int32)[None]).to(torch.int32)
        mlp, a = self._step(tokens, sources, StepBatch(kv_len, n_valid.to(torch.int32), pos.contiguous()))
        rows = torch.arange(batch, device=dev)
        r = root.long()
        logits, out = self._head(mlp[rows, r], a[rows, r])
        return logits, out

    def tree_step(self, tokens: torch.Tensor, states: torch.Tensor, positions: torch.Tensor, kv_base: torch.Tensor,
                  n_forwarded: int, q_offset: int, mask: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        batch = tokens.shape[0]
        n_new = torch.full((batch,), n_forwarded, dtype=torch.int32, device=tokens.device)
        sb = StepBatch(kv_base.to(torch.int32), n_new, positions.to(torch.int32), mask, q_offset)
        mlp, a = self._step(tokens, states.to(self.t.fc.dtype), sb)
        return self._head(mlp, a)

    def to_target(self, draft_ids: torch.Tensor) -> torch.Tensor:
        return draft_ids + self.t.d2t[draft_ids]
