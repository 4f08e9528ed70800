"""One draft decoder layer on the engine's kernels, with its own slot KV cache.

``a = r + o_proj(Attention(x))``, ``y = a + MLP(norm_post(a))`` (economize ``_draft_layer/layer.py:36-155``): the
input ``x`` and residual ``r`` come from the subclass (EAGLE-3: ``x = [norm_e(embed); norm_h(g)]``, ``r = g``).
Queries/keys are rotated and the keys/values stored by the fused rope_store kernel, attention runs on the tree
attention kernel over the draft cache, so draft steps take the same sm_100a path as the target.
"""

from __future__ import annotations

import torch
from torch import nn

from ... import ops
from ...models.config import ModelConfig, rope_inv_freq
from ...runtime.cache import KVCache, StepBatch

__all__ = ["DraftLayer"]


class DraftLayer(nn.Module):
    """Parameters of the draft layer; ``input_size`` is the width of the attention input."""

    def __init__(self, input_size: int, hidden: int, intermediate: int, heads: int, kv_heads: int, head_dim: int,
                 eps: float, bias: bool, dtype: torch.dtype, device: torch.device | str | None) -> None:
        super().__init__()
        kw = dict(dtype=dtype, device=device)
        self.heads, self.kv_heads, self.head_dim, self.eps = heads, kv_heads, head_dim, eps
        self.wqkv = nn.Parameter(torch.empty((heads + 2 * kv_heads) * head_dim, input_size, **kw))
        self.bqkv = nn.Parameter(torch.zeros((heads + 2 * kv_heads) * head_dim, **kw)) if bias else None
        self.wo = nn.Parameter(torch.empty(hidden, heads * head_dim, **kw))
        self.post_norm = nn.Parameter(torch.ones(hidden, **kw))
        self.w_gate_up = nn.Parameter(torch.empty(2 * intermediate, hidden, **kw))
        self.w_down = nn.Parameter(torch.empty(hidden, intermediate, **kw))
        self._rope: tuple[torch.Tensor, torch.Tensor] | None = None
        self._rope_config: ModelConfig | None = None

    def set_rope(self, config: ModelConfig) -> None:
        self._rope_config = config
        self._rope = None

    def rope(self, length: int = 0) -> tuple[torch.Tensor, torch.Tensor]:
        """``cos, sin`` tables with a row for every position below ``length`` (at least the configuration's
        ``max_position_embeddings``)."""
        dev = self.wqkv.device
        need = max(length, self._rope_config.max_position_embeddings)
        if self._rope is None or self._rope[0].device != dev or self._rope[0].shape[0] < need:
            inv = rope_inv_freq(self._rope_config).to(dev)
            pos = torch.arange(need, device=dev, dtype=torch.float32)
            ang = pos[:, None] * inv[None]
            self._rope = (ang.cos().contiguous(), ang.sin().contiguous())
        return self._rope

    def run(self, x: torch.Tensor, residual: torch.Tensor, cache: KVCache,
            batch: StepBatch) -> tuple[torch.Tensor, torch.Tensor]:
        """``(mlp, a)`` for attention inputs ``x`` and residuals ``residual`` ``[B, T, *]``: the layer output is
        ``a + mlp``, which the caller adds inside its next fused RMSNorm (the draft head's norm); ``mlp`` may be
        split-K :class:`~economize_b200.ops.Partials` that the norm reduces."""
        cos, sin = self.rope(cache.capacity)  # every slot's position has a row
        k_cache, v_cache = cache.layer(0)
        qkv = ops.linear_parts(x, self.wqkv) if self.bqkv is None else ops.linear(x, self.wqkv, self.bqkv)
        q = ops.rope_store(qkv, batch.positions, cos, sin, self.heads, self.kv_heads, self.head_dim, k_cache,
                           v_cache, batch.kv_len, batch.n_new, None, None, self.eps, q_offset=batch.q_offset)
        o = ops.attention(q, k_cache, v_cache, batch.kv_len, batch.n_new, batch.mask, q_offset=batch.q_offset)
        # split-K partials go straight into the consuming rope / norm / SwiGLU kernels
        h = ops.linear_parts(o.reshape(*o.shape[:2], -1), self.wo)
        x2, a = ops.rmsnorm(h, self.post_norm, self.eps, residual)
        return ops.linear_parts(ops.silu_mul(ops.linear_parts(x2, self.w_gate_up)), self.w_down), a
