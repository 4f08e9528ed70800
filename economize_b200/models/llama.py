"""The engine's own decoder executor for Llama-family models (Llama, Mistral, Qwen2, Qwen3, Mixtral-style MoE, and the
variants ``ModelConfig`` describes: Gemma's GeGLU and sandwich norms, soft-caps, sliding windows, shared experts).

Weights are stored fused for the GEMM kernels: ``wqkv = [W_q; W_k; W_v]`` and ``w_gate_up = [W_gate; W_up]`` (one
read of the activations per projection group), in contrast to economize, which calls the Hugging Face decoder layers
(``src/economize/arch/base.py:406-414``). A forward pass runs every layer through :mod:`economize_b200.ops`:

    x, r = rmsnorm(h, attn_norm, r)          # fused residual add + RMSNorm (r: output of the previous blocks)
    q    = rope_store(x @ wqkv.T, cache)      # fused rotary embedding + KV-cache write
    h    = attention(q, cache) @ wo.T         # tree / causal attention over the slot cache
    x, r = rmsnorm(h, mlp_norm, r)
    h    = silu_mul(x @ w_gate_up.T) @ w_down.T

Block outputs that a drafter reads (EAGLE-3's low/mid/high features) are the residual stream ``r`` at the start of
the following block, so capturing them costs nothing.
"""

from __future__ import annotations

import math
from typing import Any

import torch
from torch import nn

from .. import ops
from ..errors import ConfigError
from ..runtime.cache import KVCache, PagedKVCache, SplitKVCache, StepBatch
from .config import ModelConfig, rope_attention_factor, rope_inv_freq

__all__ = ["CausalLM", "DecoderLayer", "init_weights"]


class DecoderLayer(nn.Module):
    """Parameters of one pre-norm decoder block (dense or sparse-MoE MLP)."""

    def __init__(self, config: ModelConfig, dtype: torch.dtype, device: torch.device | str | None) -> None:
        super().__init__()
        h, f = config.hidden_size, config.intermediate_size
        kw = dict(dtype=dtype, device=device)
        #: block size of the online Hadamard rotation of the down projection's input (0: none); set by the
        #: rotate technique, which folds the same rotation into w_down
        self.down_hadamard = 0
        self.attn_norm = nn.Parameter(torch.ones(h, **kw))
        self.wqkv = nn.Parameter(torch.empty(config.q_size + 2 * config.kv_size, h, **kw))
        self.bqkv = nn.Parameter(torch.zeros(config.q_size + 2 * config.kv_size, **kw)) if config.attention_bias \
            else None
        self.wo = nn.Parameter(torch.empty(h, config.q_size, **kw))
        self.bo = nn.Parameter(torch.zeros(h, **kw)) if config.o_bias else None
        # q/k RMSNorm weights: one head's width (per-head norm) or all heads' (a norm over the whole projection)
        qn, kn = (config.q_size, config.kv_size) if config.qk_norm_full else (config.head_dim, config.head_dim)
        self.q_norm = nn.Parameter(torch.ones(qn, **kw)) if config.qk_norm else None
        self.k_norm = nn.Parameter(torch.ones(kn, **kw)) if config.qk_norm else None
        self.mlp_norm = nn.Parameter(torch.ones(h, **kw))
        # sandwich blocks (Gemma-2/3): attn_norm / mlp_norm precede the branches, these follow them
        self.attn_post_norm = nn.Parameter(torch.ones(h, **kw)) if config.sandwich_norm else None
        self.mlp_post_norm = nn.Parameter(torch.ones(h, **kw)) if config.sandwich_norm else None
        # Qwen2-MoE: a dense shared expert next to the routed ones, gated by sigmoid(x . shared_gate)
        se = config.shared_expert_size if config.is_moe else 0
        self.w_shared_gate_up = nn.Parameter(torch.empty(2 * se, h, **kw)) if se else None
        self.w_shared_down = nn.Parameter(torch.empty(h, se, **kw)) if se else None
        self.shared_gate = nn.Parameter(torch.empty(1, h, **kw)) if se and config.shared_expert_gated else None
        #: attention sink logits of this layer's query heads (fp32 [H]; gpt-oss), or None
        self.sinks = nn.Parameter(torch.zeros(config.num_heads, dtype=torch.float32, device=device)) \
            if config.attn_sinks else None
        # gpt-oss: biases of the router [E] and of every expert's projections ([E, 2F] as [gate; up], [E, H])
        self.router_bias = self.b_gate_up = self.b_down = None
        if config.is_moe:
            e = config.num_experts
            self.router = nn.Parameter(torch.empty(e, h, **kw))
            self.w_gate_up = nn.Parameter(torch.empty(e, 2 * f, h, **kw))
            self.w_down = nn.Parameter(torch.empty(e, h, f, **kw))
            if config.moe_bias:
                self.router_bias = nn.Parameter(torch.zeros(e, **kw))
                self.b_gate_up = nn.Parameter(torch.zeros(e, 2 * f, **kw))
                self.b_down = nn.Parameter(torch.zeros(e, h, **kw))
        else:
            self.router = None
            self.w_gate_up = nn.Parameter(torch.empty(2 * f, h, **kw))
            self.w_down = nn.Parameter(torch.empty(h, f, **kw))


class CausalLM(nn.Module):
    """A decoder-only language model executed by the engine's kernels.

    Args:
        config: The architecture.
        dtype: Parameter and activation dtype (bf16 on the GPU, fp32 for the CPU oracle).
        device: Where the parameters live.
    """

    #: class-level defaults, so views built without ``__init__`` (``techniques/_self_draft.py:layer_view``) have them
    placement = None
    _rope_local = None

    def __init__(self, config: ModelConfig, dtype: torch.dtype = torch.bfloat16,
                 device: torch.device | str | None = None) -> None:
        super().__init__()
        self.config = config
        kw = dict(dtype=dtype, device=device)
        self.embed = nn.Parameter(torch.empty(config.vocab_size, config.hidden_size, **kw))
        self.layers = nn.ModuleList(DecoderLayer(config, dtype, device) for _ in range(config.num_layers))
        self.norm = nn.Parameter(torch.ones(config.hidden_size, **kw))
        self.lm_head = None if config.tie_word_embeddings else nn.Parameter(
            torch.empty(config.vocab_size, config.hidden_size, **kw))
        self._rope: tuple[torch.Tensor, torch.Tensor] | None = None
        self._rope_local: tuple[torch.Tensor, torch.Tensor] | None = None
        #: calibration hook ``observer(layer, name, x)`` called with the input of every projection (or None)
        self.observer = None
        #: KV-cache storage set by KV techniques: dtype (None: the compute dtype) and fp8 scales ([L, H_kv] x 2)
        self.kv_dtype: torch.dtype | None = None
        #: KV eviction policy (a kv_evict technique): scores the prompt at prefill, hides evicted slots afterwards
        self.kv_evictor = None
        #: KV coder (kivi): codes committed chunks after every commit; attention reads the codes
        self.kv_quantizer = None
        self.depth_policy = None  # dynamic depth (per-token layer skipping / early exit) of the exact passes
        self.prefill_sparsity = None  # sparse prefill attention (MInference), run as a chunked prefill
        self.kv_scales: tuple[torch.Tensor, torch.Tensor] | None = None
        #: decode and verification passes (at most 64 queries) attend the keys of the last ``exact_tail`` positions
        #: before each query in position order (ops.attention's exact tail), so greedy speculative decoding with
        #: trees up to this deep reproduces plain greedy decoding bit for bit; 0 turns it off
        self.exact_tail = 16
        #: device of every decoder layer under pipeline placement (economize_b200.parallel.pipeline), else None
        self.placement: list[torch.device] | None = None
        #: tensor-parallel group (set by economize_b200.parallel.tp.shard_model) and this rank's shard sizes
        self.tp = None
        self.local = dict(num_heads=config.num_heads, num_kv_heads=config.num_kv_heads,
                          intermediate_size=config.intermediate_size, vocab_offset=0, vocab_size=config.vocab_size)

    # ---- properties --------------------------------------------------------------------------------------------
    @property
    def device(self) -> torch.device:
        return self.embed.device

    @property
    def dtype(self) -> torch.dtype:
        return self.embed.dtype

    @property
    def head_weight(self) -> torch.Tensor:
        return self.embed if self.lm_head is None else self.lm_head

    def rope_tables(self, length: int | None = None, local: bool = False) -> tuple[torch.Tensor, torch.Tensor]:
        """``cos, sin [P, D/2]`` fp32 for positions ``0..P-1`` (computed once per device, like HF: the angle is the
        fp32 product of the position and the inverse frequency). ``local``: the tables of the sliding-window layers
        when their rotary parameters differ (Gemma-3)."""
        need = max(length or 0, self.config.max_position_embeddings)
        local = local and self.config.local_rope is not None
        cached = self._rope_local if local else self._rope
        if cached is None or cached[0].shape[0] < need or cached[0].device != self.device:
            inv = rope_inv_freq(self.config, local=local).to(self.device)
            pos = torch.arange(need, device=self.device, dtype=torch.float32)
            angles = pos[:, None] * inv[None, :]
            cached = (angles.cos().contiguous(), angles.sin().contiguous())
            factor = rope_attention_factor(self.config, local=local)
            if factor != 1.0:  # YaRN scales cos and sin (and so both q and k)
                cached = (cached[0] * factor, cached[1] * factor)
            if local:
                self._rope_local = cached
            else:
                self._rope = cached
        return cached

    def _layer_rope(self, index: int, cos: torch.Tensor, sin: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """The rotary tables layer ``index`` uses: none (NoPE), the sliding layers' own, or the model's."""
        c = self.config
        if index in c.nope_layers:
            return self._identity_rope(cos)
        if c.local_rope is not None and c.window_of(index):
            return self.rope_tables(cos.shape[0], local=True)
        return cos, sin

    def new_cache(self, batch: int, capacity: int, paged: bool = False, rings: bool = False,
                  reserve: int = 512) -> KVCache | PagedKVCache:
        """A zeroed cache in the model's KV format (``kv_dtype``: the compute dtype, or fp8 e4m3 with the per-head
        ``kv_scales`` a KV technique set). ``paged``: a page pool with one page table per layer; ``rings``: the
        sliding-window layers get ring tables of their window (plus ``reserve`` slots a pass may write)."""
        c = self.config
        dtype = self.kv_dtype or self.dtype
        if self.placement is not None:  # one cache per pipeline stage, on the stage's device
            if paged or rings:
                raise ConfigError("pipeline placement keeps contiguous caches (no paged or ring caches)")
            parts, start = [], 0
            while start < c.num_layers:
                dev = self.placement[start]
                stop = start
                while stop < c.num_layers and self.placement[stop] == dev:
                    stop += 1
                scales = None if self.kv_scales is None else tuple(t[start:stop].to(dev) for t in self.kv_scales)
                parts.append((range(start, stop), KVCache(stop - start, batch, self.local["num_kv_heads"], capacity,
                                                          c.head_dim, dtype, dev, scales)))
                start = stop
            return SplitKVCache(parts)
        if paged or rings:
            windows = [c.window_of(i) for i in range(c.num_layers)] if rings else None
            return PagedKVCache(c.num_layers, batch, self.local["num_kv_heads"], capacity, c.head_dim, dtype,
                                self.device, self.kv_scales, windows=windows, reserve=reserve)
        return KVCache(c.num_layers, batch, self.local["num_kv_heads"], capacity, c.head_dim, dtype, self.device,
                       self.kv_scales)

    @property
    def tp_size(self) -> int:
        return 1 if self.tp is None else self.tp.size

    # ---- forward -----------------------------------------------------------------------------------------------
    def embed_tokens(self, tokens: torch.Tensor) -> torch.Tensor:
        h = self.embed[tokens]
        m = self.config.embedding_multiplier
        if m == 1.0:
            return h
        if self.config.embedding_multiplier_in_dtype:  # Gemma multiplies by the normalizer rounded to the dtype
            return h * torch.tensor(m, dtype=h.dtype)
        return h * m

    def _identity_rope(self, cos: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        """cos = 1, sin = 0 tables of ``cos``'s shape: rotary embedding that leaves q and k unchanged (NoPE)."""
        cached = getattr(self, "_nope_tables", None)
        if cached is None or cached[0].shape != cos.shape or cached[0].device != cos.device:
            cached = (torch.ones_like(cos), torch.zeros_like(cos))
            self._nope_tables = cached
        return cached

    def forward_step(self, tokens: torch.Tensor, batch: StepBatch, cache: KVCache,
                     capture: tuple[int, ...] = (), layers: range | None = None, hidden: torch.Tensor | None = None,
                     ) -> tuple[torch.Tensor, dict[int, torch.Tensor]]:
        """Run a pass over ``tokens [B, T]``; returns the final-normed hidden states ``[B, T, H]`` and the captured
        block outputs ``{i: [B, T, H]}`` (``0``: the embeddings, ``i``: the output of ``i`` blocks, ``-1``: the
        final-normed states again, ``-2``: the residual stream after the last block that ran). ``hidden`` replaces
        the embeddings as the input of the first block that runs (with ``layers``: one block on given inputs)."""
        c = self.config
        sparse = self.prefill_sparsity
        if sparse is not None and not sparse.active and hidden is None and layers is None and \
                sparse.covers(tokens, batch):
            return sparse.chunked_forward(self, tokens, batch, cache, capture)
        if self._sequence_parallel(tokens, layers, hidden):
            return self._forward_sp(tokens, batch, cache, capture)
        if c.post_norm or c.sandwich_norm:
            return self._forward_post_norm(tokens, batch, cache, capture, layers, hidden)
        cos, sin = self.rope_tables(cache.capacity)  # every slot's position has a row
        h = self.embed_tokens(tokens) if hidden is None else hidden
        resid: torch.Tensor | None = None
        aux: dict[int, torch.Tensor] = {}
        todo = layers if layers is not None else range(c.num_layers)
        partial = False  # h is a row-parallel partial awaiting its all-reduce (tensor parallelism)
        depth = self.depth_policy if self.depth_policy is not None and self.depth_policy.acts(batch) else None
        if depth is not None:
            depth.begin_pass(batch, h)
        staged = self._stage(batch, cos, sin) if self.placement is not None else None
        for i in todo:
            layer = self.layers[i]
            if staged is not None:  # pipeline placement: the stream moves to the layer's device
                h, resid, partial, batch, cos, sin = staged(i, h, resid, partial)
            gated = depth is not None and depth.gates(i)
            x_in = None
            # a layer view may skip a sublayer (self-drafting): the pending branch output is added at the next norm
            if not getattr(layer, "skip_attn", False):
                h, partial = self._scale_branch(h, partial)
                x, resid = self._norm(h, layer.attn_norm, resid, partial)
                if i in capture:
                    aux[i] = resid
                x_in = resid
                h = self._attention(layer, i, x, batch, cache, cos, sin)
                partial = True
            elif i in capture:
                raise ValueError(f"cannot capture the input of layer {i}: its attention is skipped")
            if not getattr(layer, "skip_mlp", False):
                h, partial = self._scale_branch(h, partial)
                x, resid = self._norm(h, layer.mlp_norm, resid, partial)
                h = self._mlp(layer, x, i)
                partial = True
            if gated and x_in is not None:
                # dynamic depth: the policy decides, per token, how the layer's output enters the stream
                out = resid + self._materialize(h, partial)
                h, resid, partial = depth.combine(i, x_in, out, batch), None, False
        if staged is not None:  # back to the home device (embedding, final norm, LM head, the engine's state)
            h, resid, partial, batch, cos, sin = staged(None, h, resid, partial)
            aux = {k: v.to(self.device) for k, v in aux.items()}
        h, partial = self._scale_branch(h, partial)
        out, resid = self._norm(h, self.norm, resid, partial)
        if c.num_layers in capture:
            aux[c.num_layers] = resid
        if -1 in capture:  # the final-normed hidden states (what the LM head reads)
            aux[-1] = out
        if -2 in capture:
            aux[-2] = resid
        return out, aux

    def _stage(self, batch: StepBatch, cos: torch.Tensor, sin: torch.Tensor):
        """Pipeline placement: a function ``(layer or None, h, resid, partial)`` that moves the residual stream, the
        pass's batch description and the rotary tables to the layer's device (``None``: the home device), with the
        per-device copies of the batch and tables made once per pass."""
        copies: dict[torch.device, tuple[StepBatch, torch.Tensor, torch.Tensor]] = {}

        def move(i, h, resid, partial):
            dev = self.device if i is None else self.placement[i]
            if dev not in copies:
                copies[dev] = (batch.to(dev), cos.to(dev), sin.to(dev))
            if h.device != dev:
                h = self._materialize(h, partial).to(dev)
                partial = False
                resid = None if resid is None else resid.to(dev)
            return (h, resid, partial) + copies[dev]

        return move

    def _scale_branch(self, h, partial: bool):
        """A branch output times Granite's residual multiplier before it joins the residual stream (a no-op for
        the other families; the embeddings entering the first block are never scaled)."""
        m = self.config.residual_multiplier
        if m == 1.0 or not partial:
            return h, partial
        return self._materialize(h, partial) * m, False

    def _forward_post_norm(self, tokens: torch.Tensor, batch: StepBatch, cache: KVCache, capture: tuple[int, ...],
                           layers: range | None, hidden: torch.Tensor | None):
        """:meth:`forward_step` for blocks whose norms follow the branches: ``h = h + norm(attn(h)); h = h +
        norm(mlp(h))`` (OLMo-2/3), or with a norm before each branch too, ``h = h + post(attn(pre(h)))`` (Gemma-2/3),
        then the final norm."""
        c = self.config
        eps = c.rms_norm_eps
        cos, sin = self.rope_tables(cache.capacity)  # every slot's position has a row
        h = self.embed_tokens(tokens) if hidden is None else hidden
        aux: dict[int, torch.Tensor] = {}
        sandwich = c.sandwich_norm
        staged = self._stage(batch, cos, sin) if self.placement is not None else None
        for i in (layers if layers is not None else range(c.num_layers)):
            layer = self.layers[i]
            if staged is not None:
                h, _, _, batch, cos, sin = staged(i, h, None, False)
            if i in capture:
                aux[i] = h
            x = ops.rmsnorm(h, layer.attn_norm, eps)[0] if sandwich else h
            a = self._materialize(self._attention(layer, i, x, batch, cache, cos, sin), True)
            h = h + ops.rmsnorm(a, layer.attn_post_norm if sandwich else layer.attn_norm, eps)[0]
            x = ops.rmsnorm(h, layer.mlp_norm, eps)[0] if sandwich else h
            m = self._materialize(self._mlp(layer, x, i), True)
            h = h + ops.rmsnorm(m, layer.mlp_post_norm if sandwich else layer.mlp_norm, eps)[0]
        if staged is not None:
            h, _, _, batch, cos, sin = staged(None, h, None, False)
            aux = {k: v.to(self.device) for k, v in aux.items()}
        out = ops.rmsnorm(h, self.norm, eps)[0]
        if c.num_layers in capture or -2 in capture:
            aux[c.num_layers] = aux[-2] = h
        if -1 in capture:
            aux[-1] = out
        return out, aux

    # ---- sequence-parallel tensor parallelism ------------------------------------------------------------------
    def _sequence_parallel(self, tokens: torch.Tensor, layers, hidden) -> bool:
        """Whether a pass runs on the fused reduce-scatter / all-gather kernels (parallel/sp.py): a whole-model pass
        of a dense model without per-token layer policies, views that skip sublayers, or calibration hooks."""
        tp = self.tp
        sp = getattr(tp, "sp", None) if tp is not None else None
        if sp is None or layers is not None or hidden is not None or not sp.fits(tokens.numel()) or \
                self.placement is not None:
            return False
        c = self.config
        if c.is_moe or self.observer is not None or self.depth_policy is not None or c.post_norm or \
                c.qk_norm_full or c.residual_multiplier != 1.0 or c.sandwich_norm or c.hidden_act != "silu" or \
                c.final_softcap or c.o_bias:
            return False
        return not any(getattr(layer, name, None) for layer in self.layers
                       for name in ("skip_attn", "skip_mlp", "mlp_rule", "attn_input_hook"))

    def _forward_sp(self, tokens: torch.Tensor, batch: StepBatch, cache: KVCache, capture: tuple[int, ...]):
        """:meth:`forward_step` with the residual stream split by token between the sublayers: every sublayer is
        an all-gather -> GEMM, this rank's heads or features, and a GEMM -> reduce-scatter whose owner adds the
        residual, applies the next RMSNorm and all-gathers the result."""
        c, sp = self.config, self.tp.sp
        eps = c.rms_norm_eps
        B, T = tokens.shape
        M = B * T
        cos, sin = self.rope_tables(cache.capacity)  # every slot's position has a row
        emb = self.embed_tokens(tokens)
        lo, n = sp.shard(M)
        resid = emb.reshape(M, -1)[lo:lo + n].contiguous()
        wanted = sorted({i for i in capture if 0 < i <= c.num_layers} | ({c.num_layers} if -2 in capture else set()))
        if len(wanted) > sp.n_cap:
            raise ConfigError(f"{len(wanted)} captured block outputs exceed the {sp.n_cap} capture slots")
        slot_of = {layer: slot for slot, layer in enumerate(wanted)}
        resid = sp.reduce_norm(resid, self.layers[0].attn_norm, eps, M, partials=False)
        for i, layer in enumerate(self.layers):
            if layer.bqkv is not None:
                qkv = (sp.ag_linear(layer.wqkv, M) + layer.bqkv).reshape(B, T, -1)
            else:  # split-K partials go straight into the rope / KV-store kernel
                qkv = sp.ag_linear_parts(layer.wqkv, M, (B, T))
            o = self._attend(layer, i, qkv, batch, cache, cos, sin)
            sp.rs_linear(o, layer.wo)
            resid = sp.reduce_norm(resid, layer.mlp_norm, eps, M)
            a = ops.glu(sp.ag_linear_parts(layer.w_gate_up, M, (M,)), self.config.hidden_act,
                        self.config.swiglu_limit, hadamard=layer.down_hadamard)
            sp.rs_linear(a, layer.w_down)
            nxt = self.layers[i + 1].attn_norm if i + 1 < len(self.layers) else self.norm
            resid = sp.reduce_norm(resid, nxt, eps, M, capture=slot_of.get(i + 1, -1))
        out = sp.fetch(M, emb).reshape(B, T, -1)
        aux: dict[int, torch.Tensor] = {}
        if 0 in capture:
            aux[0] = emb
        for layer_index, slot in slot_of.items():  # valid now: the fetch consumed the pass's last round
            aux[layer_index] = sp.captured(slot, M, emb).reshape(B, T, -1)
        if -1 in capture:
            aux[-1] = out
        if -2 in capture:
            aux[-2] = aux[c.num_layers]
        return out, aux

    def _materialize(self, h, partial: bool) -> torch.Tensor:
        """A branch output as a plain tensor: split-K partials summed, a row-parallel partial all-reduced."""
        if isinstance(h, ops.Partials):
            h = h.sum()
        tp = self.tp
        if partial and tp is not None and tp.size > 1:
            from ..parallel.comm import Pushed

            if isinstance(h, Pushed):
                raise ValueError("dynamic depth needs the all-reduced branch output; disable the fused push mode")
            h = tp.all_reduce(h)
        return h

    def _norm(self, h: torch.Tensor, weight: torch.Tensor, resid: torch.Tensor | None,
              partial: bool) -> tuple[torch.Tensor, torch.Tensor]:
        """Residual add + RMSNorm; under tensor parallelism a row-parallel partial ``h`` is first summed over the
        ranks (NCCL, or the fused NVLink push/reduce kernels that also do the add and the norm)."""
        eps = self.config.rms_norm_eps
        tp = self.tp
        if not partial or tp is None or tp.size == 1:
            return ops.rmsnorm(h, weight, eps, resid)
        from ..parallel.comm import Pushed

        if isinstance(h, Pushed) or (tp.fused and tp.comm is not None and tp.comm.fits(h.numel() // h.shape[-1])):
            return tp.comm.reduce_rmsnorm(h, weight, eps, resid)
        return ops.rmsnorm(tp.all_reduce(h), weight, eps, resid)

    def _attention(self, layer: DecoderLayer, index: int, x: torch.Tensor, batch: StepBatch, cache: KVCache,
                   cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        c = self.config
        if self.observer is not None:
            self.observer(index, "wqkv", x)
        hook = getattr(layer, "attn_input_hook", None)  # Deja Vu's lookahead predictors read the attention input
        if hook is not None:
            hook(x)
        qkv = self._linear(x, layer.wqkv) if layer.bqkv is None else ops.linear(x, layer.wqkv, layer.bqkv)
        o = self._attend(layer, index, qkv, batch, cache, cos, sin)
        if self.observer is not None:
            self.observer(index, "wo", o)
        if layer.bo is None:
            return self._row_linear(o, layer.wo)
        # the output bias joins once: on rank 0's partial sum under tensor parallelism
        first = self.tp is None or self.tp.size == 1 or self.tp.rank == 0
        return ops.linear(o, layer.wo, layer.bo if first else None)

    def _attend(self, layer: DecoderLayer, index: int, qkv, batch: StepBatch, cache: KVCache, cos: torch.Tensor,
                sin: torch.Tensor) -> torch.Tensor:
        """Rotary embedding + KV-cache write of a QKV projection and the attention over the cache: the heads'
        outputs ``[B, T, H_q * D]`` (this rank's heads under tensor parallelism)."""
        c = self.config
        k_cache, v_cache = cache.layer(index)
        pages = cache.pages(index)  # a paged cache's table (None: contiguous)
        k_scale, v_scale = cache.layer_scales(index)
        q_norm, k_norm = layer.q_norm, layer.k_norm
        if c.qk_norm_full and q_norm is not None:  # RMSNorm over all heads' features of q and of k (OLMo-2)
            if isinstance(qkv, ops.Partials):
                qkv = qkv.sum()
            qs, ks = self.local["num_heads"] * c.head_dim, self.local["num_kv_heads"] * c.head_dim
            q_part, k_part, v_part = qkv.split([qs, ks, ks], -1)
            q_part = ops.rmsnorm(q_part.contiguous(), q_norm, c.rms_norm_eps)[0]
            k_part = ops.rmsnorm(k_part.contiguous(), k_norm, c.rms_norm_eps)[0]
            qkv = torch.cat([q_part, k_part, v_part], -1)
            q_norm = k_norm = None
        cos, sin = self._layer_rope(index, cos, sin)
        q = ops.rope_store(qkv, batch.positions, cos, sin, self.local["num_heads"], self.local["num_kv_heads"],
                           c.head_dim, k_cache,
                           v_cache, batch.kv_len, batch.n_new, q_norm, k_norm, c.rms_norm_eps,
                           q_offset=batch.q_offset, k_scale=k_scale, v_scale=v_scale, pages=pages)
        if c.query_position_scale is not None:  # Ministral-3: 1 + beta ln(1 + floor(p / original)), in q's dtype
            beta, original = c.query_position_scale
            pos = batch.positions.to(torch.float32)
            q = q * (1.0 + beta * torch.log1p(torch.floor(pos / original))).to(q.dtype)[..., None, None]
        keep = self.kv_evictor.keep_for(index, k_cache, q, batch) if self.kv_evictor is not None else None
        sparse = self.prefill_sparsity
        if sparse is not None and sparse.active:  # sparse prefill (MInference): keys the chunk's pattern hides
            pattern = sparse.keep_for(index, k_cache, q, batch)
            if pattern is not None:
                keep = pattern if keep is None else keep & pattern
        kivi = self.kv_quantizer.layer_args(index, cache) if self.kv_quantizer is not None else {}
        sparse_pass = sparse is not None and sparse.active
        tail = self.exact_tail if (not batch.prompt and q.shape[1] <= 64 and not sparse_pass) else 0
        o = ops.attention(q, k_cache, v_cache, batch.kv_len, batch.n_new, batch.mask, scale=c.attention_multiplier,
                          q_offset=batch.q_offset, k_scale=k_scale, v_scale=v_scale, keep=keep, tail=tail,
                          softcap=c.attn_softcap, sinks=None if layer.sinks is None else layer.sinks.float(),
                          window=c.window_of(index), pages=pages,
                          **kivi)
        if self.kv_evictor is not None and batch.is_prefill:
            self.kv_evictor.observe_prefill(index, q, k_cache, v_cache, batch)
        return o.reshape(*o.shape[:2], -1)

    def _linear(self, x: torch.Tensor, weight):
        """A projection whose consumer is one of the engine's fused elementwise kernels: without tensor
        parallelism the GEMM may hand over its split-K partials (:class:`~economize_b200.ops.Partials`), which the
        consumer reduces while reading them."""
        if (self.tp is None or self.tp.size == 1) and self.placement is None:
            return ops.linear_parts(x, weight)
        return ops.linear(x, weight)

    def _row_linear(self, x: torch.Tensor, weight: torch.Tensor):
        """A row-parallel projection (``wo``, ``w_down``): under fused tensor parallelism the GEMM pushes its
        partial output to the peers itself and returns a :class:`~economize_b200.parallel.comm.Pushed` marker."""
        tp = self.tp
        if tp is not None and tp.size > 1 and tp.fused and tp.comm is not None and isinstance(weight, torch.Tensor) \
                and tp.comm.fits(x.numel() // x.shape[-1]):
            return tp.comm.gemm_push(x, weight)
        return self._linear(x, weight)

    def _mlp(self, layer: DecoderLayer, x: torch.Tensor, index: int = -1) -> torch.Tensor:
        if layer.router is not None:
            from ..parallel.moe import moe_mlp

            c = self.config
            biases = None if layer.router_bias is None else (layer.router_bias, layer.b_gate_up, layer.b_down)
            out = moe_mlp(x, layer.router, layer.w_gate_up, layer.w_down, c.experts_per_token,
                          getattr(self, "ep", None), renormalize=c.norm_topk_prob, act=c.hidden_act,
                          limit=c.swiglu_limit, biases=biases)
            if layer.w_shared_gate_up is not None:  # a shared expert: Qwen2-MoE gates it, GraniteMoE-shared not
                shared = ops.linear(ops.silu_mul(ops.linear(x, layer.w_shared_gate_up)), layer.w_shared_down)
                if layer.shared_gate is not None:
                    shared = torch.sigmoid(ops.linear(x, self._gate_rows(layer))[..., :1]) * shared
                out = out + shared
            return out
        if self.observer is not None:
            self.observer(index, "w_gate_up", x)
        rule = getattr(layer, "mlp_rule", None)  # activation-sparse MLPs (CATS, Deja Vu); None: the dense path
        if rule is not None:
            out = rule(self, layer, x, index)
            if out is not None:
                return out
        a = ops.glu(self._linear(x, layer.w_gate_up), self.config.hidden_act, self.config.swiglu_limit,
                    hadamard=layer.down_hadamard)
        if self.observer is not None:
            self.observer(index, "w_down", a)
        return self._row_linear(a, layer.w_down)

    @staticmethod
    def _gate_rows(layer: DecoderLayer) -> torch.Tensor:
        """The shared expert's gate vector as the first of four rows (the GEMM kernels take N in multiples of 4;
        the zero rows cost nothing next to the expert GEMMs)."""
        w = layer.shared_gate
        if not w.is_cuda:
            return w
        key = (w.data_ptr(), w._version)
        if getattr(layer, "_gate4_key", None) != key:
            layer._gate4 = torch.cat([w.detach(), w.new_zeros(3, w.shape[1])], 0)
            layer._gate4_key = key
        return layer._gate4

    def begin_sequence(self, cache: KVCache) -> None:
        """A new generation starts in ``cache`` (slot 0 on)."""
        if self.kv_quantizer is not None:
            self.kv_quantizer.reset(cache)

    def after_commit(self, cache: KVCache | PagedKVCache, kv_len: torch.Tensor, prefill: bool = False) -> None:
        """Tokens up to ``kv_len`` are committed (KV coders compress what became old)."""
        if self.kv_quantizer is not None:
            self.kv_quantizer.after_commit(cache, kv_len, max(1, cache.capacity // 128) if prefill else 1)

    def logits(self, hidden: torch.Tensor) -> torch.Tensor:
        """Logits over the full vocabulary (gathered from the vocabulary shards under tensor parallelism)."""
        local = self._soft_cap(ops.linear(hidden, self.head_weight))
        scale = self.config.logits_scaling
        if scale != 1.0:  # Granite divides its logits (a positive scale: the argmax is unchanged)
            local = local / scale
        if self.tp is None or self.tp.size == 1:
            return local
        every = self.tp.all_gather(local)  # [P, ..., V/P]
        return torch.cat(list(every.unbind(0)), -1)

    def _soft_cap(self, logits: torch.Tensor) -> torch.Tensor:
        """Gemma-2's final-logit soft-cap ``cap * tanh(logits / cap)`` (in the logits' dtype, as HF computes it)."""
        cap = self.config.final_softcap
        if not cap:
            return logits
        return torch.tanh(logits / cap) * cap

    def greedy(self, hidden: torch.Tensor) -> torch.Tensor:
        """Argmax token after every row of ``hidden`` (distributed over vocabulary shards under TP, without
        gathering the logits)."""
        # the soft-cap is monotonic, but its rounding can tie two logits, and the first of a tie wins
        local = self._soft_cap(ops.linear(hidden, self.head_weight))
        if self.tp is None or self.tp.size == 1:
            return ops.argmax(local)
        from ..parallel.tp import tp_argmax

        return tp_argmax(local, self.tp, self.local["vocab_offset"])

    # ---- Hugging Face interop ----------------------------------------------------------------------------------
    @classmethod
    def from_hf(cls, hf_model: nn.Module, dtype: torch.dtype | None = None,
                device: torch.device | str | None = None) -> CausalLM:
        """Build from a ``transformers`` causal LM of a supported family (weights are copied into fused tensors)."""
        from .hf import load_hf_state

        config = ModelConfig.from_hf(hf_model.config)
        first = next(hf_model.parameters())
        model = cls(config, dtype or first.dtype, device or first.device)
        load_hf_state(model, hf_model.state_dict())
        return model

    def hf_state_dict(self, copy: bool = True) -> dict[str, torch.Tensor]:
        from .hf import export_hf_state

        return export_hf_state(self, copy)


@torch.no_grad()
def init_weights(model: CausalLM, seed: int = 0, std: float = 0.02, scaled_residual: bool = False) -> CausalLM:
    """Random initialisation N(0, std) of every matrix (norms at one), generated on the model's device from
    ``seed`` in a fixed order, so two processes build identical weights. With ``scaled_residual`` the output
    projections of the residual branches (``wo``, ``w_down``) use ``std / sqrt(2 * num_layers)`` (the GPT-2 /
    Megatron initialisation), which keeps a deep random model's residual stream from being dominated by noise."""
    gen = torch.Generator(device=model.device)
    gen.manual_seed(seed)
    out_std = std / math.sqrt(2 * model.config.num_layers)
    for name, p in model.named_parameters():
        if p.dim() >= 2:
            s = out_std if scaled_residual and name.rsplit(".", 1)[-1] in ("wo", "w_down") else std
            p.copy_(torch.randn(p.shape, generator=gen, device=p.device, dtype=torch.float32).mul_(s))
        elif "norm" in name:
            p.fill_(1.0)
        else:
            p.zero_()
    return model


def describe(model: CausalLM) -> dict[str, Any]:
    c = model.config
    return {"layers": c.num_layers, "hidden": c.hidden_size, "params": c.num_parameters(), "dtype": str(model.dtype)}
