"""Architecture description of the decoder models the engine executes.

:class:`ModelConfig` is read from a Hugging Face ``config.json`` / ``PretrainedConfig`` (the families economize's
``arch/families/llama.py``, ``mistral.py``, ``qwen2.py``, ``qwen3.py`` and ``mixtral.py`` adapters cover) or built
directly, e.g. :func:`llama31_8b` for the benchmark's random-init Llama-3.1-8B architecture.
"""

from __future__ import annotations

import math
from dataclasses import asdict, dataclass, field
from typing import Any

import torch

from ..errors import UnsupportedModelError

__all__ = ["ModelConfig", "SUPPORTED_MODEL_TYPES", "gpt_oss_20b", "llama31_8b", "llama31_70b", "mixtral_8x7b",
           "rope_attention_factor", "rope_inv_freq", "tiny_llama"]

#: ``model_type`` values whose decoder layer is the Llama block (attention + gated MLP with RMSNorms), with the
#: differences expressed as fields: q/k/v bias (qwen2), per-head q/k RMSNorm (qwen3, qwen3_moe), sparse MoE MLP
#: (mixtral, qwen3_moe), embedding / residual / attention / logit multipliers (granite), fused projections in the
#: checkpoint (phi3), layers without rotary embedding (smollm3), norms after each branch and q/k RMSNorm over all
#: heads (olmo2).
#: Also: GeGLU MLPs, (1 + w) RMSNorms and a dtype-rounded embedding scale (gemma, gemma2, gemma3_text), a norm
#: before and after each branch with tanh soft-capped attention scores and logits (gemma2) or per-head q/k norms and
#: separate rotary tables for the sliding-window layers (gemma3_text), per-layer sliding windows (mistral, ministral,
#: gemma2, gemma3_text, olmo3, qwen2 with use_sliding_window), sparse MoE with q/k norms (olmoe) and a gated shared
#: expert (qwen2_moe), and biased projections everywhere with attention sink logits, YaRN rotary scaling and
#: clamped-SwiGLU experts (gpt_oss), Granite's scales around MoE blocks with an ungated shared expert (granitemoe,
#: granitemoeshared), and YaRN with position-scaled queries (ministral3).
SUPPORTED_MODEL_TYPES = ("llama", "mistral", "qwen2", "qwen3", "mixtral", "granite", "phi3", "smollm3", "olmo2",
                         "qwen3_moe", "gemma", "gemma2", "gemma3_text", "ministral", "olmo3", "olmoe", "qwen2_moe",
                         "gpt_oss", "granitemoe", "granitemoeshared", "ministral3", "economize_b200")

#: the layer kinds of ``ModelConfig.layer_types``
FULL, SLIDING = "full_attention", "sliding_attention"


@dataclass
class ModelConfig:
    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_layers: int
    num_heads: int
    num_kv_heads: int
    head_dim: int | None = None
    rms_norm_eps: float = 1e-5
    rope_theta: float = 10000.0
    rope_scaling: dict[str, Any] | None = None
    max_position_embeddings: int = 8192
    tie_word_embeddings: bool = False
    attention_bias: bool = False
    qk_norm: bool = False
    num_experts: int = 0
    experts_per_token: int = 2
    model_type: str = "llama"
    #: top-k router weights renormalised to sum to one (Mixtral); False keeps the softmax probabilities (Qwen3-MoE)
    norm_topk_prob: bool = True
    #: scales of Granite: embeddings, each branch output before the residual add, attention logits (replaces
    #: 1/sqrt(head_dim) when set), and a divisor of the LM head's logits
    embedding_multiplier: float = 1.0
    residual_multiplier: float = 1.0
    attention_multiplier: float | None = None
    logits_scaling: float = 1.0
    #: OLMo-2 block: each branch's output is normed before it joins the residual stream (no input norms)
    post_norm: bool = False
    #: q/k RMSNorm over all heads' features at once (OLMo-2) instead of per head (Qwen3)
    qk_norm_full: bool = False
    #: layers whose attention runs without rotary embedding (SmolLM3's NoPE layers)
    nope_layers: tuple[int, ...] = ()
    #: gated MLP activation: "silu" (SwiGLU), "gelu_tanh" (GeGLU, Gemma) or "clamped_swiglu" (gpt-oss:
    #: (clamp(up, +-swiglu_limit) + 1) * g * sigmoid(1.702 g), g = min(gate, swiglu_limit))
    hidden_act: str = "silu"
    swiglu_limit: float = 7.0
    #: Gemma's RMSNorms scale by (1 + w): checkpoints store w, this model stores 1 + w
    norm_unit_offset: bool = False
    #: the embedding multiplier is rounded to the model dtype before it multiplies (Gemma's normalizer)
    embedding_multiplier_in_dtype: bool = False
    #: Gemma-2/3 blocks: an RMSNorm before and after each branch (OLMo-2's post_norm has only the one after)
    sandwich_norm: bool = False
    #: tanh soft-caps (s -> cap * tanh(s / cap)) of the attention scores and of the final logits (Gemma-2)
    attn_softcap: float | None = None
    final_softcap: float | None = None
    #: attention kind of every layer ("full_attention" / "sliding_attention"; empty: all full) and the window
    layer_types: tuple[str, ...] = ()
    sliding_window: int = 0
    #: rotary parameters of the sliding-window layers when they differ from the others' (Gemma-3: {"rope_theta":
    #: 1e4}; keys as ``rope_scaling`` plus ``rope_theta``)
    local_rope: dict[str, Any] | None = None
    #: width of a shared expert added to every sparse MoE MLP, gated by sigmoid(x . w) (Qwen2-MoE) or added as it
    #: is (``shared_expert_gated=False``, GraniteMoE-shared); 0: none
    shared_expert_size: int = 0
    shared_expert_gated: bool = True
    #: queries scaled by 1 + beta ln(1 + floor(position / original)) after the rotary embedding (Ministral-3's
    #: ``llama_4_scaling_beta``): (beta, original), or None
    query_position_scale: tuple[float, float] | None = None
    #: gpt-oss: a bias on the attention output projection, one learned sink logit per query head that joins every
    #: softmax denominator, and biases on the router and on both expert projections
    o_bias: bool = False
    attn_sinks: bool = False
    moe_bias: bool = False
    extra: dict[str, Any] = field(default_factory=dict)

    def __post_init__(self) -> None:
        if self.head_dim is None:
            self.head_dim = self.hidden_size // self.num_heads
        self.nope_layers = tuple(int(i) for i in self.nope_layers)
        if self.query_position_scale is not None:
            beta, original = self.query_position_scale
            self.query_position_scale = (float(beta), float(original))
        self.layer_types = tuple(str(t) for t in self.layer_types)
        if self.num_heads % self.num_kv_heads:
            raise UnsupportedModelError(f"{self.num_heads} heads do not split into {self.num_kv_heads} KV groups")
        if self.hidden_act not in ("silu", "gelu_tanh", "clamped_swiglu"):
            raise UnsupportedModelError(f"gated activation {self.hidden_act!r} is not supported")
        if self.layer_types and len(self.layer_types) != self.num_layers:
            raise UnsupportedModelError(f"{len(self.layer_types)} layer types for {self.num_layers} layers")
        unknown = set(self.layer_types) - {FULL, SLIDING}
        if unknown:
            raise UnsupportedModelError(f"layer types {sorted(unknown)} are not supported")
        if SLIDING in self.layer_types and self.sliding_window < 1:
            raise UnsupportedModelError("sliding-window layers need sliding_window >= 1")

    def window_of(self, layer: int) -> int:
        """The attention window of ``layer`` in positions (0: the whole context)."""
        if self.layer_types and self.layer_types[layer] == SLIDING:
            return int(self.sliding_window)
        return 0

    @property
    def q_size(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_kv_heads * self.head_dim

    @property
    def is_moe(self) -> bool:
        return self.num_experts > 0

    def num_parameters(self) -> int:
        h, f, layers = self.hidden_size, self.intermediate_size, self.num_layers
        attn = h * (self.q_size + 2 * self.kv_size) + self.q_size * h
        mlp = 3 * h * f * (self.num_experts if self.is_moe else 1) + (h * self.num_experts if self.is_moe else 0)
        mlp += 3 * h * self.shared_expert_size + (h if self.shared_expert_size and self.shared_expert_gated else 0)
        if self.moe_bias:
            mlp += self.num_experts * (2 * f + h + 1)
        attn += (h if self.o_bias else 0) + (self.num_heads if self.attn_sinks else 0)
        embed = self.vocab_size * h * (1 if self.tie_word_embeddings else 2)
        return layers * (attn + mlp + 2 * h) + embed + h

    def to_dict(self) -> dict[str, Any]:
        return asdict(self)

    @classmethod
    def from_dict(cls, data: dict[str, Any]) -> ModelConfig:
        known = set(cls.__dataclass_fields__)
        return cls(**{k: v for k, v in data.items() if k in known})

    @classmethod
    def from_hf(cls, hf: Any) -> ModelConfig:
        """From a ``transformers`` config object or its ``config.json`` dict."""
        get = (lambda k, d=None: hf.get(k, d)) if isinstance(hf, dict) else (lambda k, d=None: getattr(hf, k, d))
        model_type = get("model_type", "llama")
        if model_type not in SUPPORTED_MODEL_TYPES:
            raise UnsupportedModelError(f"model_type {model_type!r} is not supported; supported: "
                                        f"{', '.join(SUPPORTED_MODEL_TYPES)}")
        rope = get("rope_scaling") or get("rope_parameters")
        if isinstance(rope, dict) and float(rope.get("partial_rotary_factor", 1.0)) != 1.0:
            raise UnsupportedModelError(f"{model_type}: partial rotary embedding (factor "
                                        f"{rope['partial_rotary_factor']}) is not supported")
        if float(get("partial_rotary_factor", 1.0) or 1.0) != 1.0:
            raise UnsupportedModelError(f"{model_type}: partial rotary embedding is not supported")
        heads = int(get("num_attention_heads"))
        layers = int(get("num_hidden_layers"))
        extra: dict[str, Any] = {}
        # per-layer attention kinds: transformers 5 writes layer_types; Mistral (and Qwen2 with use_sliding_window)
        # express a window without them
        window = int(get("sliding_window", 0) or 0)
        kinds = list(get("layer_types", None) or [])
        if model_type == "qwen2" and not get("use_sliding_window", False):
            kinds, window = [], 0
        if not kinds and window and model_type in ("mistral", "ministral", "ministral3"):
            kinds = [SLIDING] * layers
        if kinds and SLIDING in kinds:
            extra.update(layer_types=tuple(kinds), sliding_window=window)
        elif model_type != "qwen2" and get("use_sliding_window", False):
            raise UnsupportedModelError(f"{model_type}: use_sliding_window without layer types is not supported")
        # Gemma-3 keeps one rotary parameter set per layer kind
        if isinstance(rope, dict) and isinstance(rope.get(FULL), dict):
            local = rope.get(SLIDING)
            rope = dict(rope[FULL])
            if isinstance(local, dict):
                extra["local_rope"] = dict(local)
        theta = get("rope_theta")
        if theta is None and isinstance(rope, dict):
            theta = rope.get("rope_theta")
        if isinstance(rope, dict) and rope.get("rope_type", rope.get("type", "default")) in ("default", None):
            rope = None
        if model_type in ("gemma", "gemma2", "gemma3_text"):
            act = get("hidden_activation") or get("hidden_act")
            if act not in ("gelu_pytorch_tanh", "gelu_tanh"):
                raise UnsupportedModelError(f"{model_type}: activation {act!r} is not supported")
            extra.update(hidden_act="gelu_tanh", norm_unit_offset=True, embedding_multiplier_in_dtype=True,
                         embedding_multiplier=float(get("hidden_size")) ** 0.5)
            if model_type != "gemma":
                qpas = get("query_pre_attn_scalar")
                extra.update(sandwich_norm=True, attention_multiplier=float(qpas) ** -0.5 if qpas else None,
                             attn_softcap=get("attn_logit_softcapping"), final_softcap=get("final_logit_softcapping"))
        elif model_type == "gpt_oss":
            extra.update(hidden_act="clamped_swiglu", swiglu_limit=float(get("swiglu_limit", 7.0) or 7.0),
                         o_bias=True, attn_sinks=True, moe_bias=True)
        elif (get("hidden_act") or "silu") != "silu":
            raise UnsupportedModelError(f"{model_type}: activation {get('hidden_act')!r} is not supported")
        experts = int(get("num_local_experts", 0) or get("num_experts", 0) or 0)
        ffn = int(get("intermediate_size"))
        if model_type == "qwen3_moe":
            if int(get("decoder_sparse_step", 1) or 1) != 1 or list(get("mlp_only_layers", []) or []):
                raise UnsupportedModelError("qwen3_moe with dense layers between the sparse ones is not supported")
            ffn = int(get("moe_intermediate_size"))
        if model_type == "smollm3":
            flags = list(get("no_rope_layers", []) or [])
            extra["nope_layers"] = tuple(i for i, use_rope in enumerate(flags) if not use_rope)
        if model_type in ("granite", "granitemoe", "granitemoeshared"):
            extra.update(embedding_multiplier=float(get("embedding_multiplier", 1.0)),
                         residual_multiplier=float(get("residual_multiplier", 1.0)),
                         attention_multiplier=float(get("attention_multiplier", 1.0)),
                         logits_scaling=float(get("logits_scaling", 1.0)))
        if model_type in ("olmo2", "olmo3"):
            extra.update(post_norm=True, qk_norm_full=True)
        if model_type == "olmoe":
            if get("clip_qkv"):
                raise UnsupportedModelError("olmoe with clip_qkv is not supported")
            extra.update(qk_norm_full=True)
        if model_type == "granitemoeshared":
            extra.update(shared_expert_size=int(get("shared_intermediate_size", 0) or 0), shared_expert_gated=False)
        if model_type == "ministral3" and isinstance(rope, dict) and rope.get("llama_4_scaling_beta"):
            extra["query_position_scale"] = (float(rope["llama_4_scaling_beta"]),
                                             float(rope["original_max_position_embeddings"]))
        if model_type == "qwen2_moe":
            if int(get("decoder_sparse_step", 1) or 1) != 1 or list(get("mlp_only_layers", []) or []):
                raise UnsupportedModelError("qwen2_moe with dense layers between the sparse ones is not supported")
            ffn = int(get("moe_intermediate_size"))
            extra["shared_expert_size"] = int(get("shared_expert_intermediate_size", 0) or 0)
        return cls(
            vocab_size=int(get("vocab_size")),
            hidden_size=int(get("hidden_size")),
            intermediate_size=ffn,
            num_layers=layers,
            num_heads=heads,
            num_kv_heads=int(get("num_key_value_heads") or heads),
            head_dim=get("head_dim"),
            rms_norm_eps=float(get("rms_norm_eps", 1e-6)),
            rope_theta=float(theta if theta is not None else 10000.0),
            rope_scaling=dict(rope) if isinstance(rope, dict) else None,
            max_position_embeddings=int(get("max_position_embeddings", 8192)),
            tie_word_embeddings=bool(get("tie_word_embeddings", False)),
            attention_bias=bool(get("attention_bias", model_type in ("qwen2", "qwen2_moe"))),
            qk_norm=model_type in ("qwen3", "qwen3_moe", "olmo2", "olmo3", "olmoe", "gemma3_text"),
            num_experts=experts,
            experts_per_token=int(get("num_experts_per_tok", 2) or 2),
            model_type=model_type,
            norm_topk_prob=bool(get("norm_topk_prob", True)),
            **extra,
        )

    def to_hf(self) -> Any:
        """A ``transformers`` config of the same architecture (for the HF oracle and the reference benchmark)."""
        import transformers

        common = dict(vocab_size=self.vocab_size, hidden_size=self.hidden_size,
                      intermediate_size=self.intermediate_size, num_hidden_layers=self.num_layers,
                      num_attention_heads=self.num_heads, num_key_value_heads=self.num_kv_heads,
                      head_dim=self.head_dim, rms_norm_eps=self.rms_norm_eps, rope_theta=self.rope_theta,
                      max_position_embeddings=self.max_position_embeddings,
                      tie_word_embeddings=self.tie_word_embeddings, attention_bias=self.attention_bias)
        if self.rope_scaling is not None:
            common["rope_scaling"] = dict(self.rope_scaling)
        kind = self.model_type
        kinds = dict(layer_types=list(self.layer_types), sliding_window=self.sliding_window) if self.layer_types \
            else {}
        if kind in ("gemma", "gemma2", "gemma3_text"):
            gem = dict(hidden_activation="gelu_pytorch_tanh", **common)
            if kind == "gemma":
                return transformers.GemmaConfig(**gem)
            gem.update(query_pre_attn_scalar=round((self.attention_multiplier or self.head_dim ** -0.5) ** -2),
                       **kinds)
            if kind == "gemma2":
                return transformers.Gemma2Config(attn_logit_softcapping=self.attn_softcap,
                                                 final_logit_softcapping=self.final_softcap, **gem)
            full = {"rope_type": "default", "rope_theta": self.rope_theta, **(self.rope_scaling or {})}
            local = {"rope_type": "default", "rope_theta": self.rope_theta, **(self.local_rope or {})}
            gem.pop("rope_theta")
            gem.pop("rope_scaling", None)
            return transformers.Gemma3TextConfig(rope_parameters={FULL: full, SLIDING: local},
                                                 attn_logit_softcapping=self.attn_softcap,
                                                 final_logit_softcapping=self.final_softcap, **gem)
        if kind in ("granitemoe", "granitemoeshared"):
            scales = dict(embedding_multiplier=self.embedding_multiplier, residual_multiplier=self.residual_multiplier,
                          attention_multiplier=self.attention_multiplier or self.head_dim ** -0.5,
                          logits_scaling=self.logits_scaling, num_local_experts=self.num_experts,
                          num_experts_per_tok=self.experts_per_token)
            rest = {k: v for k, v in common.items() if k != "head_dim"}
            if kind == "granitemoe":
                return transformers.GraniteMoeConfig(**scales, **rest)
            return transformers.GraniteMoeSharedConfig(shared_intermediate_size=self.shared_expert_size, **scales,
                                                       **rest)
        if kind == "ministral3":
            rope = {"rope_type": "default", "rope_theta": self.rope_theta, **(self.rope_scaling or {})}
            if self.query_position_scale is not None:
                rope.update(llama_4_scaling_beta=self.query_position_scale[0],
                            original_max_position_embeddings=int(self.query_position_scale[1]))
            rest = {k: v for k, v in common.items() if k not in ("rope_theta", "rope_scaling", "attention_bias")}
            return transformers.Ministral3Config(rope_parameters=rope, sliding_window=self.sliding_window or None,
                                                 **rest)
        if kind == "gpt_oss":
            rope = {"rope_type": "default", "rope_theta": self.rope_theta, **(self.rope_scaling or {})}
            gpt = {k: v for k, v in common.items() if k not in ("rope_theta", "rope_scaling", "attention_bias")}
            return transformers.GptOssConfig(num_local_experts=self.num_experts,
                                             num_experts_per_tok=self.experts_per_token, rope_parameters=rope,
                                             attention_bias=self.attention_bias, **kinds, **gpt)
        if kind == "ministral":
            return transformers.MinistralConfig(**kinds, **{k: v for k, v in common.items() if k != "attention_bias"})
        if kind == "mistral":
            return transformers.MistralConfig(sliding_window=self.sliding_window or None,
                                              **{k: v for k, v in common.items() if k != "attention_bias"})
        if kind == "olmo3":
            return transformers.Olmo3Config(**kinds, **{k: v for k, v in common.items() if k != "head_dim"})
        if kind == "olmoe":
            return transformers.OlmoeConfig(num_experts=self.num_experts, num_experts_per_tok=self.experts_per_token,
                                            norm_topk_prob=self.norm_topk_prob,
                                            **{k: v for k, v in common.items() if k != "head_dim"})
        if kind == "qwen2_moe":
            return transformers.Qwen2MoeConfig(num_experts=self.num_experts, num_experts_per_tok=self.experts_per_token,
                                               moe_intermediate_size=self.intermediate_size,
                                               shared_expert_intermediate_size=self.shared_expert_size,
                                               norm_topk_prob=self.norm_topk_prob,
                                               **{k: v for k, v in common.items() if k not in ("attention_bias",)})
        if kind == "qwen3_moe":
            return transformers.Qwen3MoeConfig(num_experts=self.num_experts, num_experts_per_tok=self.experts_per_token,
                                               moe_intermediate_size=self.intermediate_size,
                                               norm_topk_prob=self.norm_topk_prob, **common)
        if self.is_moe:
            return transformers.MixtralConfig(num_local_experts=self.num_experts,
                                              num_experts_per_tok=self.experts_per_token,
                                              **{k: v for k, v in common.items() if k != "attention_bias"})
        if kind == "granite":
            return transformers.GraniteConfig(embedding_multiplier=self.embedding_multiplier,
                                              residual_multiplier=self.residual_multiplier,
                                              attention_multiplier=self.attention_multiplier or self.head_dim ** -0.5,
                                              logits_scaling=self.logits_scaling, **common)
        if kind == "phi3":
            return transformers.Phi3Config(**{k: v for k, v in common.items() if k not in ("attention_bias",
                                                                                            "head_dim")})
        if kind == "smollm3":
            flags = [0 if i in self.nope_layers else 1 for i in range(self.num_layers)]
            return transformers.SmolLM3Config(no_rope_layers=flags, **common)
        if kind == "olmo2":
            return transformers.Olmo2Config(**{k: v for k, v in common.items() if k != "head_dim"})
        if kind == "qwen3":
            return transformers.Qwen3Config(**common)
        if kind == "qwen2":
            window = dict(use_sliding_window=True, **kinds) if self.layer_types else {}
            return transformers.Qwen2Config(**window, **{k: v for k, v in common.items() if k != "attention_bias"})
        return transformers.LlamaConfig(**common)


def rope_inv_freq(config: ModelConfig, local: bool = False) -> torch.Tensor:
    """Inverse frequencies ``[D/2]`` (fp32) of the rotary embedding, with Llama-3 frequency scaling when
    ``rope_scaling`` says so (the published Llama 3.1 rule: long wavelengths divided by ``factor``, short ones
    kept, a linear blend of the two in between). ``local``: the sliding-window layers' parameters
    (``config.local_rope``)."""
    dim = config.head_dim
    theta, scaling = config.rope_theta, config.rope_scaling or {}
    if local and config.local_rope is not None:
        theta = float(config.local_rope.get("rope_theta", theta))
        scaling = {k: v for k, v in config.local_rope.items() if k != "rope_theta"}
    inv = 1.0 / (theta ** (torch.arange(0, dim, 2, dtype=torch.int64).float() / dim))
    kind = scaling.get("rope_type", scaling.get("type"))
    if kind == "llama3":
        factor = float(scaling["factor"])
        low, high = float(scaling.get("low_freq_factor", 1.0)), float(scaling.get("high_freq_factor", 4.0))
        original = float(scaling.get("original_max_position_embeddings", 8192))
        low_wavelen, high_wavelen = original / low, original / high
        wavelen = 2 * math.pi / inv
        scaled = torch.where(wavelen > low_wavelen, inv / factor, inv)
        smooth = (original / wavelen - low) / (high - low)
        blended = (1 - smooth) * scaled / factor + smooth * scaled
        medium = ~(wavelen < high_wavelen) & ~(wavelen > low_wavelen)
        inv = torch.where(medium, blended, scaled)
    elif kind == "linear":
        inv = inv / float(scaling["factor"])
    elif kind == "yarn":
        inv = _yarn_inv_freq(inv, dim, theta, scaling, config.max_position_embeddings)
    elif kind not in (None, "default"):
        raise UnsupportedModelError(f"rope_scaling type {kind!r} is not supported")
    return inv


def _yarn_inv_freq(inv: torch.Tensor, dim: int, theta: float, scaling: dict[str, Any],
                   max_positions: int) -> torch.Tensor:
    """YaRN's frequency blend (Peng et al., 2023, "YaRN: Efficient Context Window Extension of Large Language
    Models", section 3.2; the form of transformers ``modeling_rope_utils.py``, ``_compute_yarn_parameters``): a
    frequency that turns fewer than ``beta_slow`` times over the original context is interpolated (divided by
    ``factor``), one that turns more than ``beta_fast`` times is kept, and a linear ramp over the dimension index
    blends the two in between. The dimension that turns ``r`` times is ``dim * ln(L / (2 pi r)) / (2 ln theta)``."""
    factor = float(scaling.get("factor") or max_positions / float(scaling["original_max_position_embeddings"]))
    original = float(scaling["original_max_position_embeddings"])
    fast, slow = float(scaling.get("beta_fast") or 32), float(scaling.get("beta_slow") or 1)

    def turning_dim(turns: float) -> float:
        return dim * math.log(original / (turns * 2 * math.pi)) / (2 * math.log(theta))

    low, high = turning_dim(fast), turning_dim(slow)
    if scaling.get("truncate", True):
        low, high = math.floor(low), math.ceil(high)
    low, high = max(low, 0), min(high, dim - 1)
    if low == high:
        high += 0.001
    ramp = ((torch.arange(dim // 2, dtype=torch.float32) - low) / (high - low)).clamp(0, 1)
    keep = 1 - ramp  # 1: extrapolate (the original frequency), 0: interpolate
    return (inv / factor) * (1 - keep) + inv * keep


def rope_attention_factor(config: ModelConfig, local: bool = False) -> float:
    """The factor YaRN applies to cos and sin (``attention_factor``, else ``0.1 ln(factor) + 1``, or its
    ``mscale`` / ``mscale_all_dim`` ratio); 1 for every other rotary kind."""
    scaling = config.rope_scaling or {}
    if local and config.local_rope is not None:
        scaling = config.local_rope
    if scaling.get("rope_type", scaling.get("type")) != "yarn":
        return 1.0
    if scaling.get("attention_factor") is not None:
        return float(scaling["attention_factor"])
    factor = float(scaling.get("factor") or config.max_position_embeddings /
                   float(scaling["original_max_position_embeddings"]))

    def mscale(scale: float, m: float = 1.0) -> float:
        return 1.0 if scale <= 1 else 0.1 * m * math.log(scale) + 1.0

    m, m_all = scaling.get("mscale"), scaling.get("mscale_all_dim")
    if m and m_all:
        return mscale(factor, float(m)) / mscale(factor, float(m_all))
    return mscale(factor)


def gpt_oss_20b(**overrides: Any) -> ModelConfig:
    """gpt-oss-20b architecture (24 layers, hidden 2880, 64/8 heads of 64, 32 experts of width 2880, top-4; 128-token
    windows on the even layers; YaRN x32 over 4096 positions; biases everywhere and sink logits)."""
    layers = int(overrides.pop("num_layers", 24))
    cfg = dict(vocab_size=201088, hidden_size=2880, intermediate_size=2880, num_layers=layers, num_heads=64,
               num_kv_heads=8, head_dim=64, rms_norm_eps=1e-5, rope_theta=150000.0,
               rope_scaling={"rope_type": "yarn", "factor": 32.0, "beta_fast": 32.0, "beta_slow": 1.0,
                             "truncate": False, "original_max_position_embeddings": 4096},
               max_position_embeddings=131072, attention_bias=True, num_experts=32, experts_per_token=4,
               model_type="gpt_oss", hidden_act="clamped_swiglu", o_bias=True, attn_sinks=True, moe_bias=True,
               layer_types=tuple(SLIDING if i % 2 == 0 else FULL for i in range(layers)), sliding_window=128)
    cfg.update(overrides)
    return ModelConfig(**cfg)


def llama31_8b(**overrides: Any) -> ModelConfig:
    """Llama-3.1-8B architecture (32 layers, hidden 4096, 32/8 heads, FFN 14336, vocab 128256)."""
    cfg = dict(vocab_size=128256, hidden_size=4096, intermediate_size=14336, num_layers=32, num_heads=32,
               num_kv_heads=8, head_dim=128, rms_norm_eps=1e-5, rope_theta=500000.0,
               rope_scaling={"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0,
                             "high_freq_factor": 4.0, "original_max_position_embeddings": 8192},
               max_position_embeddings=131072)
    cfg.update(overrides)
    return ModelConfig(**cfg)


def llama31_70b(**overrides: Any) -> ModelConfig:
    """Llama-3.1-70B architecture (80 layers, hidden 8192, 64/8 heads, FFN 28672)."""
    return llama31_8b(**{"hidden_size": 8192, "intermediate_size": 28672, "num_layers": 80, "num_heads": 64,
                         **overrides})


def mixtral_8x7b(**overrides: Any) -> ModelConfig:
    """Mixtral-8x7B architecture (32 layers, hidden 4096, 8 experts top-2, expert FFN 14336)."""
    cfg = dict(vocab_size=32000, hidden_size=4096, intermediate_size=14336, num_layers=32, num_heads=32,
               num_kv_heads=8, head_dim=128, rms_norm_eps=1e-5, rope_theta=1e6, max_position_embeddings=32768,
               num_experts=8, experts_per_token=2, model_type="mixtral")
    cfg.update(overrides)
    return ModelConfig(**cfg)


def tiny_llama(**overrides: Any) -> ModelConfig:
    """The CPU plumbing configuration: 4 layers, hidden 256, 4 heads / 2 KV heads, FFN 688, vocab 1024, θ=1e4."""
    cfg = dict(vocab_size=1024, hidden_size=256, intermediate_size=688, num_layers=4, num_heads=4, num_kv_heads=2,
               rms_norm_eps=1e-6, rope_theta=1e4, max_position_embeddings=2048)
    cfg.update(overrides)
    return ModelConfig(**cfg)
