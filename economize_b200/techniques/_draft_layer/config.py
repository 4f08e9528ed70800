"""Hyperparameters shared by the one-layer draft decoders (fields of economize's ``DraftLayerConfig``,
``src/economize/techniques/_draft_layer/config.py``). ``None`` takes the target model's value."""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any

from ...core.technique import TechniqueConfig
from ...errors import ConfigError
from ...validation import check_choice, check_positive

__all__ = ["DraftLayerConfig", "PARAM_DTYPES"]

#: ``"model"``: the target's dtype (bf16 on the GPU, what the sm_100a kernels run); ``"float32"``: fp32 storage.
PARAM_DTYPES = ("model", "float32", "bfloat16", "float16")


@dataclass(frozen=True)
class DraftLayerConfig(TechniqueConfig):
    intermediate_size: int | None = None
    num_heads: int | None = None
    num_kv_heads: int | None = None
    head_dim: int | None = None
    attention_bias: bool | None = None
    rope_theta: float | None = None
    rope_scaling: dict[str, Any] | None = None
    partial_rotary_factor: float = 1.0
    max_position_embeddings: int | None = None
    rms_norm_eps: float | None = None
    zero_source_first: bool = False
    train_steps: int = 7
    checkpoint_steps: bool = False
    param_dtype: str = "model"

    def __post_init__(self) -> None:
        for name in ("intermediate_size", "num_heads", "num_kv_heads", "head_dim"):
            value = getattr(self, name)
            if value is not None:
                check_positive(name, value)
        if self.num_heads is not None and self.num_kv_heads is not None and self.num_heads % self.num_kv_heads:
            raise ConfigError(f"num_heads {self.num_heads} is not a multiple of num_kv_heads {self.num_kv_heads}")
        if self.partial_rotary_factor != 1.0:
            raise ConfigError("partial rotary tables are not supported by the draft layer kernels")
        if self.rope_scaling is not None and self.rope_theta is None:
            raise ConfigError("rope_scaling shapes the own rotary table: set rope_theta")
        check_positive("train_steps", self.train_steps)
        check_choice("param_dtype", self.param_dtype, PARAM_DTYPES)
