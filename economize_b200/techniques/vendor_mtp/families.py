"""Where model families keep their multi-token-prediction (MTP) modules, and how each module mixes its inputs.

Reference parity: economize ``techniques/vendor_mtp/families.py`` (``MTPLayout``, ``MTPFamily``, ``MTP_FAMILIES``).
The vendor tensor names and the three layout conventions are the checkpoints' own (DeepSeek-V3, GLM-4.5, MiMo,
Qwen3-Next / Qwen3.5 as vLLM loads them), so they have to be the same strings; the classes around them are this
package's.

A module ``i`` of a checkpoint lives below one prefix (``model.layers.{num_layers + i}.`` for DeepSeek-V3 and
GLM-4.5, ``model.mtp_layers.{i}.`` for MiMo, ``mtp.layers.{i}.`` for the Qwen families). Below it sit the module's
decoder block (vendor layer names: ``self_attn.q_proj.weight`` ...) and, except for the Qwen families, the module's
own parameters; the Qwen families keep those once below ``mtp.`` for all modules.
"""

from __future__ import annotations

import re
from collections.abc import Mapping
from dataclasses import dataclass, field
from types import MappingProxyType

from ...errors import ConfigError
from ...registry import Registry

__all__ = ["DEFAULT_FAMILY", "MTP_FAMILIES", "MTPFamily", "MTPLayout", "family_for"]

CONCAT_ORDERS = ("emb_hidden", "hidden_emb")
RECYCLE = ("raw", "normed")


@dataclass(frozen=True)
class MTPLayout:
    """How a module combines its inputs.

    Attributes:
        concat_order: ``"emb_hidden"``: ``proj([enorm(embed(x)); hnorm(h)])``; ``"hidden_emb"``: the state first
            (MiMo).
        zero_first_embedding: The embedding of the token at position 0 enters as zeros.
        recycle: The state a later draft step reads: the block output (``"raw"``) or the module's normed output
            (``"normed"``).
    """

    concat_order: str = "emb_hidden"
    zero_first_embedding: bool = True
    recycle: str = "raw"

    def __post_init__(self) -> None:
        if self.concat_order not in CONCAT_ORDERS:
            raise ConfigError(f"concat_order must be one of {CONCAT_ORDERS}, got {self.concat_order!r}")
        if self.recycle not in RECYCLE:
            raise ConfigError(f"recycle must be one of {RECYCLE}, got {self.recycle!r}")


#: this technique's names of a module's own parameters -> DeepSeek-V3's vendor names
_DEEPSEEK = MappingProxyType({"enorm": "enorm", "hnorm": "hnorm", "fc": "eh_proj", "norm": "shared_head.norm"})
_QWEN = MappingProxyType({"enorm": "pre_fc_norm_embedding", "hnorm": "pre_fc_norm_hidden", "fc": "fc",
                          "norm": "norm"})
_MIMO = MappingProxyType({"enorm": "token_layernorm", "hnorm": "hidden_layernorm", "fc": "input_proj",
                          "norm": "final_layernorm"})


@dataclass(frozen=True)
class MTPFamily:
    """One family's MTP modules in its checkpoints.

    Attributes:
        layout: The family's input order, position-0 rule and recycled state.
        model_types: ``model_type`` values of the family's ``config.json``.
        own_names: This technique's name -> the vendor's name of each module parameter outside the block.
        prefix: Prefix template of module ``{index}``.
        after_model: ``{index}`` counts on from the model's decoder layers (``num_layers + i``).
        shared_prefix: Prefix of module parameters kept once for every module (``None``: per module).
        skipped: Leaves below a module prefix that repeat the model's own weights (embedding, LM head).
    """

    layout: MTPLayout
    model_types: tuple[str, ...] = ()
    own_names: Mapping[str, str] = field(default_factory=lambda: _DEEPSEEK)
    prefix: str = "model.layers.{index}."
    after_model: bool = True
    shared_prefix: str | None = None
    skipped: tuple[str, ...] = ("shared_head.head.", "embed_tokens.")

    def module_prefix(self, index: int, num_layers: int) -> str:
        return self.prefix.format(index=index + (num_layers if self.after_model else 0))

    def locate(self, key: str, num_layers: int) -> tuple[int, str] | None:
        """``(module, leaf below its prefix)`` of a module tensor; ``None`` for any other key."""
        head, tail = self.prefix.split("{index}", 1)
        m = re.fullmatch(re.escape(head) + r"(\d+)" + re.escape(tail) + r"(.+)", key)
        if m is None:
            return None
        index = int(m.group(1)) - (num_layers if self.after_model else 0)
        return (index, m.group(2)) if index >= 0 else None

    def shared_leaf(self, key: str) -> str | None:
        """The leaf below :attr:`shared_prefix` of a shared module parameter; ``None`` for any other key."""
        if self.shared_prefix is None or not key.startswith(self.shared_prefix):
            return None
        leaf = key[len(self.shared_prefix):]
        return leaf if any(leaf.startswith(v + ".") for v in self.own_names.values()) else None

    def owns(self, key: str, num_layers: int) -> bool:
        return self.locate(key, num_layers) is not None or self.shared_leaf(key) is not None


MTP_FAMILIES: Registry[MTPFamily] = Registry("MTP family", "economize_b200.mtp_families")
MTP_FAMILIES.register("deepseek_v3", MTPFamily(MTPLayout("emb_hidden", True, "raw"), ("deepseek_v3", "kimi_k2")))
MTP_FAMILIES.register("glm4_moe", MTPFamily(MTPLayout("emb_hidden", True, "raw"), ("glm4_moe",)))
MTP_FAMILIES.register("mimo", MTPFamily(MTPLayout("hidden_emb", True, "normed"), ("mimo",), _MIMO,
                                        "model.mtp_layers.{index}.", after_model=False))
MTP_FAMILIES.register("qwen3_next", MTPFamily(MTPLayout("emb_hidden", False, "normed"), ("qwen3_next",), _QWEN,
                                              "mtp.layers.{index}.", after_model=False, shared_prefix="mtp."))
MTP_FAMILIES.register("qwen3_5", MTPFamily(MTPLayout("emb_hidden", False, "normed"),
                                           ("qwen3_5", "qwen3_5_text", "qwen3_5_moe", "qwen3_5_moe_text"), _QWEN,
                                           "mtp.layers.{index}.", after_model=False, shared_prefix="mtp."))

#: the layout of new modules on a model whose family ships none (DeepSeek-V3's, the published one)
DEFAULT_FAMILY = "deepseek_v3"


def family_for(model_type: str) -> str | None:
    """The registered family whose models have ``model_type`` (``None``: none lists it)."""
    for name in MTP_FAMILIES.names():
        if model_type in MTP_FAMILIES.get(name).model_types:
            return name
    return None
