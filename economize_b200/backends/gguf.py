"""GGUF export of the target model for llama.cpp-style runtimes (economize ``backends/gguf/writer.py``).

:func:`to_gguf` writes a Llama-block model (with any weight transform folded in: quantized, pruned or rotated
weights are dequantized first) as one GGUF v3 file: the header, the ``llama.*`` metadata, one tensor record per
weight and the tensor data, each aligned to ``general.alignment`` (32 bytes). Tensor names and metadata keys are
the ones llama.cpp reads for the ``llama`` architecture (``token_embd``, ``blk.{i}.attn_q`` ..., ``output``), and
the query and key projections are reordered from the rotate-half RoPE layout of Hugging Face checkpoints to the
interleaved pairs llama.cpp rotates. Types: ``F32``, ``F16``, ``BF16``, and ``Q8_0`` (blocks of 32 values, one fp16
scale ``max|x| / 127`` and 32 int8 codes); 1-D tensors (norms) always stay ``F32``.

A tokenizer is not part of this package's models: pass ``tokens`` (and optionally ``scores``, ``token_types``,
``tokenizer_model``, ``bos``/``eos`` ids) to include the ``tokenizer.ggml.*`` metadata a runtime needs to run the
file. :func:`read_gguf` parses a file back into metadata and float32 tensors (Q8_0 decoded), for checks.
"""

from __future__ import annotations

import struct
from pathlib import Path
from typing import Any, BinaryIO

import numpy as np
import torch

from ..errors import ConfigError

__all__ = ["GGUF_TYPES", "read_gguf", "to_gguf"]

_MAGIC = b"GGUF"
_VERSION = 3
_ALIGN = 32
#: ggml tensor type ids of the supported encodings.
GGUF_TYPES = {"F32": 0, "F16": 1, "Q8_0": 8, "BF16": 30}
_Q8_BLOCK = 32
# GGUF metadata value types
_U8, _I8, _U16, _I16, _U32, _I32, _F32, _BOOL, _STR, _ARR, _U64, _I64, _F64 = range(13)
_SCALAR = {_U8: "<B", _I8: "<b", _U16: "<H", _I16: "<h", _U32: "<I", _I32: "<i", _F32: "<f", _BOOL: "<?",
           _U64: "<Q", _I64: "<q", _F64: "<d"}
# ggml file_type of an all-F32 / mostly-F16 / mostly-Q8_0 / mostly-BF16 model
_FILE_TYPE = {"F32": 0, "F16": 1, "Q8_0": 7, "BF16": 32}


def _put_string(f: BinaryIO, s: str) -> None:
    raw = s.encode("utf-8")
    f.write(struct.pack("<Q", len(raw)))
    f.write(raw)


def _value_type(v: Any) -> int:
    if isinstance(v, bool):
        return _BOOL
    if isinstance(v, int):
        return _U32 if 0 <= v < 2 ** 32 else _I64
    if isinstance(v, float):
        return _F32
    if isinstance(v, str):
        return _STR
    if isinstance(v, (list, tuple)):
        return _ARR
    raise ConfigError(f"GGUF metadata cannot hold a {type(v).__name__}")


def _put_value(f: BinaryIO, v: Any, kind: int) -> None:
    if kind == _STR:
        _put_string(f, v)
    elif kind == _ARR:
        inner = _value_type(v[0]) if len(v) else _U32
        if inner == _U32 and any(isinstance(x, int) and not 0 <= x < 2 ** 32 for x in v):
            inner = _I64
        f.write(struct.pack("<IQ", inner, len(v)))
        for x in v:
            _put_value(f, x, inner)
    else:
        f.write(struct.pack(_SCALAR[kind], v))


def _interleave_rope(w: torch.Tensor, heads: int) -> torch.Tensor:
    """Rows of a q/k projection reordered from rotate-half halves to interleaved pairs, per head."""
    rows, cols = w.shape
    return w.reshape(heads, 2, rows // heads // 2, cols).transpose(1, 2).reshape(rows, cols)


def _q8_0(x: np.ndarray) -> bytes:
    """Q8_0 blocks of a float32 array whose size is a multiple of 32."""
    blocks = x.reshape(-1, _Q8_BLOCK)
    amax = np.abs(blocks).max(1, keepdims=True)
    d = (amax / 127.0).astype(np.float32)
    safe = np.where(d == 0, 1.0, d)
    q = np.clip(np.rint(blocks / safe), -127, 127).astype(np.int8)
    out = np.empty(len(blocks), dtype=[("d", "<f2"), ("q", "i1", (_Q8_BLOCK,))])
    out["d"] = d[:, 0].astype(np.float16)
    out["q"] = q
    return out.tobytes()


def _encode(t: torch.Tensor, kind: str) -> bytes:
    t = t.detach().to("cpu")
    if kind == "F32":
        return t.float().contiguous().numpy().tobytes()
    if kind == "F16":
        return t.half().contiguous().numpy().tobytes()
    if kind == "BF16":
        return t.bfloat16().contiguous().view(torch.int16).numpy().tobytes()
    return _q8_0(t.float().contiguous().numpy().reshape(-1))


def _tensors(model) -> dict[str, torch.Tensor]:
    """The model's weights under GGUF ``llama`` names (q/k rows interleaved for llama.cpp's RoPE)."""
    c = model.config
    if c.model_type not in ("llama", "mistral", "qwen2") or c.num_experts:
        raise ConfigError(f"the GGUF exporter writes dense Llama-block models, not {c.model_type!r}"
                          + (" with experts" if c.num_experts else ""))
    if c.qk_norm:
        raise ConfigError("the GGUF exporter does not write QK-norm models")
    hf = model.hf_state_dict()
    out = {"token_embd.weight": hf["model.embed_tokens.weight"], "output_norm.weight": hf["model.norm.weight"]}
    if "lm_head.weight" in hf and not c.tie_word_embeddings:
        out["output.weight"] = hf["lm_head.weight"]
    names = {"input_layernorm": "attn_norm", "post_attention_layernorm": "ffn_norm", "self_attn.q_proj": "attn_q",
             "self_attn.k_proj": "attn_k", "self_attn.v_proj": "attn_v", "self_attn.o_proj": "attn_output",
             "mlp.gate_proj": "ffn_gate", "mlp.up_proj": "ffn_up", "mlp.down_proj": "ffn_down"}
    for i in range(c.num_layers):
        for src, dst in names.items():
            for kind in ("weight", "bias"):
                key = f"model.layers.{i}.{src}.{kind}"
                if key not in hf:
                    continue
                t = hf[key]
                if src in ("self_attn.q_proj", "self_attn.k_proj"):
                    heads = c.num_heads if src.endswith("q_proj") else c.num_kv_heads
                    t = _interleave_rope(t if t.dim() == 2 else t[:, None], heads)
                    t = t if kind == "weight" else t[:, 0]
                out[f"blk.{i}.{dst}.{kind}"] = t
    return out


def to_gguf(model, path: str | Path, *, dtype: str = "F16", name: str = "economize_b200 export",
            tokens: list[str] | None = None, scores: list[float] | None = None,
            token_types: list[int] | None = None, tokenizer_model: str = "gpt2", bos_token_id: int | None = None,
            eos_token_id: int | None = None) -> Path:
    """Write ``model`` (an EfficientModel or a CausalLM) as a GGUF file with weight matrices in ``dtype``."""
    if dtype not in GGUF_TYPES:
        raise ConfigError(f"GGUF dtype must be one of {sorted(GGUF_TYPES)}, got {dtype!r}")
    model = getattr(model, "model", model)
    c = model.config
    tensors = _tensors(model)
    head_dim = c.head_dim or c.hidden_size // c.num_heads
    meta: dict[str, Any] = {
        "general.architecture": "llama", "general.name": name, "general.alignment": _ALIGN,
        "general.file_type": _FILE_TYPE[dtype],
        "llama.context_length": int(c.max_position_embeddings), "llama.embedding_length": int(c.hidden_size),
        "llama.block_count": int(c.num_layers), "llama.feed_forward_length": int(c.intermediate_size),
        "llama.attention.head_count": int(c.num_heads), "llama.attention.head_count_kv": int(c.num_kv_heads),
        "llama.attention.key_length": int(head_dim), "llama.attention.value_length": int(head_dim),
        "llama.rope.dimension_count": int(head_dim), "llama.rope.freq_base": float(c.rope_theta),
        "llama.attention.layer_norm_rms_epsilon": float(c.rms_norm_eps), "llama.vocab_size": int(c.vocab_size),
    }
    scaling = c.rope_scaling or {}
    if scaling.get("rope_type", scaling.get("type")) == "linear":
        meta["llama.rope.scaling.type"] = "linear"
        meta["llama.rope.scaling.factor"] = float(scaling["factor"])
    if tokens is not None:
        if len(tokens) != c.vocab_size:
            raise ConfigError(f"tokens has {len(tokens)} entries; the model's vocabulary has {c.vocab_size}")
        meta["tokenizer.ggml.model"] = tokenizer_model
        meta["tokenizer.ggml.tokens"] = list(tokens)
        if scores is not None:
            meta["tokenizer.ggml.scores"] = [float(s) for s in scores]
        if token_types is not None:
            meta["tokenizer.ggml.token_type"] = [int(t) for t in token_types]
        if bos_token_id is not None:
            meta["tokenizer.ggml.bos_token_id"] = int(bos_token_id)
        if eos_token_id is not None:
            meta["tokenizer.ggml.eos_token_id"] = int(eos_token_id)
    records = []
    offset = 0
    for tname, t in tensors.items():
        kind = "F32" if t.dim() == 1 else dtype
        if kind == "Q8_0" and t.shape[-1] % _Q8_BLOCK:
            kind = "F16"  # rows that do not split into 32-value blocks
        data = _encode(t, kind)
        records.append((tname, tuple(reversed(t.shape)), GGUF_TYPES[kind], offset, data))
        offset += (len(data) + _ALIGN - 1) // _ALIGN * _ALIGN
    out = Path(path)
    out.parent.mkdir(parents=True, exist_ok=True)
    with open(out, "wb") as f:
        f.write(_MAGIC)
        f.write(struct.pack("<IQQ", _VERSION, len(records), len(meta)))
        for key, value in meta.items():
            _put_string(f, key)
            kind = _value_type(value)
            f.write(struct.pack("<I", kind))
            _put_value(f, value, kind)
        for tname, dims, kind, off, _ in records:
            _put_string(f, tname)
            f.write(struct.pack("<I", len(dims)))
            f.write(struct.pack(f"<{len(dims)}Q", *dims))
            f.write(struct.pack("<IQ", kind, off))
        f.write(b"\0" * (-f.tell() % _ALIGN))
        start = f.tell()
        for _, _, _, off, data in records:
            f.write(b"\0" * (start + off - f.tell()))
            f.write(data)
    return out


# ---- reading ----------------------------------------------------------------------------------------------------
def _get(f: BinaryIO, fmt: str):
    size = struct.calcsize(fmt)
    return struct.unpack(fmt, f.read(size))[0]


def _get_string(f: BinaryIO) -> str:
    return f.read(_get(f, "<Q")).decode("utf-8")


def _get_value(f: BinaryIO, kind: int):
    if kind == _STR:
        return _get_string(f)
    if kind == _ARR:
        inner, n = _get(f, "<I"), _get(f, "<Q")
        return [_get_value(f, inner) for _ in range(n)]
    return _get(f, _SCALAR[kind])


def read_gguf(path: str | Path) -> tuple[dict[str, Any], dict[str, torch.Tensor], dict[str, str]]:
    """``(metadata, tensors, types)`` of a GGUF file: tensors as float32 in their PyTorch shape (Q8_0 decoded)."""
    names = {v: k for k, v in GGUF_TYPES.items()}
    with open(path, "rb") as f:
        if f.read(4) != _MAGIC:
            raise ConfigError(f"{path} is not a GGUF file")
        version, n_tensors, n_meta = struct.unpack("<IQQ", f.read(20))
        if version != _VERSION:
            raise ConfigError(f"GGUF version {version} is not supported")
        meta = {}
        for _ in range(n_meta):
            key = _get_string(f)
            meta[key] = _get_value(f, _get(f, "<I"))
        infos = []
        for _ in range(n_tensors):
            tname = _get_string(f)
            n_dims = _get(f, "<I")
            dims = struct.unpack(f"<{n_dims}Q", f.read(8 * n_dims))
            kind, off = struct.unpack("<IQ", f.read(12))
            infos.append((tname, tuple(reversed(dims)), kind, off))
        align = int(meta.get("general.alignment", _ALIGN))
        start = f.tell() + (-f.tell() % align)
        tensors, types = {}, {}
        for tname, shape, kind, off in infos:
            if kind not in names:
                raise ConfigError(f"tensor {tname} has ggml type {kind}, which this reader does not decode")
            count = int(np.prod(shape))
            f.seek(start + off)
            if names[kind] == "F32":
                arr = np.frombuffer(f.read(4 * count), "<f4").astype(np.float32)
            elif names[kind] == "F16":
                arr = np.frombuffer(f.read(2 * count), "<f2").astype(np.float32)
            elif names[kind] == "BF16":
                raw = np.frombuffer(f.read(2 * count), "<u2").astype(np.uint32) << 16
                arr = raw.view(np.float32)
            else:
                blocks = np.frombuffer(f.read(count // _Q8_BLOCK * 34),
                                       dtype=[("d", "<f2"), ("q", "i1", (_Q8_BLOCK,))])
                arr = (blocks["d"].astype(np.float32)[:, None] * blocks["q"].astype(np.float32)).reshape(-1)
            tensors[tname] = torch.from_numpy(arr.copy()).reshape(shape)
            types[tname] = names[kind]
    return meta, tensors, types
