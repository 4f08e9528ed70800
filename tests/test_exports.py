"""MLX and TensorRT-LLM checkpoint writers: the tensors, read back with independent unpackers, give the model's
weights (dequantized codes equal the engine's), and the configs name the architecture."""

import json

import numpy as np
import pytest
import torch
from safetensors.torch import load_file

import economize_b200 as eco
from economize_b200.backends.mlx import to_mlx
from economize_b200.backends.trtllm import to_trtllm
from economize_b200.techniques.quant.config import QuantConfig

from .helpers import tiny_model


def _mlx_unpack(words: torch.Tensor, bits: int, count: int) -> np.ndarray:
    w = words.view(torch.int32).numpy().view(np.uint32).astype(np.uint64)
    out = np.zeros((w.shape[0], count), dtype=np.int64)
    for j in range(count):
        bit = j * bits
        word, off = bit // 32, bit % 32
        val = w[:, word] >> np.uint64(off)
        if off + bits > 32:
            val |= w[:, word + 1] << np.uint64(32 - off)
        out[:, j] = (val & np.uint64((1 << bits) - 1)).astype(np.int64)
    return out


def test_mlx_folder_holds_the_dequantized_weights(tmp_path):
    for fmt, sym in (("int4", False), ("int8", True), ("int3", False)):
        model = tiny_model()
        em = eco.apply(model, QuantConfig(format=fmt, group_size=64, symmetric=sym))
        to_mlx(em, tmp_path / fmt, dtype=torch.float32)
        state = load_file(str(tmp_path / fmt / "model.safetensors"))
        cfg = json.loads((tmp_path / fmt / "config.json").read_text())
        bits = {"int4": 4, "int8": 8, "int3": 3}[fmt]
        assert cfg["quantization"] == {"group_size": 64, "bits": bits}
        c = model.config
        layer = model.layers[1]
        want = layer.wqkv.dequantize(torch.float32)[c.q_size:c.q_size + c.kv_size]  # k_proj rows
        key = "model.layers.1.self_attn.k_proj"
        codes = _mlx_unpack(state[key + ".weight"], bits, c.hidden_size)
        got = torch.from_numpy(codes).float() * state[key + ".scales"].repeat_interleave(64, 1) + \
            state[key + ".biases"].repeat_interleave(64, 1)
        torch.testing.assert_close(got, want, atol=1e-3, rtol=1e-3)


def test_trtllm_checkpoint_names_shards_and_awq_codes(tmp_path):
    model = tiny_model()
    em = eco.apply(model, QuantConfig(format="int4", group_size=64, symmetric=True))
    to_trtllm(em, tmp_path, tp=2, dtype=torch.float32)
    cfg = json.loads((tmp_path / "config.json").read_text())
    assert cfg["architecture"] == "LlamaForCausalLM" and cfg["mapping"]["tp_size"] == 2
    assert cfg["quantization"]["quant_algo"] == "W4A16_AWQ" and cfg["quantization"]["group_size"] == 64
    c = model.config
    ranks = [load_file(str(tmp_path / f"rank{r}.safetensors")) for r in range(2)]
    p = "transformer.layers.0."
    dense = model.layers[0].wo.dequantize(torch.float32)  # row-parallel: columns split over the ranks
    for r, state in enumerate(ranks):
        packed = state[p + "attention.dense.weight"].view(torch.uint8).to(torch.int16)
        lo, hi = packed & 0xF, packed >> 4
        signed = torch.stack([lo, hi], 1).reshape(-1, packed.shape[1])
        signed = torch.where(signed >= 8, signed - 16, signed).float()
        scales = state[p + "attention.dense.weights_scaling_factor"].t().repeat_interleave(64, 1)
        k = dense.shape[1] // 2
        torch.testing.assert_close(signed * scales, dense[:, r * k:(r + 1) * k], atol=1e-3, rtol=1e-3)
        assert state[p + "attention.qkv.weight"].shape[0] == (c.q_size + 2 * c.kv_size) // 2 // 2  # rows / 2 / tp
        assert state[p + "mlp.proj.weight"].shape == (c.hidden_size, c.intermediate_size // 2)  # dense (K 688)


def test_exports_refuse_an_online_rotation(tmp_path):
    import economize_b200 as eco
    from economize_b200.backends.mlx import to_mlx
    from economize_b200.backends.trtllm import to_trtllm
    from economize_b200.integrations.compressed_tensors import export_compressed_tensors
    from economize_b200.techniques.rotate import RotateConfig

    from .helpers import tiny_model

    em = eco.apply(tiny_model(), RotateConfig())
    for write in (to_mlx, to_trtllm, export_compressed_tensors):
        with pytest.raises(eco.ConfigError, match="online Hadamard"):
            write(em, tmp_path / write.__name__)
