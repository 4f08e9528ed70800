"""Exporters (economize ``tests/backends``): drafter folders for vLLM and SGLang load back into a fresh model with
identical weights and drafts, and the GGUF file of a model decodes to the model's own logits under llama.cpp's
conventions (interleaved RoPE pairs, row-major ``[out, in]`` matrices with reversed dims)."""

import json

import numpy as np
import pytest
import torch

import economize_b200 as eco
from economize_b200.backends import EXPORTERS, UnsupportedBackendError, export_drafter, read_gguf, to_gguf
from economize_b200.errors import ConfigError
from economize_b200.techniques.eagle import EagleConfig
from economize_b200.techniques.eagle3 import Eagle3Config
from economize_b200.techniques.medusa import MedusaConfig

from .helpers import prompts, tiny_model


def test_registry_names():
    assert {"vllm/eagle3", "vllm/eagle", "vllm/medusa", "sglang/eagle3", "sglang/eagle"} <= set(EXPORTERS.names())


@pytest.mark.parametrize("draft_vocab", [None, 512])
def test_eagle3_roundtrip_through_vllm_layout(tmp_path, draft_vocab):
    em = eco.apply(tiny_model(), Eagle3Config(draft_vocab=draft_vocab))
    em.techniques["eagle3"].reset_parameters(seed=3)
    out = export_drafter(em, tmp_path / "d", backend="vllm")
    cfg = json.loads((out / "config.json").read_text())
    assert cfg["architectures"] == ["LlamaForCausalLM"] and cfg["num_hidden_layers"] == 1
    assert cfg["draft_vocab_size"] == (draft_vocab or 1024)
    assert cfg["eagle_aux_hidden_state_layer_ids"] == list(em.techniques["eagle3"].aux_layers)
    from safetensors.torch import load_file

    state = load_file(str(out / "model.safetensors"))
    assert ("d2t" in state) == (draft_vocab is not None)
    assert "midlayer.self_attn.q_proj.weight" in state and not any(k.startswith("embed") for k in state)
    back = eco.load(tiny_model(), out)  # the official EAGLE-3 reader
    a, b = em.techniques["eagle3"], back.techniques["eagle3"]
    for (n, p), (_, q) in zip(a.state_dict().items(), b.state_dict().items()):
        assert torch.equal(p, q), n
    cfg = eco.DecodeConfig(cycle_length=5)
    for x, y in zip(em.decode_batch(prompts(), 16, decoding=cfg), back.decode_batch(prompts(), 16, decoding=cfg)):
        assert torch.equal(x.tokens, y.tokens) and x.accepted == y.accepted


def test_eagle3_speculators_and_sglang(tmp_path):
    em = eco.apply(tiny_model(), Eagle3Config())
    with pytest.raises(ConfigError, match="verifier"):
        export_drafter(em, tmp_path / "s", backend="vllm", format="speculators")
    out = export_drafter(em, tmp_path / "s", backend="vllm", format="speculators", verifier="meta-llama/x")
    cfg = json.loads((out / "config.json").read_text())
    assert cfg["architectures"] == ["Eagle3Speculator"]
    assert cfg["speculators_config"]["verifier"]["name_or_path"] == "meta-llama/x"
    assert cfg["transformer_layer_config"]["num_hidden_layers"] == 1
    sg = json.loads((export_drafter(em, tmp_path / "g", backend="sglang") / "config.json").read_text())
    assert sg["architectures"] == ["LlamaForCausalLMEagle3"]


def test_eagle_and_medusa_layouts(tmp_path):
    from safetensors.torch import load_file

    em = eco.apply(tiny_model(), EagleConfig())
    state = load_file(str(export_drafter(em, tmp_path / "e", backend="vllm") / "model.safetensors"))
    assert state["fc.weight"].shape == (256, 512) and "fc.bias" in state
    assert state["layers.0.self_attn.k_proj.weight"].shape == (2 * 64, 256)
    med = eco.apply(tiny_model(), MedusaConfig(num_heads=3, num_layers=2))
    out = export_drafter(med, tmp_path / "m", backend="vllm")
    cfg = json.loads((out / "config.json").read_text())
    state = load_file(str(out / "model.safetensors"))
    assert cfg["num_heads"] == 3 and cfg["num_hidden_layers"] == 2
    tech = med.techniques["medusa"]
    assert torch.equal(state["blocks.2.layers.1.weight"], tech.heads[2].blocks[1].linear.weight)
    assert torch.equal(state["lm_heads.0.weight"], tech.heads[0].proj.weight)
    shared = eco.apply(tiny_model(), MedusaConfig(head="shared"))
    with pytest.raises(ConfigError, match="head='own'"):
        export_drafter(shared, tmp_path / "x", backend="vllm")
    with pytest.raises(UnsupportedBackendError):
        export_drafter(med, tmp_path / "y", backend="sglang")


def _rms(x, w, eps):
    return x / np.sqrt((x * x).mean(-1, keepdims=True) + eps) * w


def _gguf_forward(meta, t, tokens):
    """A plain numpy Llama forward over GGUF tensors with llama.cpp's interleaved RoPE (pairs ``2j, 2j + 1``)."""
    heads, kv = meta["llama.attention.head_count"], meta["llama.attention.head_count_kv"]
    eps, base, hd = meta["llama.attention.layer_norm_rms_epsilon"], meta["llama.rope.freq_base"], \
        meta["llama.rope.dimension_count"]
    g = {k: v.double().numpy() for k, v in t.items()}
    x = g["token_embd.weight"][tokens]
    n = len(tokens)
    theta = base ** (-np.arange(0, hd, 2) / hd)
    ang = np.arange(n)[:, None] * theta[None]
    cos, sin = np.cos(ang)[:, None], np.sin(ang)[:, None]

    def rope(v):
        a, b = v[..., 0::2], v[..., 1::2]
        out = np.empty_like(v)
        out[..., 0::2] = a * cos - b * sin
        out[..., 1::2] = a * sin + b * cos
        return out

    for i in range(meta["llama.block_count"]):
        p = f"blk.{i}."
        h = _rms(x, g[p + "attn_norm.weight"], eps)
        q = rope((h @ g[p + "attn_q.weight"].T).reshape(n, heads, hd))
        k = rope((h @ g[p + "attn_k.weight"].T).reshape(n, kv, hd))
        v = (h @ g[p + "attn_v.weight"].T).reshape(n, kv, hd)
        k, v = np.repeat(k, heads // kv, 1), np.repeat(v, heads // kv, 1)
        s = np.einsum("qhd,khd->hqk", q, k) / np.sqrt(hd) + np.triu(np.full((n, n), -np.inf), 1)
        s = np.exp(s - s.max(-1, keepdims=True))
        s /= s.sum(-1, keepdims=True)
        x = x + np.einsum("hqk,khd->qhd", s, v).reshape(n, heads * hd) @ g[p + "attn_output.weight"].T
        h = _rms(x, g[p + "ffn_norm.weight"], eps)
        gate = h @ g[p + "ffn_gate.weight"].T
        x = x + (gate / (1 + np.exp(-gate)) * (h @ g[p + "ffn_up.weight"].T)) @ g[p + "ffn_down.weight"].T
    return _rms(x, g["output_norm.weight"], eps) @ g["output.weight"].T


def test_gguf_decodes_to_the_models_logits(tmp_path):
    model = tiny_model()
    path = to_gguf(model, tmp_path / "m.gguf", dtype="F32", tokens=[f"t{i}" for i in range(1024)], eos_token_id=2)
    meta, t, types = read_gguf(path)
    assert meta["general.architecture"] == "llama" and meta["llama.block_count"] == 4
    assert meta["tokenizer.ggml.tokens"][5] == "t5" and meta["tokenizer.ggml.eos_token_id"] == 2
    assert len(t) == 3 + 9 * 4 and set(types.values()) == {"F32"}
    tokens = prompts()[0].numpy()
    from economize_b200.runtime.cache import StepBatch

    n = len(tokens)
    h, _ = model.forward_step(torch.from_numpy(tokens)[None], StepBatch.prefill(torch.tensor([n], dtype=torch.int32),
                                                                                 n), model.new_cache(1, 128))
    ref = model.logits(h[0]).detach().double().numpy()
    assert np.abs(_gguf_forward(meta, t, tokens) - ref).max() < 1e-4


def test_gguf_encodings(tmp_path):
    model = tiny_model()
    hf = model.hf_state_dict()
    _, f16, ty16 = read_gguf(to_gguf(model, tmp_path / "a.gguf", dtype="F16"))
    _, bf16, _ = read_gguf(to_gguf(model, tmp_path / "b.gguf", dtype="BF16"))
    _, q8, tyq = read_gguf(to_gguf(model, tmp_path / "c.gguf", dtype="Q8_0"))
    w = hf["model.layers.0.mlp.gate_proj.weight"]
    assert ty16["blk.0.ffn_gate.weight"] == "F16" and ty16["blk.0.attn_norm.weight"] == "F32"
    assert torch.equal(f16["blk.0.ffn_gate.weight"], w.half().float())
    assert torch.equal(bf16["blk.0.ffn_gate.weight"], w.bfloat16().float())
    assert tyq["blk.0.ffn_gate.weight"] == "Q8_0" and tyq["blk.0.ffn_down.weight"] == "F16"  # 688 columns
    blocks = w.reshape(-1, 32)
    d = blocks.abs().amax(1, keepdim=True) / 127
    bound = d * (0.5 + 127 * 2.0 ** -11)  # half a step, plus the fp16 rounding of the block scale
    assert ((q8["blk.0.ffn_gate.weight"].reshape(-1, 32) - blocks).abs() <= bound).all()
    with pytest.raises(ConfigError, match="dtype"):
        to_gguf(model, tmp_path / "d.gguf", dtype="Q4_K")
