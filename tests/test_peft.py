"""PEFT interoperability (economize ``tests/integrations/test_peft.py``): a technique's LoRA round-trips through the
PEFT adapter files, and a PEFT adapter merged into the target equals the dense ``W + alpha/r B A`` forward."""

import json

import pytest
import torch

import economize_b200 as eco
from economize_b200.errors import CheckpointFormatError, ConfigError
from economize_b200.integrations.peft import load_lora, lora_modules, merge_adapter, save_lora
from economize_b200.techniques.early_exit import EarlyExitConfig

from .helpers import prompts, reference_greedy, tiny_model


def test_early_exit_lora_roundtrip(tmp_path):
    em = eco.apply(tiny_model(), EarlyExitConfig(exit_layer=2, adaptation="lora", lora_rank=8, lora_alpha=16.0))
    mods = lora_modules(em)
    assert list(mods) == ["lm_head"]
    with torch.no_grad():
        mods["lm_head"].b.normal_(0, 0.01)
    out = save_lora(em, tmp_path / "a", base_model="tiny")
    cfg = json.loads((out / "adapter_config.json").read_text())
    assert cfg["r"] == 8 and cfg["lora_alpha"] == 16.0 and cfg["target_modules"] == ["lm_head"]
    other = eco.apply(tiny_model(), EarlyExitConfig(exit_layer=2, adaptation="lora", lora_rank=8, lora_alpha=16.0))
    load_lora(other, out)
    a, b = lora_modules(other)["lm_head"], mods["lm_head"]
    assert torch.equal(a.a, b.a) and torch.equal(a.b, b.b) and a.scale == b.scale
    dc = eco.DecodeConfig(cycle_length=4)
    p = prompts()
    for x, y in zip(em.decode_batch(p, 12, decoding=dc), other.decode_batch(p, 12, decoding=dc)):
        assert torch.equal(x.tokens, y.tokens) and x.accepted == y.accepted
    wrong = eco.apply(tiny_model(), EarlyExitConfig(exit_layer=2, adaptation="lora", lora_rank=4))
    with pytest.raises(CheckpointFormatError, match="shapes"):
        load_lora(wrong, out)
    with pytest.raises(ConfigError, match="LoRA"):
        lora_modules(eco.apply(tiny_model(), EarlyExitConfig(exit_layer=2)))


def _write_adapter(path, modules, r=4, alpha=8.0, seed=0):
    from safetensors.torch import save_file

    g = torch.Generator().manual_seed(seed)
    tensors = {}
    for name, (out_f, in_f) in modules.items():
        tensors[f"base_model.model.{name}.lora_A.weight"] = torch.randn(r, in_f, generator=g) * 0.05
        tensors[f"base_model.model.{name}.lora_B.weight"] = torch.randn(out_f, r, generator=g) * 0.05
    path.mkdir(parents=True)
    (path / "adapter_config.json").write_text(json.dumps({"peft_type": "LORA", "r": r, "lora_alpha": alpha,
                                                          "target_modules": ["q_proj", "v_proj", "down_proj"]}))
    save_file(tensors, str(path / "adapter_model.safetensors"))
    return tensors


def test_merge_adapter_matches_dense_update(tmp_path):
    model = tiny_model()
    c = model.config
    mods = {"model.layers.0.self_attn.q_proj": (c.q_size, c.hidden_size),
            "model.layers.1.self_attn.v_proj": (c.kv_size, c.hidden_size),
            "model.layers.3.mlp.down_proj": (c.hidden_size, c.intermediate_size)}
    tensors = _write_adapter(tmp_path / "ad", mods)
    before = model.hf_state_dict()
    merged = merge_adapter(model, tmp_path / "ad")
    assert sorted(merged) == sorted(mods)
    after = model.hf_state_dict()
    for name in mods:
        a = tensors[f"base_model.model.{name}.lora_A.weight"]
        b = tensors[f"base_model.model.{name}.lora_B.weight"]
        torch.testing.assert_close(after[name + ".weight"], before[name + ".weight"] + 2.0 * b @ a)
    untouched = "model.layers.0.self_attn.k_proj.weight"
    assert torch.equal(after[untouched], before[untouched])
    p = prompts((17,))[0]
    eff = eco.apply(model, EarlyExitConfig(exit_layer=2))
    assert torch.equal(eff.decode(p, 8, decoding=eco.DecodeConfig(cycle_length=4)).tokens,
                       reference_greedy(model, p, 8))


def test_merge_refuses_unknown_modules(tmp_path):
    _write_adapter(tmp_path / "bad", {"model.layers.0.self_attn.rotary": (4, 4)})
    with pytest.raises(CheckpointFormatError, match="not a decoder projection"):
        merge_adapter(tiny_model(), tmp_path / "bad")
