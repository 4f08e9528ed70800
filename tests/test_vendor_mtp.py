"""vendor_mtp: the family layouts draft losslessly, module states round-trip through every family's checkpoint names,
model directories that ship MTP modules load through read_checkpoint / attach, FP8 block weights dequantize, and
blocks this engine's draft layer cannot hold are refused."""

import json

import pytest
import torch

import economize_b200 as eco
from economize_b200.errors import CheckpointFormatError, ConfigError
from economize_b200.techniques.vendor_mtp import VendorMTPConfig, state_from_vendor
from economize_b200.techniques.vendor_mtp.formats import dequantize_fp8_blocks
from economize_b200.train import fit

from .helpers import prompts, reference_greedy, tiny_model


def _randomize(tech, seed=3):
    g = torch.Generator().manual_seed(seed)
    with torch.no_grad():
        for p in tech.parameters():
            if p is not tech.model.embed and not any(p is q for q in tech.model.parameters()):
                p.copy_(torch.randn(p.shape, generator=g) * 0.05 + (1.0 if p.dim() == 1 else 0.0))


@pytest.mark.parametrize("cfg", [
    dict(),                                                        # DeepSeek-V3 layout, normed target state
    dict(family="mimo", attention_bias=True),                      # [h; e], recycled after the norm
    dict(family="qwen3_next"),                                     # no position-0 zeroing, normed recycling
    dict(concat_order="hidden_emb", zero_first_embedding=False, recycle="normed", target_state="raw"),
])
def test_layouts_draft_losslessly(cfg):
    model = tiny_model()
    eff = eco.apply(model, VendorMTPConfig(**cfg))
    _randomize(eff.techniques["vendor_mtp"])
    p = prompts((19,))[0]
    want = reference_greedy(model, p, 10)
    assert torch.equal(eff.decode(p, 10).tokens, want)
    tree = eco.DecodeConfig(cycle_length=4, draft_policy="dynamic_tree",
                            draft_policy_options={"depth": 3, "topk": 3, "total_tokens": 8})
    assert torch.equal(eff.decode(p, 10, decoding=tree).tokens, want)


def test_layout_resolution_and_checks():
    model = tiny_model()
    tech = eco.apply(model, VendorMTPConfig()).techniques["vendor_mtp"]
    assert tech.family == "deepseek_v3" and tech.layout.recycle == "raw" and tech.layout.zero_first_embedding
    assert VendorMTPConfig(family="mimo").layout("llama").concat_order == "hidden_emb"
    with pytest.raises(ConfigError):
        VendorMTPConfig(family="nope")
    with pytest.raises(ConfigError):
        VendorMTPConfig(num_modules=2)
    with pytest.raises(ConfigError):
        VendorMTPConfig(recycle="both")


@pytest.mark.parametrize("family", ["deepseek_v3", "glm4_moe", "mimo", "qwen3_next"])
def test_vendor_names_round_trip(family):
    model = tiny_model()
    eff = eco.apply(model, VendorMTPConfig(family=family, attention_bias=family == "mimo"))
    tech = eff.techniques["vendor_mtp"]
    _randomize(tech)
    vendor = tech.vendor_state()
    n = model.config.num_layers
    if family in ("deepseek_v3", "glm4_moe"):
        assert f"model.layers.{n}.eh_proj.weight" in vendor and f"model.layers.{n}.shared_head.norm.weight" in vendor
    elif family == "mimo":
        assert "model.mtp_layers.0.input_proj.weight" in vendor and "model.mtp_layers.0.self_attn.q_proj.bias" in vendor
    else:
        assert "mtp.fc.weight" in vendor and "mtp.layers.0.self_attn.q_proj.weight" in vendor
    back = state_from_vendor(vendor, family, n)
    assert len(back) == 1
    ours = tech.export_state()
    assert back[0].keys() == ours.keys()
    assert all(torch.equal(back[0][k], ours[k]) for k in ours)


def test_model_directory_loads_and_attaches(tmp_path):
    safetensors = pytest.importorskip("safetensors.torch")
    model = tiny_model()
    n = model.config.num_layers
    tech = eco.apply(model, VendorMTPConfig()).techniques["vendor_mtp"]
    _randomize(tech, seed=7)
    tensors = {k: v.contiguous() for k, v in tech.vendor_state().items()}
    tensors.update({f"model.layers.{n}.embed_tokens.weight": model.embed.detach().clone(),  # copies, not read
                    f"model.layers.{n}.shared_head.head.weight": model.head_weight.detach().clone(),
                    "model.layers.0.self_attn.q_proj.weight": torch.zeros(4, 4)})             # main model: ignored
    safetensors.save_file(tensors, str(tmp_path / "model.safetensors"))
    (tmp_path / "config.json").write_text(json.dumps({"model_type": "deepseek_v3", "num_hidden_layers": n,
                                                      "num_nextn_predict_layers": 1}))
    ck = eco.read_checkpoint(tmp_path)
    assert ck.configs[0].family == "deepseek_v3"
    eff = eco.attach(tiny_model(), ck)
    got = eff.techniques["vendor_mtp"].export_state()
    want = tech.export_state()
    assert all(torch.equal(got[k], want[k]) for k in want)
    p = prompts((13,))[0]
    assert torch.equal(eff.decode(p, 8).tokens, reference_greedy(eff.model, p, 8))


def test_unsupported_blocks_are_refused():
    model = tiny_model()
    tech = eco.apply(model, VendorMTPConfig()).techniques["vendor_mtp"]
    vendor = tech.vendor_state()
    n = model.config.num_layers
    vendor[f"model.layers.{n}.mlp.experts.0.gate_proj.weight"] = torch.zeros(8, 8)
    with pytest.raises(CheckpointFormatError, match="experts"):
        state_from_vendor(vendor, "deepseek_v3", n)
    mla = {k: v for k, v in tech.vendor_state().items() if "q_proj" not in k}
    mla[f"model.layers.{n}.self_attn.q_a_proj.weight"] = torch.zeros(8, 8)
    with pytest.raises(CheckpointFormatError):
        state_from_vendor(mla, "deepseek_v3", n)


def test_fp8_block_weights_dequantize():
    g = torch.Generator().manual_seed(0)
    w = torch.randn(200, 300, generator=g)
    padded = torch.nn.functional.pad(w.abs(), (0, 84, 0, 56))  # 256 x 384: whole 128 x 128 tiles
    blocks = padded.reshape(2, 128, 3, 128).amax((1, 3)) / 448  # one scale per tile, as the release format
    scale = blocks.repeat_interleave(128, 0)[:200].repeat_interleave(128, 1)[:, :300]
    codes = (w / scale).clamp(-448, 448).to(torch.float8_e4m3fn)
    out = dequantize_fp8_blocks({"a.weight": codes, "a.weight_scale_inv": blocks, "b.weight": w})
    assert set(out) == {"a.weight", "b.weight"} and out["a.weight"].dtype == torch.bfloat16
    torch.testing.assert_close(out["a.weight"].float(), w, atol=0.02, rtol=0.07)  # e4m3: 3 mantissa bits
    with pytest.raises(CheckpointFormatError):
        dequantize_fp8_blocks({"c.weight": codes})


def test_mtp_objective_trains():
    eff = eco.apply(tiny_model(), VendorMTPConfig(family="mimo"))
    before = eff.techniques["vendor_mtp"].fc.detach().clone()
    fit(eff, torch.randint(0, 1024, (4, 24)), steps=2, batch_size=2)
    assert not torch.equal(before, eff.techniques["vendor_mtp"].fc)
