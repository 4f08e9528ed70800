"""Public API surface, registries, configuration checks and checkpoint round-trips."""

import json

import pytest
import torch

import economize_b200 as eco
from economize_b200.decoding.policies import POLICIES
from economize_b200.decoding.tree import TreeOptions, ancestor_bits, popcount64, select_candidates
from economize_b200.decoding.verifiers import VERIFIERS
from economize_b200.techniques.eagle3 import Eagle3Config

from .helpers import prompts, tiny_model


def test_exports():
    for name in ("apply", "load", "save", "from_pretrained", "attach", "compatible", "incompatibility",
                 "compatibility_matrix", "EfficientModel", "DecodeConfig", "ConfigError", "TECHNIQUES", "FORMATS"):
        assert hasattr(eco, name)
    assert issubclass(eco.ConfigError, ValueError)
    assert issubclass(eco.UnknownNameError, KeyError)


def test_registries():
    assert {"greedy", "rejection", "typical", "accept_all"} <= set(VERIFIERS.names())
    assert {"fixed", "confidence", "dynamic_tree"} <= set(POLICIES.names())
    assert "eagle3" in eco.TECHNIQUES
    with pytest.raises(eco.UnknownNameError):
        eco.TECHNIQUES.get("nope")


def test_decode_config_checks():
    with pytest.raises(eco.ConfigError):
        eco.DecodeConfig(cycle_length=0)
    assert eco.DecodeConfig(window_cache=True).window_cache  # ring caches of sliding-window layers
    with pytest.raises(eco.ConfigError):
        eco.DecodeConfig(prefill_chunk=0)
    cfg = eco.DecodeConfig(cycle_length=7, draft_policy="dynamic_tree", draft_policy_options={"depth": 6})
    assert eco.DecodeConfig.from_dict(cfg.to_dict()) == cfg
    assert hash(cfg) == hash(eco.DecodeConfig.from_dict(json.loads(json.dumps(cfg.to_dict()))))


def test_tree_options():
    t = TreeOptions.from_options({"depth": 6, "topk": 10}, 7)
    assert t.total_tokens == 60 and t.forwarded == 50
    with pytest.raises(eco.ConfigError):
        TreeOptions.from_options({"depth": 2, "topk": 2, "total_tokens": 10}, 3)
    with pytest.raises(eco.ConfigError):
        TreeOptions.from_options({"bogus": 1}, 3)


def test_tree_rejects_rejection_verifier():
    em = eco.apply(tiny_model(), Eagle3Config())
    cfg = eco.DecodeConfig(cycle_length=4, verifier="rejection", draft_policy="dynamic_tree")
    with pytest.raises(eco.ConfigError):
        em.decoder(cfg, eco.TopPSampler())


def test_select_candidates_closed_under_ancestors():
    tokens = torch.arange(7)[None]
    scores = torch.tensor([[-1.0, -2.0, -1.5, -3.0, -2.5, -1.5, -9.0]])
    parents = torch.tensor([[-1, -1, 0, 0, 1, 2, 2]])
    depth = torch.tensor([0, 0, 1, 1, 1, 2, 2.0])
    tok, par = select_candidates(tokens, scores, parents, depth, 4)
    assert tok.tolist() == [[0, 1, 2, 5]]
    assert par.tolist() == [[-1, -1, 0, 2]]


def test_ancestor_bits():
    parents = torch.tensor([[0, 0, 1, 1, 3, 0]])
    bits = ancestor_bits(parents, 4)
    assert bits.tolist() == [[1, 3, 7, 11, 27, 33]]
    assert (popcount64(bits) - 1).tolist() == [[0, 1, 2, 2, 3, 1]]


def test_compatibility():
    assert not eco.compatible("eagle3", "eagle3")
    assert "twice" in eco.incompatibility("eagle3", "eagle3")
    assert eco.compatibility_matrix(["eagle3"]) == {"eagle3": {"eagle3": None}}
    with pytest.raises(eco.IncompatibleTechniquesError):
        eco.apply(tiny_model(), Eagle3Config(), Eagle3Config())


def test_save_load_roundtrip(tmp_path):
    model = tiny_model()
    em = eco.apply(model, Eagle3Config(draft_vocab=512), decoding=eco.DecodeConfig(cycle_length=3))
    em.techniques["eagle3"].reset_parameters(seed=3)
    em.save_pretrained(tmp_path)
    meta = json.loads((tmp_path / "economize_config.json").read_text())
    assert meta["techniques"][0]["technique"] == "eagle3" and meta["schema_version"] == 1
    em2 = eco.load(model, tmp_path)
    a, b = em.techniques["eagle3"].export_state(), em2.techniques["eagle3"].export_state()
    assert a.keys() == b.keys() and all(torch.equal(a[k], b[k]) for k in a)
    assert em2.decoding == em.decoding
    r1 = em.decode_batch(prompts(), 8)
    r2 = em2.decode_batch(prompts(), 8)
    assert all(torch.equal(x.tokens, y.tokens) for x, y in zip(r1, r2))


def test_official_eagle3_layout(tmp_path):
    safetensors = pytest.importorskip("safetensors.torch")
    model = tiny_model()
    em = eco.apply(model, Eagle3Config(draft_vocab=512))
    tech = em.techniques["eagle3"]
    tech.reset_parameters(seed=4)
    from economize_b200.techniques.eagle3.formats import to_official_state

    c = model.config
    cfg = {"architectures": ["LlamaForCausalLMEagle3"], "hidden_size": c.hidden_size, "num_attention_heads": c.num_heads,
           "num_key_value_heads": c.num_kv_heads, "intermediate_size": c.intermediate_size, "vocab_size": c.vocab_size,
           "draft_vocab_size": 512, "rms_norm_eps": c.rms_norm_eps, "rope_theta": c.rope_theta, "num_hidden_layers": 1}
    (tmp_path / "config.json").write_text(json.dumps(cfg))
    safetensors.save_file({k: v.contiguous() for k, v in to_official_state(tech).items()},
                          str(tmp_path / "model.safetensors"))
    ck = eco.read_checkpoint(tmp_path)
    assert ck.configs[0].draft_vocab == 512
    em2 = eco.attach(model, ck)
    a, b = tech.export_state(), em2.techniques["eagle3"].export_state()
    assert all(torch.equal(a[k], b[k]) for k in a)


def test_reference_checkpoint_interop(tmp_path):
    """A checkpoint written by the reference library (if installed) loads here with identical tensors. The
    reference runs in a subprocess: importing it patches transformers' attention functions process-wide."""
    import os
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    ref_dir = os.path.join(root, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_dir, "economize")):
        pytest.skip("reference not installed")
    script = f"""
import sys, torch
sys.path.insert(0, {root!r}); sys.path.insert(0, {ref_dir!r})
import transformers, economize as ref
from economize.techniques.eagle3 import Eagle3Config
from tests.helpers import tiny_model
model = tiny_model()
hf = transformers.LlamaForCausalLM(model.config.to_hf()).eval()
hf.load_state_dict(model.hf_state_dict())
rm = ref.apply(hf, Eagle3Config(draft_vocab=512))
torch.manual_seed(0)
with torch.no_grad():
    for p in rm.techniques["eagle3"].parameters():
        p.normal_(0, 0.02)
ref.save(rm, {str(tmp_path)!r})
torch.save(rm.techniques["eagle3"].state_dict(), {str(tmp_path / "expected.pt")!r})
"""
    proc = subprocess.run([sys.executable, "-c", script], capture_output=True, text=True, timeout=600)
    if proc.returncode != 0:
        pytest.skip(f"reference could not write a checkpoint here: {proc.stderr.strip().splitlines()[-1:]}")
    em = eco.load(tiny_model(), tmp_path, check_teacher=False)
    ours = em.techniques["eagle3"].export_state()
    theirs = torch.load(tmp_path / "expected.pt", weights_only=True)
    for k, v in theirs.items():
        assert torch.equal(ours[k].to(v.dtype), v), k
