"""The north-star benchmark configurations as compositions of the public API, at the small scale the CPU runs:
configuration 1 exactly as defined (its output equals plain greedy decoding), and 3 / 4 / 5 with every technique of
the recipe attached (depth pruning, int4 weights, fp8 KV, a quantized EAGLE-3 drafter; MoE + Medusa; KIVI + a
placed draft model with a StreamingLLM cache view)."""

import torch

import economize_b200 as eco
from economize_b200.bench import configs


def test_config1_plumbing_equals_plain_greedy():
    spec = configs.config1("cpu")
    assert spec.model.model.dtype == torch.float32 and [p.numel() for p in spec.prompts] == [17, 40]
    out = spec.step()
    plain = spec.model.decode_batch(spec.prompts, spec.new_tokens, decoding=eco.DecodeConfig(cycle_length=1))
    for a, b in zip(out, plain):
        assert a.tokens.numel() == 32 and torch.equal(a.tokens, b.tokens)


def test_config3_composition():
    spec = configs.config3("tiny", "cpu", batch=2, prompt_len=24, new_tokens=6, calibration_rows=2)
    assert set(spec.model.techniques) == {"depth_prune", "quant", "kv_fp8", "eagle3", "draft_quant"}
    assert len(spec.notes["removed_blocks"]) == 2 and spec.model.model.config.num_layers == 8
    assert all(r.tokens.numel() == 6 for r in spec.step())


def test_config4_composition():
    spec = configs.config4("tiny", "cpu", batch=2, prompt_len=20, new_tokens=6)
    assert "medusa" in spec.model.techniques and spec.model.model.config.num_experts == 8
    assert all(r.tokens.numel() == 6 for r in spec.step())


def test_config5_composition():
    spec = configs.config5("tiny", "cpu", batch=2, prompt_len=300, new_tokens=6, window=128, sink=4)
    assert set(spec.model.techniques) == {"kivi", "placed_draft_model"}
    draft = spec.model.techniques["placed_draft_model"].draft
    assert draft.kv_evictor is not None  # the draft model attends to a StreamingLLM view of its cache
    out = spec.step()
    plain = spec.model.decode_batch(spec.prompts, 6, decoding=eco.DecodeConfig(cycle_length=1))
    for a, b in zip(out, plain):  # drafting through the view leaves the target's greedy output unchanged
        assert torch.equal(a.tokens, b.tokens)
