"""Model families beyond Llama/Mistral/Qwen2/Qwen3/Mixtral against the ``transformers`` implementation on the CPU
(fp32): the converted engine model's logits equal Hugging Face's, greedy decoding equals HF ``generate``, and the
state dict exports back to HF names. Tiny random configurations of each family's real ``model_type``."""

import pytest
import torch
import transformers

import economize_b200 as eco
from economize_b200.errors import UnsupportedModelError
from economize_b200.models.config import ModelConfig
from economize_b200.models.llama import CausalLM

BASE = dict(vocab_size=128, hidden_size=64, intermediate_size=96, num_hidden_layers=3, num_attention_heads=4,
            num_key_value_heads=2, max_position_embeddings=256, pad_token_id=0, rms_norm_eps=1e-6)

FAMILIES = {
    "granite": dict(embedding_multiplier=12.0, residual_multiplier=0.22, attention_multiplier=0.0078125,
                    logits_scaling=8.0),
    "phi3": dict(),
    "smollm3": dict(no_rope_layers=[1, 0, 1]),
    "olmo2": dict(),
    "qwen3_moe": dict(num_experts=4, num_experts_per_tok=2, moe_intermediate_size=48, norm_topk_prob=False),
    # GeGLU, (1 + w) norms, dtype-rounded embedding scale, head_dim 16
    "gemma": dict(head_dim=16),
    # + sandwich norms, soft-capped scores and logits, sliding window on alternate layers
    "gemma2": dict(head_dim=16, sliding_window=6, query_pre_attn_scalar=16, attn_logit_softcapping=5.0,
                   final_logit_softcapping=3.0),
    # + per-head q/k norms, separate rotary tables for the sliding layers
    "gemma3_text": dict(head_dim=16, sliding_window=5, query_pre_attn_scalar=24,
                        layer_types=["sliding_attention", "full_attention", "sliding_attention"],
                        rope_parameters={"sliding_attention": {"rope_type": "default", "rope_theta": 100.0},
                                         "full_attention": {"rope_type": "default", "rope_theta": 10000.0}}),
    "ministral": dict(head_dim=16, sliding_window=7,
                      layer_types=["sliding_attention", "full_attention", "sliding_attention"]),
    "olmo3": dict(sliding_window=6, layer_types=["sliding_attention", "sliding_attention", "full_attention"]),
    "olmoe": dict(num_experts=4, num_experts_per_tok=2, norm_topk_prob=False),
    "qwen2_moe": dict(num_experts=4, num_experts_per_tok=2, moe_intermediate_size=48,
                      shared_expert_intermediate_size=40, norm_topk_prob=False),
    # Granite's scales around MoE blocks; the shared variant adds an ungated shared expert
    "granitemoe": dict(num_local_experts=4, num_experts_per_tok=2, embedding_multiplier=6.0, residual_multiplier=0.3,
                       attention_multiplier=0.02, logits_scaling=4.0),
    "granitemoeshared": dict(num_local_experts=4, num_experts_per_tok=2, shared_intermediate_size=40,
                             embedding_multiplier=6.0, residual_multiplier=0.3, attention_multiplier=0.02,
                             logits_scaling=4.0),
    # YaRN and queries scaled by position beyond the original context (small here, so the scale moves)
    "ministral3": dict(head_dim=16, eos_token_id=None, rope_parameters={"rope_type": "yarn", "rope_theta": 10000.0, "factor": 4.0,
                                                     "original_max_position_embeddings": 8, "beta_fast": 32.0,
                                                     "beta_slow": 1.0, "mscale": 1.0, "mscale_all_dim": 1.0,
                                                     "llama_4_scaling_beta": 0.1}),
    # biased q/k/v/o, sink logits, sliding windows on alternate layers, YaRN, clamped-SwiGLU experts with biases
    "gpt_oss": dict(head_dim=16, num_local_experts=4, num_experts_per_tok=2, sliding_window=6,
                    rope_parameters={"rope_type": "yarn", "factor": 4.0, "beta_fast": 32.0, "beta_slow": 1.0,
                                     "truncate": False, "original_max_position_embeddings": 64,
                                     "rope_theta": 10000.0}),
}


def _hf(name, seed=0):
    cfg = transformers.CONFIG_MAPPING[name](**{**BASE, **FAMILIES[name]})
    torch.manual_seed(seed)
    # eager: the reference attention (sdpa drops Gemma-2's score soft-cap)
    model = transformers.AutoModelForCausalLM.from_config(cfg, attn_implementation="eager").float().eval()
    with torch.no_grad():  # larger than HF's 0.02 init, so the families' differences show in the logits
        for n, p in model.named_parameters():
            if p.dim() >= 2:
                p.normal_(0, 0.2)
            elif "norm" in n:
                p.uniform_(0.5, 1.5)
            elif name == "gpt_oss":  # biases and sink logits
                p.normal_(0, 0.5)
    return model


@pytest.mark.parametrize("name", list(FAMILIES))
def test_logits_match_transformers(name):
    hf = _hf(name)
    ours = CausalLM.from_hf(hf)
    ids = torch.randint(1, 128, (2, 19), generator=torch.Generator().manual_seed(1))
    with torch.no_grad():
        want = hf(ids).logits
    got = eco.apply(ours)(ids)
    torch.testing.assert_close(got, want, atol=2e-4, rtol=2e-4)


@pytest.mark.parametrize("name", list(FAMILIES))
def test_greedy_decoding_matches_generate(name):
    hf = _hf(name, seed=3)
    em = eco.apply(CausalLM.from_hf(hf))
    prompt = torch.randint(1, 128, (11,), generator=torch.Generator().manual_seed(2))
    with torch.no_grad():
        want = hf.generate(prompt[None], max_new_tokens=12, do_sample=False, min_new_tokens=12)[0, 11:]
    got = em.decode_batch([prompt], 12, decoding=eco.DecodeConfig(cycle_length=1))[0].tokens
    assert torch.equal(got, want)


@pytest.mark.parametrize("name", list(FAMILIES))
def test_state_dict_round_trip(name):
    hf = _hf(name)
    ours = CausalLM.from_hf(hf)
    exported = ours.hf_state_dict()
    ref = hf.state_dict()
    for key, value in ref.items():
        if key.endswith("inv_freq") or "rotary" in key:
            continue
        if key == "lm_head.weight" and hf.config.tie_word_embeddings:
            continue  # a tied head is the embedding
        assert key in exported, key
        torch.testing.assert_close(exported[key], value)
    assert ModelConfig.from_hf(ours.config.to_hf()).model_type == name


def test_unsupported_variants_are_refused():
    with pytest.raises(UnsupportedModelError):
        ModelConfig.from_hf(transformers.Phi3Config(**BASE, partial_rotary_factor=0.75))
    with pytest.raises(UnsupportedModelError):
        ModelConfig.from_hf(transformers.Qwen3MoeConfig(**{**BASE, **FAMILIES["qwen3_moe"]}, mlp_only_layers=[1]))
