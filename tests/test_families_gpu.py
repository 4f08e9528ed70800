"""The added model families on the CUDA path (bf16, sm_100a kernels): logits close to the fp32 CPU oracle of the
same weights, and greedy tree decoding equal to plain decoding token for token."""

import pytest
import torch
import transformers

import economize_b200 as eco
from economize_b200.models.llama import CausalLM
from economize_b200.techniques.eagle3 import Eagle3Config

pytestmark = pytest.mark.gpu

BASE = dict(vocab_size=1024, hidden_size=512, intermediate_size=1024, num_hidden_layers=3, num_attention_heads=8,
            num_key_value_heads=2, max_position_embeddings=1024, pad_token_id=0, rms_norm_eps=1e-6)
FAMILIES = {
    "granite": dict(embedding_multiplier=12.0, residual_multiplier=0.22, attention_multiplier=0.0078125,
                    logits_scaling=8.0),
    "phi3": dict(),
    "smollm3": dict(no_rope_layers=[1, 0, 1]),
    "olmo2": dict(),
    "qwen3_moe": dict(num_experts=8, num_experts_per_tok=2, moe_intermediate_size=256, norm_topk_prob=False),
    # head dimension 256 (the attention kernel's one-stage layout), GeGLU, (1 + w) norms
    "gemma": dict(head_dim=256, num_attention_heads=4, num_key_value_heads=1),
    # soft-capped scores and logits, sandwich norms, sliding windows on alternate layers
    "gemma2": dict(head_dim=128, sliding_window=80, query_pre_attn_scalar=128, attn_logit_softcapping=20.0,
                   final_logit_softcapping=15.0),
    "gemma3_text": dict(head_dim=256, num_attention_heads=4, num_key_value_heads=2, sliding_window=96,
                        query_pre_attn_scalar=256,
                        layer_types=["sliding_attention", "full_attention", "sliding_attention"]),
    "ministral": dict(head_dim=64, sliding_window=70,
                      layer_types=["sliding_attention", "full_attention", "sliding_attention"]),
    "olmo3": dict(sliding_window=90, layer_types=["sliding_attention", "sliding_attention", "full_attention"]),
    "olmoe": dict(num_experts=8, num_experts_per_tok=2, norm_topk_prob=False, intermediate_size=256),
    "qwen2_moe": dict(num_experts=8, num_experts_per_tok=2, moe_intermediate_size=256,
                      shared_expert_intermediate_size=384, norm_topk_prob=False),
    "granitemoe": dict(num_local_experts=8, num_experts_per_tok=2, intermediate_size=256, embedding_multiplier=6.0,
                       residual_multiplier=0.3, attention_multiplier=0.0125, logits_scaling=4.0),
    "granitemoeshared": dict(num_local_experts=8, num_experts_per_tok=2, intermediate_size=256,
                             shared_intermediate_size=384, embedding_multiplier=6.0, residual_multiplier=0.3,
                             attention_multiplier=0.0125, logits_scaling=4.0),
    # YaRN; queries scaled by position past 64 tokens
    "ministral3": dict(head_dim=64, eos_token_id=None,
                       rope_parameters={"rope_type": "yarn", "rope_theta": 1e6, "factor": 4.0,
                                        "original_max_position_embeddings": 64, "beta_fast": 32.0, "beta_slow": 1.0,
                                        "mscale": 1.0, "mscale_all_dim": 1.0, "llama_4_scaling_beta": 0.1}),
    # biased projections, sink logits, sliding windows on alternate layers, YaRN, clamped-SwiGLU biased experts
    "gpt_oss": dict(head_dim=64, num_local_experts=8, num_experts_per_tok=4, intermediate_size=256,
                    sliding_window=80),
}


@pytest.mark.parametrize("name", list(FAMILIES))
def test_family_on_gpu(cuda, name):
    cfg = transformers.CONFIG_MAPPING[name](**{**BASE, **FAMILIES[name]})
    torch.manual_seed(0)
    hf = transformers.AutoModelForCausalLM.from_config(cfg, attn_implementation="eager").float().eval()
    if name == "gpt_oss":  # non-zero biases and sink logits, so their kernels' paths count
        with torch.no_grad():
            for n, p in hf.named_parameters():
                if p.dim() == 1 and "norm" not in n or n.endswith("_bias"):
                    p.normal_(0, 0.1)
    cpu = CausalLM.from_hf(hf)
    gpu = CausalLM.from_hf(hf, dtype=torch.bfloat16, device=cuda)
    ids = torch.randint(1, 1024, (1, 160), generator=torch.Generator().manual_seed(1))  # longer than the windows
    want = eco.apply(cpu)(ids).float()
    got = eco.apply(gpu)(ids.to(cuda)).float().cpu()
    err = (got - want).abs().max().item()
    assert err <= 0.05 * want.abs().max().item() + 0.02, err
    em = eco.apply(gpu, Eagle3Config())
    prompts = [ids[0].to(cuda), ids[0, :17].to(cuda)]
    eco.ops.attention_usage(reset=True)
    plain = em.decode_batch(prompts, 20, decoding=eco.DecodeConfig(cycle_length=1))
    tree = em.decode_batch(prompts, 20, decoding=eco.DecodeConfig(
        cycle_length=7, draft_policy="dynamic_tree", draft_policy_options={"depth": 6, "topk": 10, "total_tokens": 60},
        cuda_graphs=True))
    for a, b in zip(plain, tree):
        assert torch.equal(a.tokens, b.tokens)
    assert eco.ops.require().status(0) == 0
    if gpu.config.sliding_window:  # the windowed layers ran the kernel's window path
        assert any("window" in mode for (_, _, _, mode) in eco.ops.attention_usage())
