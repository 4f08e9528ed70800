"""Pipeline placement over two GPUs: a model whose layers sit on cuda:0 and cuda:1 decodes exactly as the same model
on cuda:0 (the kernels are the same; only the stream moves between the devices). Skipped below two GPUs."""

import pytest
import torch

import economize_b200 as eco
from economize_b200.models.config import tiny_llama
from economize_b200.models.llama import CausalLM, init_weights
from economize_b200.parallel.pipeline import pipeline_split
from economize_b200.techniques.eagle3 import Eagle3Config

pytestmark = pytest.mark.gpu


def test_two_gpu_pipeline_equals_one(cuda):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    cfg = tiny_llama(hidden_size=512, num_heads=4, num_kv_heads=2, head_dim=128, num_layers=4, intermediate_size=1024)
    prompts = [torch.randint(0, 1024, (n,), generator=torch.Generator().manual_seed(n)).to(cuda) for n in (90, 17)]
    tree = eco.DecodeConfig(cycle_length=7, draft_policy="dynamic_tree",
                            draft_policy_options={"depth": 6, "topk": 10, "total_tokens": 60})
    whole = eco.apply(init_weights(CausalLM(cfg, torch.bfloat16, cuda), seed=0), Eagle3Config())
    whole.techniques["eagle3"].reset_parameters(seed=3)
    want = whole.decode_batch(prompts, 20, decoding=tree)
    split = eco.apply(init_weights(CausalLM(cfg, torch.bfloat16, cuda), seed=0), Eagle3Config())
    split.techniques["eagle3"].load_state_dict(whole.techniques["eagle3"].state_dict())
    pipeline_split(split, ["cuda:0", "cuda:1"])
    got = split.decode_batch(prompts, 20, decoding=tree)
    for a, b in zip(want, got):
        assert torch.equal(a.tokens, b.tokens)
    assert eco.ops.require().status(0) == 0 and eco.ops.require().status(1) == 0
