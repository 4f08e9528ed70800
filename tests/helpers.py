"""Shared fixtures of the CPU tests: tiny fp32 models and the full-recompute greedy oracle."""

from __future__ import annotations

import torch

from economize_b200.models.config import tiny_llama
from economize_b200.models.llama import CausalLM, init_weights


def tiny_model(seed: int = 0, **overrides) -> CausalLM:
    """4 layers, hidden 256, 4 heads / 2 KV heads, FFN 688, vocab 1024, theta 1e4, N(0, 0.02)."""
    return init_weights(CausalLM(tiny_llama(**overrides), torch.float32, "cpu"), seed=seed)


def micro_model(vocab: int = 16, seed: int = 0) -> CausalLM:
    return init_weights(CausalLM(tiny_llama(vocab_size=vocab, hidden_size=64, intermediate_size=128, num_layers=2,
                                            num_heads=2, num_kv_heads=1), torch.float32, "cpu"), seed=seed, std=0.3)


def prompts(lengths=(17, 40), vocab: int = 1024, seed: int = 0) -> list[torch.Tensor]:
    g = torch.Generator().manual_seed(seed)
    return [torch.randint(0, vocab, (n,), generator=g) for n in lengths]


@torch.no_grad()
def reference_greedy(model: CausalLM, prompt: torch.Tensor, n: int) -> torch.Tensor:
    """Greedy continuation by full causal recompute (no cache), the ground truth of every lossless path."""
    from economize_b200.runtime.cache import StepBatch

    seq = prompt.clone()
    out = []
    for _ in range(n):
        length = seq.numel()
        cache = model.new_cache(1, ((length + 127) // 128) * 128)
        h, _ = model.forward_step(seq[None], StepBatch.prefill(torch.tensor([length], dtype=torch.int32), length),
                                  cache)
        tok = int(model.logits(h[0, -1]).argmax())
        out.append(tok)
        seq = torch.cat([seq, torch.tensor([tok])])
    return torch.tensor(out)


def gpu_tiny_model(device, seed: int = 0) -> CausalLM:
    """A tiny bf16 model the CUDA kernels accept (head_dim 128, widths multiples of 64)."""
    cfg = tiny_llama(hidden_size=512, head_dim=128, num_heads=4, num_kv_heads=2, intermediate_size=1024)
    return init_weights(CausalLM(cfg, torch.bfloat16, device), seed=seed)
