"""Training data sources: token tensors, and the target's own greedy continuations of synthetic prompts (the
data the EAGLE heads are trained on when no corpus is available)."""

from __future__ import annotations

import torch

from ..decoding.config import DecodeConfig

__all__ = ["TensorSource", "greedy_continuations"]


class TensorSource:
    """Random row batches of a ``[N, S]`` token tensor, reproducible from ``seed`` and resumable."""

    def __init__(self, tokens: torch.Tensor, batch_size: int, seed: int = 0) -> None:
        self.tokens = tokens
        self.batch_size = batch_size
        self.gen = torch.Generator().manual_seed(seed)
        self.drawn = 0

    def next(self) -> torch.Tensor:
        idx = torch.randint(0, self.tokens.shape[0], (self.batch_size,), generator=self.gen)
        self.drawn += 1
        return self.tokens[idx.to(self.tokens.device)]

    def state(self) -> dict:
        return {"drawn": self.drawn, "gen": self.gen.get_state()}

    def restore(self, state: dict) -> None:
        self.drawn = state["drawn"]
        self.gen.set_state(state["gen"])


@torch.no_grad()
def greedy_continuations(model, n: int, prompt_len: int, new_tokens: int, batch: int = 32, seed: int = 0,
                         vocab: int | None = None) -> torch.Tensor:
    """``[n, prompt_len + new_tokens]`` rows: uniform-random prompts followed by the model's plain greedy
    continuation (CUDA graphs on the GPU)."""
    vocab = vocab or model.model.config.vocab_size
    gen = torch.Generator().manual_seed(seed)
    dev = model.device
    rows = []
    cfg = DecodeConfig(cycle_length=1, cuda_graphs=dev.type == "cuda")
    for start in range(0, n, batch):
        count = min(batch, n - start)
        prompts = torch.randint(0, vocab, (count, prompt_len), generator=gen).to(dev)
        results = model.decode_batch(list(prompts), new_tokens, decoding=cfg)
        for p, r in zip(prompts, results):
            rows.append(torch.cat([p, r.tokens.to(dev)]))
    return torch.stack(rows)
