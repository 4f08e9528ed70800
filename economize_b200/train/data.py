"""Training data sources (economize ``train/data``): token tensors, memory-mapped token files, data-parallel
sharding, chats through a tokenizer's chat template, synthetic passkey prompts, and the target's own greedy
continuations of synthetic prompts (the data the EAGLE heads are trained on when no corpus is available)."""

from __future__ import annotations

import torch

from ..decoding.config import DecodeConfig

__all__ = ["ShardedSource", "TensorSource", "TokenFileSource", "chat_tokens", "greedy_continuations",
           "passkey_prompts"]


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


class TokenFileSource:
    """Random windows of ``seq_len + 1`` tokens from a flat binary token file (``uint16`` or ``uint32``, memory
    mapped), reproducible from ``seed`` and resumable; ``rank`` / ``world`` give each data-parallel rank its own
    stream."""

    def __init__(self, path, batch_size: int, seq_len: int, dtype: str = "uint16", seed: int = 0, rank: int = 0,
                 world: int = 1) -> None:
        import numpy as np

        self.data = np.memmap(path, dtype=np.dtype(dtype), mode="r")
        if self.data.shape[0] <= seq_len + 1:
            raise ValueError(f"{path} holds fewer than seq_len + 1 = {seq_len + 1} tokens")
        self.batch_size, self.seq_len = batch_size, seq_len
        self.gen = torch.Generator().manual_seed(seed + 1000003 * rank)
        self.drawn = 0

    def next(self) -> torch.Tensor:
        import numpy as np

        starts = torch.randint(0, self.data.shape[0] - self.seq_len - 1, (self.batch_size,), generator=self.gen)
        rows = [np.asarray(self.data[s: s + self.seq_len + 1], dtype=np.int64) for s in starts.tolist()]
        self.drawn += 1
        return torch.from_numpy(np.stack(rows))

    def state(self) -> dict:
        return {"drawn": self.drawn, "gen": self.gen.get_state()}

    def restore(self, state: dict) -> None:
        self.drawn = state["drawn"]
        self.gen.set_state(state["gen"])


class ShardedSource:
    """Every ``world``-th batch of ``source``, starting at ``rank`` (data-parallel sharding of a shared stream)."""

    def __init__(self, source, rank: int, world: int) -> None:
        self.source, self.rank, self.world = source, rank, world
        for _ in range(rank):
            source.next()

    def next(self) -> torch.Tensor:
        batch = self.source.next()
        for _ in range(self.world - 1):
            self.source.next()
        return batch

    def state(self) -> dict:
        return self.source.state() if hasattr(self.source, "state") else {}

    def restore(self, state: dict) -> None:
        if hasattr(self.source, "restore"):
            self.source.restore(state)


def chat_tokens(tokenizer, conversations, max_len: int) -> torch.Tensor:
    """Chats (lists of ``{"role", "content"}`` messages) rendered by the tokenizer's chat template and padded or cut
    to ``max_len`` tokens: ``[N, max_len]`` (pad: the tokenizer's pad or eos id)."""
    pad = tokenizer.pad_token_id if tokenizer.pad_token_id is not None else tokenizer.eos_token_id
    rows = []
    for chat in conversations:
        ids = tokenizer.apply_chat_template(chat, tokenize=True)
        ids = list(ids["input_ids"] if isinstance(ids, dict) else ids)[:max_len]
        rows.append(ids + [pad] * (max_len - len(ids)))
    return torch.tensor(rows, dtype=torch.long)


def passkey_prompts(n: int, length: int, vocab: int, key_len: int = 5, seed: int = 0,
                    filler: int = 7) -> tuple[torch.Tensor, torch.Tensor]:
    """Synthetic passkey retrieval: ``[n, length]`` prompts of repeated filler tokens with a ``key_len``-token key
    at a random depth, followed by the key's first token as a cue; returns the prompts and the keys."""
    gen = torch.Generator().manual_seed(seed)
    prompts = torch.full((n, length), filler, dtype=torch.long)
    keys = torch.randint(16, vocab, (n, key_len), generator=gen)
    depth = torch.randint(1, length - 2 * key_len - 1, (n,), generator=gen)
    for i in range(n):
        d = int(depth[i])
        prompts[i, d: d + key_len] = keys[i]
        prompts[i, -1] = keys[i, 0]
    return prompts, keys
