"""Speculative speculative decoding (SSD; Kumar et al., 2026) across two ranks: the target verifies on its GPU while
the drafter, on another GPU, already drafts the next chain behind every likely verification outcome (economize
``distributed/ssd.py:175-295``, ``distributed/workers.py:265-454``).

One process per GPU. Rank ``target_rank`` holds the target model, rank ``draft_rank`` a draft LM; the handoff is
point-to-point over ``torch.distributed`` (NCCL on GPUs, on a side stream so the messages do not queue behind the
drafter's speculation; Gloo on the CPU). Per round:

    drafter  sends the spine d_1..d_k, then speculates: for every guess (a, y') of the outcome (the ``fanout``
             likeliest tokens at depth a other than d_{a+1}, and after d_k for a = k) it drafts the next chain,
             all (k + 1) fanout chains in k + 1 tree passes of the draft LM against its own cache
    target   receives the spine, verifies [y, d_1..d_k] in one chain pass (greedy), sends (a, y, done)
    drafter  on a hit the next spine is ready at once (its K/V are moved to their slots by the compaction kernel);
             on a miss it drafts after y

The output equals the target's greedy decoding, or with ``temperature > 0`` is distributed as the target's own
sampling (speculative sampling verification). Batch size one: SSD trades drafter work for latency.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import torch
import torch.distributed as dist

from .. import ops
from ..errors import ConfigError
from ..runtime.cache import KVCache, StepBatch
from ..validation import check_choice, check_positive

__all__ = ["AsyncSpeculativeDecoder", "SSDConfig", "SSDResult", "ssd_generate"]


@dataclass(frozen=True)
class SSDConfig:
    """``draft_length`` ``k`` drafts per round; ``fanout`` guesses per outcome depth; ``mode``: ``"async"``
    (speculate while the target verifies) or ``"sync"`` (draft after every outcome). ``temperature`` 0 verifies
    greedily; above 0 the target samples losslessly from its (``top_p``-filtered) distribution by speculative
    sampling: the drafter's greedy drafts are point masses ``q``, so draft ``d`` is kept with probability ``p(d)``
    and a rejection draws from ``p`` without ``d`` renormalised, the output distribution being the target's own.
    ``seed`` starts the target's sampling generator afresh for every generation."""

    draft_length: int = 4
    fanout: int = 2
    mode: str = "async"
    temperature: float = 0.0
    top_p: float = 1.0
    seed: int = 0

    def __post_init__(self) -> None:
        check_positive("draft_length", self.draft_length)
        check_positive("fanout", self.fanout)
        check_choice("mode", self.mode, ("async", "sync"))
        if self.temperature < 0.0 or not 0.0 < self.top_p <= 1.0:
            raise ConfigError(f"SSD needs temperature >= 0 and 0 < top_p <= 1, got {self.temperature}, {self.top_p}")
        k, g = self.draft_length, (self.draft_length + 1) * self.fanout
        if (k + 1) + g * (k + 1) > 64:
            raise ConfigError("(k + 1) (1 + (k + 1) fanout) must not exceed 64 (the speculation tree's ancestor "
                              "bits are one int64 per node)")

    @property
    def sampling(self) -> bool:
        return self.temperature > 0.0


def _probs(logits: torch.Tensor, config: SSDConfig) -> torch.Tensor:
    """The target's sampling distribution ``[..., V]``: softmax at ``temperature``, then nucleus ``top_p``."""
    p = torch.softmax(logits.float() / config.temperature, -1)
    if config.top_p < 1.0:
        sorted_p, order = p.sort(-1, descending=True)
        keep = sorted_p.cumsum(-1) - sorted_p < config.top_p  # the smallest prefix whose mass reaches top_p
        p = torch.zeros_like(p).scatter_(-1, order, sorted_p * keep)
        p = p / p.sum(-1, keepdim=True)
    return p


@dataclass
class SSDResult:
    tokens: torch.Tensor
    rounds: int = 0
    hits: int = 0
    acceptance: list = field(default_factory=list)

    @property
    def hit_rate(self) -> float:
        return self.hits / max(self.rounds - 1, 1)

    @property
    def acceptance_length(self) -> float:
        """Tokens committed per verification pass."""
        return 1.0 + sum(self.acceptance) / max(len(self.acceptance), 1)


class _Link:
    """Point-to-point messages between the two ranks (a side CUDA stream under NCCL)."""

    def __init__(self, peer: int, device: torch.device, group=None) -> None:
        self.peer, self.device, self.group = peer, device, group
        self.stream = torch.cuda.Stream(device) if device.type == "cuda" else None

    def send(self, t: torch.Tensor) -> None:
        if self.stream is None:
            dist.send(t, self.peer, group=self.group)
            return
        self.stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.stream):
            dist.send(t, self.peer, group=self.group)
        t.record_stream(self.stream)

    def recv(self, like: torch.Tensor) -> torch.Tensor:
        if self.stream is None:
            dist.recv(like, self.peer, group=self.group)
            return like
        with torch.cuda.stream(self.stream):
            dist.recv(like, self.peer, group=self.group)
        torch.cuda.current_stream(self.device).wait_stream(self.stream)
        return like


def _prefill(model, tokens: torch.Tensor, cache: KVCache) -> torch.Tensor:
    n = tokens.numel()
    lengths = torch.tensor([n], dtype=torch.int32, device=tokens.device)
    hidden, _ = model.forward_step(tokens[None], StepBatch.prefill(lengths, n), cache)
    return hidden[0]


def _chain_pass(model, tokens: torch.Tensor, start: int, cache: KVCache) -> torch.Tensor:
    """Forward ``tokens [T]`` at positions ``start ..`` (causal); returns the final hidden states ``[T, H]``."""
    dev = tokens.device
    t = tokens.numel()
    kv = torch.tensor([start], dtype=torch.int32, device=dev)
    n = torch.tensor([t], dtype=torch.int32, device=dev)
    pos = (start + torch.arange(t, device=dev, dtype=torch.int32))[None]
    hidden, _ = model.forward_step(tokens[None], StepBatch(kv, n, pos), cache)
    return hidden[0]


class _Drafter:
    """The draft LM's side: spines, speculation trees and their adoption."""

    def __init__(self, model, config: SSDConfig, capacity: int) -> None:
        self.model, self.k, self.fanout = model, config.draft_length, config.fanout
        self.g = (self.k + 1) * self.fanout
        self.cache = model.new_cache(1, ((capacity + (self.k + 1) * (1 + self.g) + 127) // 128) * 128)

    def logits(self, hidden: torch.Tensor) -> torch.Tensor:
        return self.model.logits(hidden).float()

    def draft(self, root: int, pos: int) -> tuple[torch.Tensor, torch.Tensor]:
        """The spine after ``root`` at position ``pos``: tokens ``[k]`` and the distributions ``[k + 1, V]`` after
        root, d_1, .., d_k (their K/V end up in slots ``pos .. pos + k``)."""
        dev = self.model.device
        tok = torch.tensor([root], dtype=torch.long, device=dev)
        tokens, dists = [], []
        for j in range(self.k + 1):
            logits = self.logits(_chain_pass(self.model, tok, pos + j, self.cache))[-1]
            dists.append(logits)
            tok = ops.argmax(logits[None]).reshape(1)
            if j < self.k:
                tokens.append(tok)
        return torch.cat(tokens), torch.stack(dists)

    def speculate(self, spine: torch.Tensor, dists: torch.Tensor, pos: int):
        """Chains behind every guessed outcome: guesses ``[G]`` (depth ``a`` and token), chains ``[G, k]`` and the
        distributions after each chain's last token ``[G, V]``; the nodes' K/V sit in the region after the spine."""
        k, f, g = self.k, self.fanout, self.g
        dev = spine.device
        masked = dists.clone()
        masked[torch.arange(k, device=dev), spine] = -float("inf")  # d_{a+1} was rejected at depth a < k
        guesses = masked.topk(f, -1).indices.reshape(-1)  # [G]: depth a = index // f
        depth_a = torch.arange(k + 1, device=dev).repeat_interleave(f)
        base = (k + 1)  # region offsets: [root, d_1..d_k][depth-0 nodes][depth-1 nodes]...
        spine_bits = (torch.ones(g, dtype=torch.int64, device=dev) << (depth_a + 1)) - 1  # root + d_1..d_a
        own = torch.zeros(g, dtype=torch.int64, device=dev)
        tok = guesses
        chain, dist_all = [], []
        kv = torch.tensor([pos], dtype=torch.int32, device=dev)
        for t in range(k + 1):
            own = own | (torch.ones(g, dtype=torch.int64, device=dev) << (base + t * g + torch.arange(g, device=dev)))
            positions = (pos + 1 + depth_a + t).to(torch.int32)[None]
            n_fwd = torch.tensor([base + (t + 1) * g], dtype=torch.int32, device=dev)
            sb = StepBatch(kv, n_fwd, positions, (spine_bits | own)[None], base + t * g)
            hidden, _ = self.model.forward_step(tok[None], sb, self.cache)
            logits = self.logits(hidden[0])
            dist_all.append(logits)
            if t < k:
                tok = ops.argmax(logits)
                chain.append(tok)
        return guesses, depth_a, torch.stack(chain, 1), torch.stack(dist_all, 1)

    def adopt(self, spec, pos: int, a: int, y: int):
        """The next spine if ``(a, y)`` was guessed (moving its K/V to slots ``pos + 1 + a ..``), else ``None``."""
        guesses, depth_a, chains, dists = spec
        hit = ((depth_a == a) & (guesses == y)).nonzero()
        if hit.numel() == 0:
            return None
        gi = int(hit[0, 0])
        dev = guesses.device
        k, g = self.k, self.g
        path = ((k + 1) + torch.arange(k + 1, device=dev) * g + gi - (1 + a)).to(torch.int32)[None]
        ops.kv_compact(self.cache.data, torch.tensor([pos + 1 + a], dtype=torch.int32, device=dev), path,
                       torch.tensor([k], dtype=torch.int32, device=dev))
        return chains[gi], dists[gi]


def ssd_generate(model, prompt: torch.Tensor, max_new_tokens: int, config: SSDConfig | None = None, *,
                 target_rank: int = 0, draft_rank: int = 1, group=None) -> SSDResult | None:
    """Run SSD on this rank: the target's rank returns the :class:`SSDResult`, the drafter's rank returns ``None``.
    ``model`` is this rank's model (the target or the draft LM); both ranks pass the same prompt and config."""
    config = config or SSDConfig()
    rank = dist.get_rank(group) if group is not None else dist.get_rank()
    if rank not in (target_rank, draft_rank):
        raise ConfigError(f"rank {rank} is neither the SSD target ({target_rank}) nor the drafter ({draft_rank})")
    dev = model.device
    prompt = prompt.reshape(-1).to(dev)
    k = config.draft_length
    p = prompt.numel()
    capacity = p + max_new_tokens + k + 2
    if rank == target_rank:
        return _target_loop(model, prompt, max_new_tokens, config, _Link(draft_rank, dev, group), capacity)
    _draft_loop(model, prompt, config, _Link(target_rank, dev, group), capacity)
    return None


@torch.no_grad()
def _target_loop(model, prompt, max_new, config, link: _Link, capacity: int) -> SSDResult:
    dev = model.device
    k = config.draft_length
    cache = model.new_cache(1, ((capacity + 127) // 128) * 128)
    if prompt.numel() > 1:
        _prefill(model, prompt[:-1], cache)
    last = _chain_pass(model, prompt[-1:], prompt.numel() - 1, cache)[-1]
    gen = torch.Generator(device=dev)
    gen.manual_seed(config.seed)
    if config.sampling:
        u = torch.rand(1, generator=gen, device=dev)
        root = int(ops.sample(_probs(model.logits(last[None]), config), u)[0])
    else:
        root = int(ops.argmax(model.logits(last[None]))[0])
    out = [root]
    n = prompt.numel() + 1  # committed tokens; the last (root) sits at position n - 1 without K/V yet
    result = SSDResult(torch.empty(0))
    done = max_new <= 1
    link.send(torch.tensor([root, int(done)], dtype=torch.long, device=dev))
    spine = torch.zeros(k, dtype=torch.long, device=dev)
    while not done:
        link.recv(spine)
        chain = torch.cat([torch.tensor([out[-1]], device=dev), spine])
        hidden = _chain_pass(model, chain, n - 1, cache)
        if config.sampling:  # speculative sampling with point-mass drafts (lossless for any drafter)
            p = _probs(model.logits(hidden), config)[None]  # [1, k + 1, V]
            q = torch.zeros(1, k, p.shape[-1], dtype=p.dtype, device=dev)
            q[0, torch.arange(k, device=dev), spine] = 1.0
            n_acc, drawn = ops.rejection(p, q, spine[None], torch.rand(1, k, generator=gen, device=dev),
                                         torch.rand(1, generator=gen, device=dev))
            a, y = n_acc[0], drawn[0, n_acc[0]]
        else:
            pred = model.greedy(hidden)  # [k + 1]
            ok = (pred[:-1] == spine).int().cumprod(0)
            a = ok.sum()
            y = pred[a]
        a_i, y_i = int(a), int(y)  # waits for the target's pass only
        committed = spine[:a_i].tolist() + [y_i]
        out.extend(committed)
        n += a_i + 1
        result.rounds += 1
        result.acceptance.append(a_i)
        done = len(out) >= max_new
        link.send(torch.tensor([a_i, y_i, int(done)], dtype=torch.long, device=dev))
    result.tokens = torch.tensor(out[:max_new], dtype=torch.long)
    # the drafter reports its hits at the end
    hits = torch.zeros(1, dtype=torch.long, device=dev)
    link.recv(hits)
    result.hits = int(hits)
    return result


@torch.no_grad()
def _draft_loop(model, prompt, config, link: _Link, capacity: int) -> None:
    dev = model.device
    drafter = _Drafter(model, config, capacity)
    if prompt.numel() > 1:
        _prefill(model, prompt[:-1], drafter.cache)
    first = torch.zeros(2, dtype=torch.long, device=dev)
    link.recv(first)
    hits = 0
    if int(first[1]) == 0:
        # the cache holds the prompt but its last token: the spine pass writes it, then the root
        _chain_pass(model, prompt[-1:], prompt.numel() - 1, drafter.cache)
        pos = prompt.numel()  # the root's position
        spine, dists = drafter.draft(int(first[0]), pos)
        outcome = torch.zeros(3, dtype=torch.long, device=dev)
        while True:
            link.send(spine)
            spec = drafter.speculate(spine, dists, pos) if config.mode == "async" else None
            link.recv(outcome)
            a, y, done = (int(v) for v in outcome.tolist())
            if done:
                break
            nxt = drafter.adopt(spec, pos, a, y) if spec is not None else None
            if nxt is not None:
                hits += 1
                spine, dists = nxt
            else:
                spine, dists = drafter.draft(y, pos + 1 + a)
            pos = pos + 1 + a
    link.send(torch.tensor([hits], dtype=torch.long, device=dev))


class AsyncSpeculativeDecoder:
    """The per-rank SSD decoder: ``generate`` on the target's rank returns the :class:`SSDResult`, on the drafter's
    rank it serves the drafts and returns ``None`` (both ranks call it with the same prompt)."""

    def __init__(self, model, config: SSDConfig | None = None, *, target_rank: int = 0, draft_rank: int = 1,
                 group=None) -> None:
        self.model, self.config = model, config or SSDConfig()
        self.target_rank, self.draft_rank, self.group = target_rank, draft_rank, group

    def generate(self, prompt: torch.Tensor, max_new_tokens: int) -> SSDResult | None:
        return ssd_generate(self.model, prompt, max_new_tokens, self.config, target_rank=self.target_rank,
                            draft_rank=self.draft_rank, group=self.group)
