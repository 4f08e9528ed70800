"""Building blocks for on-policy RL with a drafter in the loop (economize ``train/rl.py``).

* :func:`token_log_probs`: log-probabilities of chosen tokens and the entropies of the distributions, computed over
  chunks of positions so that the ``[tokens, vocab]`` float32 buffers stay small (gradients flow to the logits);
* :func:`acceptance`: the speculative-sampling acceptance ``sum_v min(p_v, q_v)`` of a draft distribution ``q``
  against the target distribution ``p`` at every step (Leviathan et al., 2023, Theorem 3.5);
* :func:`expected_tokens`: the expected tokens per cycle of a chain with per-step acceptances ``a_1 .. a_K``,
  ``1 + sum_k prod_{j <= k} a_j`` (the closed form ``(1 - a^{K+1}) / (1 - a)`` for equal rates).

An RL objective that rewards drafter-friendly policies combines them: the policy's log-probabilities with gradients
from :func:`token_log_probs`, and a reward shaped by :func:`expected_tokens` of the drafter's acceptances.
"""

from __future__ import annotations

from collections.abc import Callable

import torch

__all__ = ["acceptance", "expected_tokens", "token_log_probs"]


def token_log_probs(hidden: torch.Tensor, tokens: torch.Tensor, logits_fn: Callable[[torch.Tensor], torch.Tensor],
                    chunk: int = 256) -> tuple[torch.Tensor, torch.Tensor]:
    """``(log p(tokens), entropy)`` ``[B, T]`` for hidden states ``[B, T, H]`` read out by ``logits_fn``, computed
    ``chunk`` positions at a time."""
    b, t = tokens.shape
    logps, ents = [], []
    for s in range(0, t, chunk):
        logits = logits_fn(hidden[:, s:s + chunk]).float()
        lp = torch.log_softmax(logits, -1)
        logps.append(lp.gather(-1, tokens[:, s:s + chunk, None].long())[..., 0])
        ents.append(-(lp.exp() * lp).sum(-1))
    return torch.cat(logps, 1), torch.cat(ents, 1)


def acceptance(p: torch.Tensor, q: torch.Tensor) -> torch.Tensor:
    """``sum_v min(p, q)`` over the last axis: the probability that a token drawn from ``q`` survives verification
    against ``p`` (both normalized distributions)."""
    return torch.minimum(p, q).sum(-1)


def expected_tokens(alpha: torch.Tensor) -> torch.Tensor:
    """Expected tokens per cycle ``1 + sum_k prod_{j <= k} alpha_j`` of a chain with step acceptances
    ``alpha [..., K]``."""
    return 1.0 + torch.cumprod(alpha, -1).sum(-1)
