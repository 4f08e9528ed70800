"""On-policy RL pieces for a jump drafter (economize ``techniques/jump/rl.py:1-9``), built on the open-loop rollout.

* :func:`jump_acceptance`: teacher-forced on sequences the policy produced, the speculative acceptance
  ``sum_v min(p, q)`` of every draft step from every start (``p`` the target's distribution of the drafted position,
  ``q`` the drafter's); :func:`~economize_b200.train.rl.expected_tokens` turns a row of it into tokens per cycle.
* :func:`hybrid_log_probs`: log-probabilities of the tokens under the policy that lossy cycle decoding samples from
  (``DecodeConfig(cycle_length=N, lossless=False)``): the target's distribution at the first token of every cycle,
  the drafter's at the ``N - 1`` after it. Both come from one prompt pass and one rollout of ``N - 1`` steps.

The target's distributions come from the engine's forward pass (no gradient); the drafted positions' log-probabilities
carry gradients to the predictor, the mixer and any target weight of layers ``m + 1 .. r`` that requires them.
"""

from __future__ import annotations

import torch

from ...errors import ConfigError
from ...runtime.cache import StepBatch

__all__ = ["hybrid_log_probs", "jump_acceptance"]


def _teacher(tech, tokens: torch.Tensor):
    model = tech.model
    m, _, r = tech.layers
    b, s = tokens.shape
    capture = tuple(sorted({*range(m, r + 1), *tech.sources}))
    with torch.no_grad():
        cache = model.new_cache(b, ((s + 127) // 128) * 128)
        lengths = torch.full((b,), s, dtype=torch.int32, device=tokens.device)
        final, aux = model.forward_step(tokens, StepBatch.prefill(lengths, s), cache, capture=capture)
        logits = model.logits(final).float()
    return aux, logits


def _draft_logits(tech, h_r: torch.Tensor) -> torch.Tensor:
    from ...ops import reference
    from ...train.objective import dense_linear

    model = tech.model
    x = reference.rmsnorm(h_r, model.norm, model.config.rms_norm_eps)[0]
    return dense_linear(x, model.head_weight, None).float() / model.config.logits_scaling


def jump_acceptance(tech, tokens: torch.Tensor, horizon: int, temperature: float = 1.0) -> torch.Tensor:
    """``[B, S - horizon, horizon]``: the acceptance of draft step ``j`` (last axis) from every start ``p`` (rows of
    the middle axis), against the target's distribution of position ``p + j`` at ``temperature``."""
    from ...train.rl import acceptance
    from .rollout import rollout_steps

    if temperature <= 0:
        raise ConfigError("acceptance needs a positive temperature (greedy decoding accepts by argmax equality)")
    aux, target = _teacher(tech, tokens)
    starts, steps = rollout_steps(tech, tokens, aux, horizon)
    out = []
    for j, (_, h_r) in enumerate(steps, start=1):
        p = torch.softmax(target[:, starts + j] / temperature, -1)
        q = torch.softmax(_draft_logits(tech, h_r) / temperature, -1)
        out.append(acceptance(p, q))
    return torch.stack(out, -1)


def hybrid_log_probs(tech, tokens: torch.Tensor, first: int, cycle_length: int) -> torch.Tensor:
    """``[B, S - first]``: the log-probability of every token from index ``first`` on (the first generated one)
    under lossy cycle decoding with cycles of ``cycle_length`` tokens: token ``t = first + i`` is sampled from the
    target at ``t - 1`` when ``i`` is a multiple of ``cycle_length``, else from draft step ``k = i mod cycle_length``
    of the rollout that starts at the cycle's last exact position ``t - k - 1``."""
    from .rollout import rollout_steps

    b, s = tokens.shape
    if cycle_length < 2 or not 1 <= first < s:
        raise ConfigError(f"hybrid log-probabilities need cycle_length >= 2 and 1 <= first < {s}, got "
                          f"{cycle_length}, {first}")
    horizon = cycle_length - 1
    # rollouts from the last starts run past the sequence: pad it (causal attention keeps every position up to a
    # row's own step independent of the padding)
    padded = torch.cat([tokens, tokens[:, -1:].expand(b, horizon)], 1)
    aux, target = _teacher(tech, padded)
    _, steps = rollout_steps(tech, padded, aux, horizon)
    exact = torch.log_softmax(target, -1)
    drafted = [torch.log_softmax(_draft_logits(tech, h_r), -1) for _, h_r in steps]
    columns = []
    for t in range(first, s):
        k = (t - first) % cycle_length
        tok = tokens[:, t]
        if k == 0:
            columns.append(exact[:, t - 1].gather(-1, tok[:, None])[:, 0])
        else:
            columns.append(drafted[k - 1][:, t - k - 1].gather(-1, tok[:, None])[:, 0])
    return torch.stack(columns, -1)
