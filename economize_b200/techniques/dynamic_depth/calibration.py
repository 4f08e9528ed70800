"""Threshold calibration of the early-exit methods: CALM's Learn then Test and FREE's Beta-mixture estimator.

Learn then Test calibration of CALM's exit threshold (Schuster et al., 2022, "Confident Adaptive Language
Modeling", Section 4; Angelopoulos et al., 2021, "Learn then Test"; economize ``dynamic_depth/calm.py:268-380``).

CALM picks the threshold ``lambda`` so that, with probability at least ``1 - delta`` over the calibration set, the
expected inconsistency between early-exit and full-model generations stays below ``epsilon``. Every candidate
``lambda`` is a hypothesis test of ``H_lambda: risk(lambda) > epsilon``, with the Hoeffding-Bentkus p-value of the
candidate's mean loss on ``n`` calibration prompts (Bates et al., 2021, "Distribution-free, risk-controlling
prediction sets", Proposition 5):

    p = min( exp(-n h(min(mean, eps), eps)),  e * P(Binomial(n, eps) <= ceil(n * mean)) ),
    h(a, b) = a log(a / b) + (1 - a) log((1 - a) / (1 - b)).

Fixed-sequence testing walks the candidates from the most conservative (largest) down and keeps every one whose
p-value is at most ``delta``, stopping at the first that is not; the smallest kept candidate is returned (``1.0``,
never exit early, when none is). No multiple-testing correction is needed for a fixed order.
"""

from __future__ import annotations

import dataclasses
import math
from collections.abc import Callable, Sequence

import torch

from ...errors import ConfigError

__all__ = ["beta_moments", "bmm_threshold", "calibrate_threshold", "free_calibration_pairs", "hoeffding_bentkus_pvalue",
           "ltt_threshold", "token_mismatch"]

DEFAULT_CANDIDATES = tuple(round(0.05 * i, 2) for i in range(1, 20))


def hoeffding_bentkus_pvalue(mean_loss: float, n: int, epsilon: float) -> float:
    """p-value of ``risk > epsilon`` given the mean of ``n`` losses in ``[0, 1]``."""
    from scipy.stats import binom

    if not 0.0 < epsilon < 1.0:
        raise ConfigError(f"epsilon must lie in (0, 1), got {epsilon}")
    if n < 1:
        raise ConfigError("Learn then Test needs at least one calibration example")
    a = min(max(float(mean_loss), 0.0), epsilon)
    kl = (a * math.log(a / epsilon) if a > 0 else 0.0) + (1.0 - a) * math.log((1.0 - a) / (1.0 - epsilon))
    hoeffding = math.exp(-n * kl)
    bentkus = math.e * float(binom.cdf(math.ceil(n * float(mean_loss) - 1e-12), n, epsilon))
    return min(1.0, hoeffding, bentkus)


def ltt_threshold(candidates: Sequence[float], losses, *, delta: float, epsilon: float) -> float:
    """The smallest candidate certified by fixed-sequence testing; ``losses[i]`` are the per-prompt losses in
    ``[0, 1]`` at ``candidates[i]``."""
    if not 0.0 < delta < 1.0:
        raise ConfigError(f"delta must lie in (0, 1), got {delta}")
    table = torch.as_tensor(losses, dtype=torch.float64)
    if table.dim() != 2 or table.shape[0] != len(candidates):
        raise ConfigError(f"losses must be [len(candidates), n], got {tuple(table.shape)}")
    if bool(((table < 0) | (table > 1)).any()):
        raise ConfigError("losses must lie in [0, 1]")
    chosen = 1.0
    for i in sorted(range(len(candidates)), key=lambda j: -float(candidates[j])):
        if hoeffding_bentkus_pvalue(float(table[i].mean()), table.shape[1], epsilon) > delta:
            break
        chosen = float(candidates[i])
    return chosen


def token_mismatch(tokens: torch.Tensor, reference: torch.Tensor) -> float:
    """CALM's token-level consistency loss: the fraction of positions (of the longer generation) at which two
    generations differ, a missing token counting as a difference."""
    a, b = tokens.reshape(-1).cpu(), reference.reshape(-1).cpu()
    length = max(a.numel(), b.numel())
    if length == 0:
        return 0.0
    shared = min(a.numel(), b.numel())
    return 1.0 - int((a[:shared] == b[:shared]).sum()) / length


def calibrate_threshold(model, prompts: Sequence[torch.Tensor], max_new_tokens: int, *, delta: float = 0.1,
                        epsilon: float = 0.1, candidates: Sequence[float] = DEFAULT_CANDIDATES,
                        loss: Callable[[torch.Tensor, torch.Tensor], float] = token_mismatch,
                        technique: str = "calm") -> float:
    """Calibrate the threshold of ``model``'s CALM technique on ``prompts`` and return it.

    Every prompt is decoded greedily by the full model (threshold 1: no token exits) and once per candidate;
    ``loss(early, full)`` scores each generation. The technique's configuration is restored afterwards; apply the
    result with ``dataclasses.replace(config, threshold=...)``. Decoding runs without CUDA graphs, since a captured
    pass would keep the threshold it was recorded with.
    """
    from ...decoding.config import DecodeConfig
    from .methods import CalmTechnique

    calm = model.techniques[technique]
    if not isinstance(calm, CalmTechnique):
        raise ConfigError(f"{technique!r} is a {type(calm).__name__}, not a CALM technique")
    if not prompts:
        raise ConfigError("calibration needs at least one prompt")
    decoding = DecodeConfig(cycle_length=1, cuda_graphs=False)
    original = calm.config
    rows: list[list[float]] = []
    try:
        calm.config = dataclasses.replace(original, threshold=1.0, decay_temperature=0.0)
        full = [model.decode(p, max_new_tokens, decoding=decoding).tokens for p in prompts]
        for lam in candidates:
            calm.config = dataclasses.replace(original, threshold=float(lam))
            rows.append([loss(model.decode(p, max_new_tokens, decoding=decoding).tokens, ref)
                         for p, ref in zip(prompts, full)])
    finally:
        calm.config = original
    return ltt_threshold(candidates, rows, delta=delta, epsilon=epsilon)


# ---- FREE's adaptive threshold (Bae et al., 2023, "Fast and Robust Early-Exiting Framework for Autoregressive
# Language Models with Synchronized Parallel Decoding", Section 4.3; economize ``dynamic_depth/free.py:170-230``) ----
def beta_moments(values: torch.Tensor, eps: float = 1e-4) -> tuple[float, float]:
    """Beta ``(alpha, beta)`` matching the mean ``m`` and variance ``v`` of samples in ``(0, 1)``:
    ``alpha = m c``, ``beta = (1 - m) c`` with ``c = m (1 - m) / v - 1`` (``v`` kept inside the valid range)."""
    x = values.double().flatten().clamp(eps, 1.0 - eps)
    m = float(x.mean())
    v = float(x.var(unbiased=False)) if x.numel() > 1 else 0.0
    v = min(max(v, eps * eps), m * (1.0 - m) * (1.0 - eps))
    c = m * (1.0 - m) / v - 1.0
    return m * c, (1.0 - m) * c


def bmm_threshold(confidence: torch.Tensor, agree: torch.Tensor, posterior: float = 0.4,
                  grid: Sequence[float] | None = None, default: float = 0.9) -> float:
    """FREE's threshold: the smallest ``lambda`` on ``grid`` whose posterior probability that the shallow and deep
    predictions agree reaches ``posterior``, under a two-component Beta mixture with equal priors fitted by moments
    to the confidences of agreeing and of disagreeing tokens. ``default`` while a class has fewer than two samples."""
    from scipy.stats import beta as beta_dist

    conf = confidence.detach().double().flatten().cpu()
    ok = agree.detach().bool().flatten().cpu()
    if int(ok.sum()) < 2 or int((~ok).sum()) < 2:
        return float(default)
    a1, b1 = beta_moments(conf[ok])
    a0, b0 = beta_moments(conf[~ok])
    lam = torch.tensor(list(grid) if grid is not None else [i / 100 for i in range(101)], dtype=torch.float64)
    x = lam.clamp(1e-4, 1 - 1e-4).numpy()
    p1, p0 = beta_dist.pdf(x, a1, b1), beta_dist.pdf(x, a0, b0)
    post = p1 / (p1 + p0 + 1e-300)
    hits = [i for i in range(len(lam)) if post[i] >= posterior]
    return float(lam[hits[0]]) if hits else float(lam[-1])


@torch.no_grad()
def free_calibration_pairs(model, input_ids: torch.Tensor, technique: str = "free") -> tuple[torch.Tensor, torch.Tensor]:
    """Shallow confidences (top-1 minus top-2 probability of the shallow exit) and shallow-deep agreement at every
    position of ``input_ids [B, T]`` (one teacher-forced pass), the inputs of :func:`bmm_threshold`."""
    from ... import ops
    from ...runtime.cache import StepBatch
    from .drafters import FreeTechnique

    free = model.techniques[technique]
    if not isinstance(free, FreeTechnique):
        raise ConfigError(f"{technique!r} is a {type(free).__name__}, not a FREE technique")
    lm = model.model
    ids = input_ids if input_ids.dim() == 2 else input_ids[None]
    ids = ids.to(lm.device)
    b, t = ids.shape
    k = len(free.view_layers())
    cache = lm.new_cache(b, ((t + 127) // 128) * 128)
    lengths = torch.full((b,), t, dtype=torch.int32, device=lm.device)
    h, aux = lm.forward_step(ids, StepBatch.prefill(lengths, t), cache, (k,))
    deep = lm.logits(h).float()
    shallow_h = ops.rmsnorm(aux[k].to(lm.dtype), lm.norm, lm.config.rms_norm_eps)[0]
    probs = torch.softmax(lm.logits(shallow_h).float(), -1)
    top = probs.topk(2, -1)
    conf = (top.values[..., 0] - top.values[..., 1]).reshape(-1)
    agree = (top.indices[..., 0] == deep.argmax(-1)).reshape(-1)
    return conf.cpu(), agree.cpu()
