"""Open-loop rollouts of a jump drafter for training (economize ``techniques/jump/rollout.py:41``,
``train/rollout/cache.py``).

At decode time the drafter drafts ``h`` tokens after the last exact position ``p``: step ``j`` maps the previous
step's states (the exact ones of ``p`` at ``j = 1``) and the embedding of token ``p + j`` to a state after layer
``m``, runs the target's layers ``m + 1 .. r`` on it against the target's exact keys of positions ``<= p`` and its own
keys of positions ``p + 1 .. p + j``, and exits through the final norm and LM head. Training on teacher-forced
sources only (``horizon=1``) never shows the predictor its own errors; a rollout trains every step on the states the
drafter itself produced.

Every start ``p`` of a sequence rolls out at once: the stream of step ``j`` is a tensor whose row ``n`` is the token
at position ``starts[n] + j``. Per layer, a row's query sees the teacher's keys up to its start (one masked score
matrix against the whole sequence) and the keys of its own earlier steps (one score per step, a row-wise dot
product), so ``h`` steps cost ``h`` partial passes of ``S`` rows each. Target weights are frozen; gradients reach the
predictor and the mixer through every later step.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

from ...errors import ConfigError
from ...ops import reference

__all__ = ["rollout_steps"]


def _qkv(layer, config, x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor):
    """q ``[B, Hq, N, D]``, k and v ``[B, Hkv, N, D]`` of the normed stream ``x [B, N, H]`` at rows whose rotary
    rows are ``cos``/``sin`` ``[N, D/2]``."""
    from ...train.objective import dense_linear

    b, n, _ = x.shape
    hq, hkv, d = config.num_heads, config.num_kv_heads, config.head_dim
    q, k, v = dense_linear(x, layer.wqkv, layer.bqkv).split([hq * d, hkv * d, hkv * d], -1)
    q, k, v = q.reshape(b, n, hq, d), k.reshape(b, n, hkv, d), v.reshape(b, n, hkv, d)
    if layer.q_norm is not None:
        q = reference.rmsnorm(q, layer.q_norm, config.rms_norm_eps)[0]
        k = reference.rmsnorm(k, layer.k_norm, config.rms_norm_eps)[0]
    c, s = cos[None, :, None].to(q.dtype), sin[None, :, None].to(q.dtype)

    def rot(t):
        a, e = t[..., : d // 2], t[..., d // 2:]
        return torch.cat([a * c - e * s, e * c + a * s], -1)

    return rot(q).transpose(1, 2), rot(k).transpose(1, 2), v.transpose(1, 2)


def _mlp(layer, config, h: torch.Tensor) -> torch.Tensor:
    from ...train.objective import dense_linear

    x = reference.rmsnorm(h, layer.mlp_norm, config.rms_norm_eps)[0]
    a = reference.glu(dense_linear(x, layer.w_gate_up, None), config.hidden_act, config.swiglu_limit)
    if layer.down_hadamard:
        a = reference.hadamard(a, layer.down_hadamard)
    return h + dense_linear(a, layer.w_down, None)


def _rollout_layer(layer, config, h, starts, teacher_kv, own, cos, sin):
    """One target layer over the rollout stream ``h [B, N, H]`` of the current step; ``own`` collects this layer's
    keys and values of the steps so far (this step's is appended)."""
    from ...train.objective import dense_linear

    hq, hkv, d = config.num_heads, config.num_kv_heads, config.head_dim
    group = hq // hkv
    x = reference.rmsnorm(h, layer.attn_norm, config.rms_norm_eps)[0]
    q, k, v = _qkv(layer, config, x, cos, sin)
    own.append((k, v))
    tk, tv = teacher_kv
    scale = d ** -0.5
    scores = torch.matmul(q, tk.repeat_interleave(group, 1).transpose(-1, -2)).float() * scale  # [B, Hq, N, S]
    seen = torch.arange(tk.shape[2], device=h.device)[None, :] <= starts[:, None]  # keys up to each row's start
    scores = scores.masked_fill(~seen[None, None], float("-inf"))
    mine = [(q * ki.repeat_interleave(group, 1)).sum(-1, keepdim=True).float() * scale for ki, _ in own]
    probs = torch.softmax(torch.cat([scores, *mine], -1), -1).to(q.dtype)
    width = tk.shape[2]
    att = torch.matmul(probs[..., :width], tv.repeat_interleave(group, 1))
    for i, (_, vi) in enumerate(own):
        att = att + probs[..., width + i: width + i + 1] * vi.repeat_interleave(group, 1)
    b, _, n, _ = att.shape
    h = h + dense_linear(att.transpose(1, 2).reshape(b, n, hq * d), layer.wo, None)
    return _mlp(layer, config, h)


def rollout_steps(tech, tokens: torch.Tensor, aux: dict[int, torch.Tensor], horizon: int):
    """Roll the jump drafter out ``horizon`` steps from every start ``p <= S - 1 - horizon`` of ``tokens [B, S]``.

    ``aux`` holds the teacher's streams after ``v`` layers for ``v`` in ``m .. r - 1`` and the source layers. Returns
    ``starts [N]`` and, per step ``j``, ``(h_m_hat, h_r_hat)``: the predicted state after layer ``m`` and the stream
    after layer ``r`` of the tokens at positions ``starts + j`` (``[B, N, H]`` each)."""
    from ...train.objective import _check_plain_block

    model = tech.model
    config = model.config
    _check_plain_block(config)
    m, _, r = tech.layers
    b, s = tokens.shape
    if not 1 <= horizon <= s - 1:
        raise ConfigError(f"a rollout horizon of {horizon} needs sequences longer than it (got length {s})")
    starts = torch.arange(s - horizon, device=tokens.device)
    cos_all, sin_all = model.rope_tables(s)
    with torch.no_grad():  # the teacher's keys and values of layers m .. r - 1 over the whole sequence
        teacher_kv = {}
        for li in range(m, r):
            layer = model.layers[li]
            x = reference.rmsnorm(aux[li].to(layer.wqkv.dtype), layer.attn_norm, config.rms_norm_eps)[0]
            _, k, v = _qkv(layer, config, x, cos_all[:s].float(), sin_all[:s].float())
            teacher_kv[li] = (k, v)
    emb = model.embed_tokens(tokens)
    source = tech.mix({v: aux[v] for v in tech.sources})[:, starts]  # exact sources of every start
    own = {li: [] for li in range(m, r)}
    steps = []
    for j in range(1, horizon + 1):
        pos = starts + j
        h_m = tech.predictor(source.float(), emb[:, pos].float())
        h = h_m.to(model.layers[m].wqkv.dtype)
        captured = {}
        for li in range(m, r):
            if li in tech.sources:
                captured[li] = h
            h = _rollout_layer(model.layers[li], config, h, starts, teacher_kv[li], own[li],
                               cos_all[pos].float(), sin_all[pos].float())
        if r in tech.sources:
            captured[r] = h
        steps.append((h_m, h))
        source = tech.mix(captured)
    return starts, steps
