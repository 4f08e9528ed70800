"""Plain PyTorch implementations of every operator (CPU path and fp32 numerics oracle of the CUDA kernels).

Each function computes the same thing as the kernel of the same name in ``economize_b200/csrc``. The dtype
behaviour follows Hugging Face's Llama modules where the result is rounded (RMSNorm rounds the normalized value to
the input dtype before the weight multiply; rotary products are taken in the input dtype), so fp32 runs on CPU
reproduce ``transformers`` exactly.
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

__all__ = [
    "attention",
    "ngram",
    "rejection",
    "sample",
    "greedy_accept",
    "kv_compact",
    "linear",
    "rmsnorm",
    "rope_store",
    "silu_mul",
    "visible_mask",
]


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float,
            residual: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """``(norm(x + residual) * weight, x + residual)``; the sum is rounded to ``x.dtype`` first."""
    summed = x if residual is None else (x + residual)
    h = summed.float()
    h = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps)
    return weight * h.to(x.dtype), summed


def _rotate(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    half = x.shape[-1] // 2
    rot = torch.cat((-x[..., half:], x[..., :half]), -1)
    c = torch.cat((cos, cos), -1).to(x.dtype)
    s = torch.cat((sin, sin), -1).to(x.dtype)
    return x * c + rot * s


def paged_logical(pool: torch.Tensor, pages: torch.Tensor) -> torch.Tensor:
    """A logical ``[B, H_kv, C * 128, D]`` copy of one layer's K (or V) pool view ``[P, H_kv, 128, D]`` read through its
    page table ``[B, C]`` (chunks that share a ring page repeat it)."""
    blocks = pool[pages.long()]  # [B, C, H_kv, 128, D]
    b, c, h, w, d = blocks.shape
    return blocks.permute(0, 2, 1, 3, 4).reshape(b, h, c * w, d)


def _paged_slot(pages: torch.Tensor, b: int, slot: int) -> tuple[int, int]:
    return int(pages[b, slot // 128]), slot % 128


def rope_store(qkv: torch.Tensor, positions: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor, num_heads: int,
               num_kv_heads: int, head_dim: int, k_cache: torch.Tensor, v_cache: torch.Tensor,
               kv_len: torch.Tensor, n_new: torch.Tensor, q_norm: torch.Tensor | None = None,
               k_norm: torch.Tensor | None = None, eps: float = 1e-6, q_offset: int = 0,
               k_scale: torch.Tensor | None = None, v_scale: torch.Tensor | None = None,
               pages: torch.Tensor | None = None) -> torch.Tensor:
    """Rotate queries and keys of ``qkv [B, T, (H + 2 H_kv) D]`` (optionally after a per-head RMSNorm), write the keys
    and values of token ``t`` to cache slot ``kv_len[b] + q_offset + t`` of ``k_cache/v_cache [B, H_kv, S, D]`` when
    ``q_offset + t < n_new[b]``, and return the rotated queries ``[B, T, H, D]``. fp8 caches store
    ``e4m3(value / scale)`` with one fp32 scale per KV head (``k_scale``, ``v_scale`` ``[H_kv]``)."""
    batch, length, _ = qkv.shape
    q, k, v = qkv.split([num_heads * head_dim, num_kv_heads * head_dim, num_kv_heads * head_dim], -1)
    q = q.reshape(batch, length, num_heads, head_dim)
    k = k.reshape(batch, length, num_kv_heads, head_dim)
    v = v.reshape(batch, length, num_kv_heads, head_dim)
    if q_norm is not None:
        q = rmsnorm(q, q_norm, eps)[0]
    if k_norm is not None:
        k = rmsnorm(k, k_norm, eps)[0]
    pos = positions.long()
    c, s = cos[pos][:, :, None], sin[pos][:, :, None]  # [B, T, 1, D/2]
    q, k = _rotate(q, c, s), _rotate(k, c, s)
    if k_cache.dtype == torch.float8_e4m3fn:
        k = (k.to(torch.bfloat16).float() / k_scale.float()[:, None]).clamp(-448, 448)
        v = (v.to(torch.bfloat16).float() / v_scale.float()[:, None]).clamp(-448, 448)
    for b in range(batch):
        n, start = min(int(n_new[b]) - q_offset, length), int(kv_len[b]) + q_offset
        if n > 0 and pages is not None:  # paged pool views [P, H_kv, 128, D]
            for i in range(n):
                page, row = _paged_slot(pages, b, start + i)
                k_cache[page, :, row] = k[b, i].to(k_cache.dtype)
                v_cache[page, :, row] = v[b, i].to(v_cache.dtype)
        elif n > 0:
            k_cache[b, :, start:start + n] = k[b, :n].transpose(0, 1).to(k_cache.dtype)
            v_cache[b, :, start:start + n] = v[b, :n].transpose(0, 1).to(v_cache.dtype)
    return q


def visible_mask(kv_len: torch.Tensor, n_new: torch.Tensor, length: int, width: int,
                 mask: torch.Tensor | None, q_offset: int = 0, window: int = 0) -> torch.Tensor:
    """Boolean ``[B, T, width]`` visibility of cache slots for the queries of a pass (see :func:`attention`).
    ``window > 0`` also hides the slots below ``position - window + 1`` (the query's position is the committed length
    plus its tree depth, or plus its index among the new tokens without a tree)."""
    vis = _visible(kv_len, n_new, length, width, mask, q_offset)
    if window > 0:
        t = torch.arange(length, device=kv_len.device)
        if mask is None:
            depth = (q_offset + t)[None, :].expand(kv_len.shape[0], length)
        else:
            ones = ((mask.long()[..., None] >> torch.arange(64, device=mask.device)) & 1).sum(-1)
            depth = (ones - 1).clamp_min(0)
        lo = kv_len.long()[:, None] + depth - window + 1  # [B, T]
        vis = vis & (torch.arange(width, device=kv_len.device)[None, None, :] >= lo[:, :, None])
    return vis


def _visible(kv_len: torch.Tensor, n_new: torch.Tensor, length: int, width: int,
             mask: torch.Tensor | None, q_offset: int = 0) -> torch.Tensor:
    device = kv_len.device
    slots = torch.arange(width, device=device)
    t = torch.arange(length, device=device)
    base = kv_len.long()[:, None, None]
    prefix = slots[None, None, :] < base  # [B, 1, W]
    j = slots[None, None, :] - base  # index of the new token in that slot
    valid_new = (j >= 0) & (j < n_new.long()[:, None, None])
    if mask is None:
        new_vis = j <= (q_offset + t)[None, :, None]
    else:
        bits = mask.long()[:, :, None]  # [B, T, 1]
        jj = j.clamp(0, 63)
        new_vis = ((bits >> jj) & 1).bool()
    return prefix | (valid_new & new_vis)


def attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, kv_len: torch.Tensor,
              n_new: torch.Tensor, mask: torch.Tensor | None = None, scale: float | None = None,
              softcap: float | None = None, q_offset: int = 0, k_scale: torch.Tensor | None = None,
              v_scale: torch.Tensor | None = None, keep: torch.Tensor | None = None,
              lse_out: torch.Tensor | None = None, kivi: torch.Tensor | None = None,
              kivi_chunks: torch.Tensor | None = None, kivi_bits: int = 0, sinks: torch.Tensor | None = None,
              window: int = 0, pages: torch.Tensor | None = None) -> torch.Tensor:
    """Attention of queries ``[B, T, H, D]`` over the slot cache ``[B, H_kv, S, D]`` (bf16, fp32, or e4m3 codes with
    per-KV-head scales ``k_scale``/``v_scale``).

    Query ``t`` of row ``b`` sees every committed slot ``< kv_len[b]`` and the new tokens' slots ``kv_len[b] + j``
    (``j < n_new[b]``) for which bit ``j`` of ``mask[b, t]`` is set (``mask=None``: causal, ``j <= q_offset + t``).
    Heads are grouped: query head ``h`` reads KV head ``h // (H / H_kv)``. ``softcap`` maps every scaled score ``s``
    to ``softcap * tanh(s / softcap)``; ``sinks [H]`` adds one logit per query head to the softmax denominator (it
    carries no value); ``window`` hides keys more than ``window - 1`` positions behind the query.
    """
    if pages is not None:  # paged pool views: read the logical caches through the page table
        k_cache, v_cache = paged_logical(k_cache, pages), paged_logical(v_cache, pages)
    batch, length, heads, dim = q.shape
    kv_heads = k_cache.shape[1]
    width = max(int((kv_len + n_new).max()), 1)
    vis = visible_mask(kv_len, n_new, length, width, mask, q_offset, window)  # [B, T, W]
    keys = k_cache[:, :, :width].float()
    values = v_cache[:, :, :width].float()
    if k_scale is not None:
        keys = keys * k_scale.float()[None, :, None, None]
        values = values * v_scale.float()[None, :, None, None]
    if kivi is not None:  # KIVI-coded chunks replace the bf16 entries of their slots
        from .kivi import dequant_chunks

        dk, dv = dequant_chunks(kivi, kivi_bits, dim)  # [B, H_kv, C, 128, D]
        for b in range(batch):
            n = int(kivi_chunks[b]) * 128
            if n:
                keys[b, :, :n] = dk[b, :, : n // 128].reshape(kv_heads, n, dim)
                values[b, :, :n] = dv[b, :, : n // 128].reshape(kv_heads, n, dim)
    group = heads // kv_heads
    keys = keys.repeat_interleave(group, 1)
    values = values.repeat_interleave(group, 1)
    scores = torch.matmul(q.float().transpose(1, 2), keys.transpose(-1, -2)) * (scale or dim ** -0.5)
    if softcap is not None:
        scores = torch.tanh(scores / softcap) * softcap
    vis = vis[:, None].expand(batch, heads, length, width)
    if keep is not None:  # evicted committed slots (bit words [B, H_kv, S / 32]) are invisible
        bits = ((keep.long()[..., None] >> torch.arange(32, device=keep.device)) & 1).bool()
        kept = bits.reshape(batch, kv_heads, -1)[..., :width].repeat_interleave(group, 1)  # [B, H, W]
        committed = torch.arange(width, device=keep.device)[None, :] < kv_len.long()[:, None]  # [B, W]
        vis = vis & (kept | ~committed[:, None])[:, :, None, :]
    scores = scores.masked_fill(~vis, float("-inf"))
    if sinks is not None:  # one extra logit per query head that joins the denominator only
        sink = sinks.float()[None, :, None, None].expand(batch, heads, length, 1)
        scores = torch.cat([scores, sink], -1)
        values = torch.cat([values, values.new_zeros(*values.shape[:2], 1, dim)], 2)
    if lse_out is not None:  # log2-domain log-sum-exp per (row, token, head), like the kernel's
        lse = torch.logsumexp(scores, -1) * 1.4426950408889634  # [B, H, T]
        lse_out.copy_(lse.transpose(1, 2))
    probs = torch.softmax(scores, -1).nan_to_num(0.0)
    out = torch.matmul(probs, values).transpose(1, 2)
    return out.to(q.dtype)


def silu_mul(gate_up: torch.Tensor) -> torch.Tensor:
    """``silu(gate) * up`` for ``gate_up = [..., 2F]`` holding the gate first (rounded like HF's Llama MLP)."""
    gate, up = gate_up.chunk(2, -1)
    return F.silu(gate) * up


def gelu_tanh_mul(gate_up: torch.Tensor) -> torch.Tensor:
    """``gelu_tanh(gate) * up`` (Gemma's GeGLU MLP, rounded like HF's)."""
    gate, up = gate_up.chunk(2, -1)
    return F.gelu(gate, approximate="tanh") * up


def clamped_swiglu(gate_up: torch.Tensor, limit: float = 7.0) -> torch.Tensor:
    """gpt-oss's gated activation of ``[gate; up]``: ``g = min(gate, limit)``, ``(clamp(up, -limit, limit) + 1) *
    g * sigmoid(1.702 g)`` (transformers ``models/gpt_oss/modeling_gpt_oss.py``, ``GptOssExperts._apply_gate``, with
    gate and up as halves instead of interleaved columns)."""
    gate, up = gate_up.chunk(2, -1)
    gate = gate.clamp(max=limit)
    up = up.clamp(-limit, limit)
    return (up + 1) * (gate * torch.sigmoid(gate * 1.702))


def glu(gate_up: torch.Tensor, act: str = "silu", limit: float = 7.0) -> torch.Tensor:
    """The gated activations of :func:`economize_b200.ops.glu` in plain PyTorch (any device and dtype)."""
    if act == "silu":
        return silu_mul(gate_up)
    if act == "gelu_tanh":
        return gelu_tanh_mul(gate_up)
    if act == "clamped_swiglu":
        return clamped_swiglu(gate_up, limit)
    raise ValueError(f"unsupported gated activation {act!r}")


def vs_keep(cols: torch.Tensor, offsets: torch.Tensor, base: int, t: int, limit: int, size: int) -> torch.Tensor:
    """MInference's vertical-slash pattern as keep bit words ``int32 [..., size / 32]``: key ``j < limit`` is kept
    when it is one of ``cols`` or lies in ``[base - o, base + t - o)`` for a diagonal offset ``o`` of ``offsets``.
    The diagonals' union is a difference array and a prefix sum (memory ``O(size)``, not ``O(ns * size)``)."""
    lead = cols.shape[:-1]
    rows = 1
    for n in lead:
        rows *= n
    cols2, offs = cols.reshape(rows, cols.shape[-1]), offsets.reshape(rows, offsets.shape[-1])
    diff = torch.zeros(rows, size + 1, dtype=torch.int32, device=cols.device)
    ones = torch.ones_like(offs, dtype=torch.int32)
    diff.scatter_add_(1, (base - offs).clamp(0, size), ones)
    diff.scatter_add_(1, (base + t - offs).clamp(0, size), -ones)
    keep = diff.cumsum(1)[:, :size] > 0
    valid = (cols2 >= 0) & (cols2 < size)
    keep.scatter_(1, cols2.clamp(0, size - 1), valid | keep.gather(1, cols2.clamp(0, size - 1)))
    keep &= torch.arange(size, device=cols.device)[None] < limit
    bits = keep.reshape(rows, size // 32, 32).to(torch.int64)
    words = (bits << torch.arange(32, device=cols.device)).sum(-1)
    return torch.where(words >= 2 ** 31, words - 2 ** 32, words).to(torch.int32).reshape(*lead, size // 32)


def hadamard(x: torch.Tensor, block: int) -> torch.Tensor:
    """``x H_b / sqrt(b)`` over consecutive blocks of ``block`` (a power of two) of the last dimension, with ``H_b``
    the Sylvester matrix: the fast Walsh-Hadamard transform in fp32, butterflies of half-width 1, 2, 4, ... (the
    order of the CUDA kernel), rounded once to ``x``'s dtype."""
    if block < 1 or block & (block - 1) or x.shape[-1] % block:
        raise ValueError(f"hadamard block {block} must be a power of two dividing the width {x.shape[-1]}")
    work = x.float().reshape(-1, block)
    h = 1
    while h < block:
        pairs = work.view(-1, block // (2 * h), 2, h)
        a, b = pairs[:, :, 0], pairs[:, :, 1]
        work = torch.stack((a + b, a - b), dim=2).reshape(-1, block)
        h *= 2
    return (work * block ** -0.5).reshape(x.shape).to(x.dtype)


def linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None) -> torch.Tensor:
    return F.linear(x, weight, bias)


def greedy_accept(tokens: torch.Tensor, parents: torch.Tensor, pred: torch.Tensor, ok: torch.Tensor | None = None
                  ) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Longest accepted path of a verified draft tree.

    Args:
        tokens: ``[B, T]`` tokens of the pass: node 0 is the root (the last committed token), nodes ``1..T-1`` the
            drafts in topological order.
        parents: ``[B, T]`` parent node of every node (``parents[:, 0]`` is ignored); a chain has ``parents[t] = t-1``.
        pred: ``[B, T]`` the exact model's choice after every node.
        ok: optional ``[B, T]`` bools replacing the match rule: node ``t`` is acceptable given its parent.

    Returns:
        ``n_acc [B]`` accepted drafts, ``path [B, T]`` node index of the path's ``i``-th node (``path[:, 0] = 0``,
        entries past ``n_acc`` repeat the last node), and ``out [B, T]`` the tokens the cycle commits after the root:
        the path's draft tokens followed by the bonus token ``pred[last node]``.
    """
    batch, length = tokens.shape
    device = tokens.device
    acc = torch.zeros(batch, length, dtype=torch.bool, device=device)
    depth = torch.zeros(batch, length, dtype=torch.long, device=device)
    acc[:, 0] = True
    for t in range(1, length):
        p = parents[:, t].long().clamp_min(0)
        par_acc = acc.gather(1, p[:, None])[:, 0]
        match = ok[:, t].bool() if ok is not None else tokens[:, t] == pred.gather(1, p[:, None])[:, 0]
        acc[:, t] = par_acc & match & (parents[:, t] >= 0)
        depth[:, t] = depth.gather(1, p[:, None])[:, 0] + 1
    score = torch.where(acc, depth, torch.full_like(depth, -1))
    # deepest accepted node, first one on ties
    best_depth = score.max(1).values
    idx = torch.arange(length, device=device)[None].expand(batch, length)
    best = torch.where(score == best_depth[:, None], idx, torch.full_like(idx, length)).min(1).values
    n_acc = best_depth
    path = torch.zeros(batch, length, dtype=torch.long, device=device)
    out = torch.zeros(batch, length, dtype=tokens.dtype, device=device)
    for b in range(batch):
        node, chain = int(best[b]), []
        while node > 0:
            chain.append(node)
            node = int(parents[b, node])
        chain = chain[::-1]
        nodes = [0, *chain]
        for i, n in enumerate(nodes):
            path[b, i] = n
        for i in range(len(nodes), length):
            path[b, i] = nodes[-1]
        for i, n in enumerate(chain):
            out[b, i] = tokens[b, n]
        out[b, len(chain)] = pred[b, nodes[-1]]
    return n_acc.to(torch.int32), path.to(torch.int32), out


def kv_compact(cache: torch.Tensor, kv_len: torch.Tensor, path: torch.Tensor, n_acc: torch.Tensor,
               pages: torch.Tensor | None = None) -> None:
    """Move the cache entries of an accepted tree path to consecutive slots: slot ``kv_len + path[b, i]`` to
    ``kv_len + i`` for ``i <= n_acc[b]``, in every layer of ``cache [L, 2, B, H_kv, S, D]`` (or of a page pool
    ``[P, 2, H_kv, 128, D]`` with page tables ``pages [L, B, C]``)."""
    if cache.dtype == torch.float8_e4m3fn:
        cache = cache.view(torch.uint8)
    if pages is not None:
        for layer in range(pages.shape[0]):
            for b in range(pages.shape[1]):
                n, base = int(n_acc[b]), int(kv_len[b])
                src = [_paged_slot(pages[layer], b, base + int(p)) for p in path[b, : n + 1]]
                moved = [cache[page, :, :, row].clone() for page, row in src]
                for i, value in enumerate(moved):
                    page, row = _paged_slot(pages[layer], b, base + i)
                    cache[page, :, :, row] = value
        return
    for b in range(cache.shape[2]):
        n, base = int(n_acc[b]), int(kv_len[b])
        src = base + path[b, : n + 1].long()
        moved = cache[:, :, b, :, src].clone()
        cache[:, :, b, :, base:base + n + 1] = moved


def _draw(weights: torch.Tensor, u: float) -> int:
    total = float(weights.sum())
    if total <= 0:
        return -1
    cdf = torch.cumsum(weights.double(), 0)
    idx = int(torch.searchsorted(cdf, torch.tensor([u * float(cdf[-1])], dtype=torch.float64), right=True))
    idx = min(idx, weights.numel() - 1)
    while idx > 0 and weights[idx] <= 0:
        idx -= 1
    return idx


def sample(probs: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    """One token per row of ``probs [..., V]`` by inverse CDF at ``u [...]``."""
    flat = probs.reshape(-1, probs.shape[-1])
    out = [max(_draw(flat[i], float(u.reshape(-1)[i])), 0) for i in range(flat.shape[0])]
    return torch.tensor(out, dtype=torch.int64, device=probs.device).reshape(probs.shape[:-1])


def rejection(p: torch.Tensor, q: torch.Tensor, drafts: torch.Tensor, u_acc: torch.Tensor,
              u_draw: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Lossless speculative sampling of draft chains (see ``csrc/sampling.cu``): ``n_acc [B]`` and ``out [B, k+1]``
    (accepted drafts, then the correction or bonus token)."""
    batch, k = drafts.shape
    n_acc = torch.zeros(batch, dtype=torch.int32, device=p.device)
    out = torch.zeros(batch, k + 1, dtype=torch.int64, device=p.device)
    for b in range(batch):
        j = 0
        while j < k:
            x = int(drafts[b, j])
            if not float(u_acc[b, j]) * float(q[b, j, x]) < float(p[b, j, x]):
                break
            out[b, j] = x
            j += 1
        if j < k:
            tok = _draw((p[b, j] - q[b, j]).clamp_min(0), float(u_draw[b]))
            if tok < 0:
                tok = _draw(p[b, j], float(u_draw[b]))
        else:
            tok = _draw(p[b, k], float(u_draw[b]))
        out[b, j] = max(tok, 0)
        n_acc[b] = j
    return n_acc, out


def ngram(history: torch.Tensor, length: torch.Tensor, k: int, min_n: int, max_n: int,
          earliest: bool = True) -> torch.Tensor:
    """Prompt-lookup proposals ``[B, k]`` (see ``csrc/ngram.cu``): the ``k`` tokens after an earlier occurrence
    of the history's last ``n`` tokens, longest ``n`` first; ``-1`` where there is none."""
    batch = history.shape[0]
    out = torch.full((batch, k), -1, dtype=torch.int64, device=history.device)
    for b in range(batch):
        n_hist = min(int(length[b]), history.shape[1])
        h = history[b, :n_hist].tolist()
        for n in range(max_n, min_n - 1, -1):
            if n_hist <= n:
                continue
            pattern = h[n_hist - n:]
            starts = [i for i in range(0, n_hist - n) if h[i:i + n] == pattern]
            if starts:
                i = starts[0] if earliest else starts[-1]
                for j in range(k):
                    if i + n + j < n_hist:
                        out[b, j] = h[i + n + j]
                break
    return out


def attention_scores(q: torch.Tensor, k_cache: torch.Tensor, kv_len: torch.Tensor, n_new: torch.Tensor,
                     mask: torch.Tensor | None, lse2: torch.Tensor, scores: torch.Tensor, scale: float,
                     q_offset: int = 0, pages: torch.Tensor | None = None) -> None:
    """``scores [B, H_kv, S] +=`` the attention probability mass every visible slot receives from the queries
    ``q [B, T, H, D]`` (probabilities ``exp2(s * scale * log2 e - lse2)``), summed over each KV head's group."""
    if pages is not None:
        k_cache = paged_logical(k_cache, pages)
    batch, length, heads, dim = q.shape
    kv_heads, width = k_cache.shape[1], scores.shape[-1]
    group = heads // kv_heads
    vis = visible_mask(kv_len, n_new, length, width, mask, q_offset)
    keys = k_cache[:, :, :width].float().repeat_interleave(group, 1)
    s = torch.matmul(q.float().transpose(1, 2), keys.transpose(-1, -2)) * scale * 1.4426950408889634
    p = torch.exp2(s - lse2.float().transpose(1, 2)[..., None]).masked_fill(~vis[:, None], 0.0)
    scores += p.sum(2).reshape(batch, kv_heads, group, width).sum(2)


def kivi_quantize(cache: torch.Tensor, kivi: torch.Tensor, kv_len: torch.Tensor, chunks: torch.Tensor, bits: int,
                  residual: int, max_new: int, pages: torch.Tensor | None = None) -> None:
    """Code the committed chunks ``chunks[b] .. `` of ``cache [L, 2, B, H_kv, S, D]`` that lie at least
    ``residual`` slots behind ``kv_len[b]`` (at most ``max_new`` per row) into ``kivi [L, B, H_kv, S/128, bytes]``
    (a page pool ``[P, 2, H_kv, 128, D]`` with tables ``pages [L, B, C]`` is read through them)."""
    from .kivi import pack_chunks

    if pages is not None:
        cache = torch.stack([torch.stack([paged_logical(cache[:, kv], pages[layer]) for kv in (0, 1)])
                             for layer in range(pages.shape[0])])

    for b in range(cache.shape[2]):
        ready = max(0, (int(kv_len[b]) - residual) // 128)
        start = int(chunks[b])
        stop = min(ready, start + max_new)
        for c in range(start, stop):
            k = cache[:, 0, b, :, c * 128:(c + 1) * 128]
            v = cache[:, 1, b, :, c * 128:(c + 1) * 128]
            kivi[:, b, :, c] = pack_chunks(k, v, bits)
        chunks[b] = max(start, stop)
