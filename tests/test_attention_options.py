"""Semantics of the attention options in the fp32 reference (the oracle of the CUDA kernel's tests), checked
against direct formulas: sliding windows hide keys more than ``window - 1`` positions behind the query (tree
queries sit at the committed length plus their depth), sinks add one logit per head to the denominator only, and
the soft-cap maps every scaled score through ``cap * tanh(s / cap)``."""

import math

import torch

from economize_b200.ops import reference as ref


def _inputs(B=2, T=5, H=4, Hkv=2, S=64, D=16, seed=0):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, T, H, D, generator=g)
    k = torch.randn(B, Hkv, S, D, generator=g)
    v = torch.randn(B, Hkv, S, D, generator=g)
    return q, k, v


def _brute(q, k, v, vis, scale, softcap=None, sinks=None):
    B, T, H, D = q.shape
    G = H // k.shape[1]
    out = torch.zeros(B, T, H, D)
    for b in range(B):
        for t in range(T):
            for h in range(H):
                idx = vis[b, t].nonzero().flatten()
                s = (k[b, h // G, idx] @ q[b, t, h]) * scale
                if softcap:
                    s = softcap * torch.tanh(s / softcap)
                w = torch.exp(s - s.max()) if len(idx) else s
                denom = w.sum()
                if sinks is not None:
                    denom = denom + math.exp(float(sinks[h]) - float(s.max()))
                out[b, t, h] = (w[:, None] * v[b, h // G, idx]).sum(0) / denom
    return out


def test_causal_window_and_softcap():
    q, k, v = _inputs()
    kv_len = torch.tensor([20, 3], dtype=torch.int32)
    n_new = torch.tensor([5, 5], dtype=torch.int32)
    got = ref.attention(q, k, v, kv_len, n_new, None, softcap=2.0, window=6)
    pos = kv_len.long()[:, None] + torch.arange(5)[None]  # [B, T] positions
    slots = torch.arange(int((kv_len + n_new).max()))
    vis = (slots[None, None] <= pos[..., None]) & (slots[None, None] > pos[..., None] - 6)
    want = _brute(q, k, v, vis, 16 ** -0.5, softcap=2.0)
    torch.testing.assert_close(got, want, atol=1e-5, rtol=1e-5)


def test_tree_window_uses_depth_and_sinks():
    q, k, v = _inputs(B=1, T=4)
    kv_len = torch.tensor([30], dtype=torch.int32)
    n_new = torch.tensor([4], dtype=torch.int32)
    # tree: 0 root; 1, 2 children of 0; 3 child of 1 (depths 0, 1, 1, 2)
    bits = [0b1, 0b11, 0b101, 0b1011]
    mask = torch.tensor([bits], dtype=torch.int64)
    sinks = torch.tensor([0.5, -1.0, 2.0, 0.0])
    got = ref.attention(q, k, v, kv_len, n_new, mask, sinks=sinks, window=10)
    vis = torch.zeros(1, 4, 34, dtype=torch.bool)
    for t, (d, b) in enumerate(zip((0, 1, 1, 2), bits)):
        lo = 30 + d - 10 + 1
        vis[0, t, max(lo, 0):30] = True
        for j in range(4):
            vis[0, t, 30 + j] = bool((b >> j) & 1)
    want = _brute(q, k, v, vis, 16 ** -0.5, sinks=sinks)
    torch.testing.assert_close(got, want, atol=1e-5, rtol=1e-5)


def test_sink_lse_and_no_visible_key():
    q, k, v = _inputs(B=1, T=1)
    kv_len = torch.tensor([0], dtype=torch.int32)
    n_new = torch.tensor([1], dtype=torch.int32)
    sinks = torch.zeros(4)
    lse = torch.empty(1, 1, 4)
    out = ref.attention(q, k, v, kv_len, n_new, None, sinks=sinks, lse_out=lse)
    s = (k[0, torch.arange(4) // 2, 0] * q[0, 0]).sum(-1) * 16 ** -0.5  # each head's one score
    torch.testing.assert_close(lse[0, 0], torch.logaddexp(s, torch.zeros(4)) / math.log(2))
    w = torch.exp(s) / (torch.exp(s) + 1)
    torch.testing.assert_close(out[0, 0], w[:, None] * v[0, torch.arange(4) // 2, 0])
