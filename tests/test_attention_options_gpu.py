"""Attention options on the tcgen05 kernel against the fp32 PyTorch reference of the same op: tanh soft-capped scores
(Gemma-2), sink logits (gpt-oss), sliding windows (the kernel walks only the window's chunks), and head dimension
256 (Gemma), in tree, causal-prefill and exact-tail passes; a windowed tree pass still equals one-token passes bit for
bit; the GeGLU activation kernel."""

import pytest
import torch

from economize_b200 import ops
from economize_b200.ops import reference as ref

pytestmark = pytest.mark.gpu


def _tree_bits(T, gc):
    """A random topological tree: (int64 ancestor bit words, parents)."""
    bits, parents = [1], [-1]
    for t in range(1, T):
        p = int(torch.randint(0, t, (1,), generator=gc))
        parents.append(p)
        bits.append(bits[p] | (1 << t))
    return [b if b < 2**63 else b - 2**64 for b in bits], parents


def _inputs(B, T, H, Hkv, S, D, dev, seed):
    g = torch.Generator(device=dev).manual_seed(seed)
    k = torch.randn(B, Hkv, S, D, device=dev, generator=g).bfloat16()
    v = torch.randn(B, Hkv, S, D, device=dev, generator=g).bfloat16()
    q = (2.0 * torch.randn(B, T, H, D, device=dev, generator=g)).bfloat16()
    sinks = torch.randn(H, device=dev, generator=g) * 2.0
    return q, k, v, sinks


@pytest.mark.parametrize("D", [64, 128, 256])
@pytest.mark.parametrize("opts", [dict(softcap=5.0), dict(sinks=True), dict(window=100),
                                  dict(softcap=3.0, sinks=True, window=80), dict()])
@pytest.mark.parametrize("tail", [0, 16])
def test_tree_pass_options(cuda, D, opts, tail):
    B, T, H, Hkv, S = 2, 61, 8, 2, 1024
    q, k, v, sinks = _inputs(B, T, H, Hkv, S, D, cuda, D + tail)
    gc = torch.Generator().manual_seed(D)
    mask = torch.tensor([_tree_bits(T, gc)[0] for _ in range(B)], device=cuda)
    kv_len = torch.tensor([700, 90], dtype=torch.int32, device=cuda)
    n_new = torch.full((B,), T, dtype=torch.int32, device=cuda)
    kw = dict(softcap=opts.get("softcap"), sinks=sinks if opts.get("sinks") else None, window=opts.get("window", 0))
    lse = torch.empty(B, T, H, device=cuda)
    out = ops.attention(q, k, v, kv_len, n_new, mask, tail=tail, lse_out=lse, **kw)
    lse_ref = torch.empty(B, T, H, device=cuda)
    want = ref.attention(q.float(), k.float(), v.float(), kv_len, n_new, mask, lse_out=lse_ref, **kw)
    torch.testing.assert_close(out.float(), want.float(), atol=3e-2, rtol=3e-2)
    torch.testing.assert_close(lse, lse_ref, atol=2e-2, rtol=1e-3)
    assert ops.require().status(0) == 0


@pytest.mark.parametrize("D", [128, 256])
@pytest.mark.parametrize("window", [0, 40, 300])
def test_causal_prefill_window(cuda, D, window):
    B, T, H, Hkv = 2, 400, 8, 2
    S = 512
    q, k, v, _ = _inputs(B, T, H, Hkv, S, D, cuda, window + 1)
    kv_len = torch.zeros(B, dtype=torch.int32, device=cuda)
    n_new = torch.tensor([400, 233], dtype=torch.int32, device=cuda)
    out = ops.attention(q, k, v, kv_len, n_new, None, window=window, softcap=20.0 if window else None)
    want = ref.attention(q.float(), k.float(), v.float(), kv_len, n_new, None, window=window,
                         softcap=20.0 if window else None)
    for b, n in enumerate((400, 233)):
        torch.testing.assert_close(out[b, :n].float(), want[b, :n].float(), atol=3e-2, rtol=3e-2)
    assert ops.require().status(0) == 0


@pytest.mark.parametrize("D,window", [(128, 100), (256, 0), (256, 130)])
def test_windowed_tree_pass_equals_one_token_passes(cuda, D, window):
    """Exact tail with a window and a soft-cap: every node of a tree pass has the bits of a one-token pass at its
    position (the key split is planned on absolute chunk groups, the same for both passes)."""
    B, T, H, Hkv, S, base = 1, 40, 8, 2, 2048, 900
    q, k, v, sinks = _inputs(B, T, H, Hkv, S, D, cuda, 7)
    gc = torch.Generator().manual_seed(11)
    signed, parents = _tree_bits(T, gc)
    mask = torch.tensor([signed], device=cuda)
    kv_len = torch.tensor([base], dtype=torch.int32, device=cuda)
    n_new = torch.tensor([T], dtype=torch.int32, device=cuda)
    kw = dict(softcap=30.0, sinks=sinks, window=window)
    tree = ops.attention(q, k, v, kv_len, n_new, mask, tail=16, **kw)
    for node in range(T):
        path, n = [], node
        while n >= 0:
            path.append(n)
            n = parents[n]
        path.reverse()
        k2, v2 = k.clone(), v.clone()
        for depth, n in enumerate(path):
            k2[:, :, base + depth] = k[:, :, base + n]
            v2[:, :, base + depth] = v[:, :, base + n]
        one = ops.attention(q[:, node:node + 1].contiguous(), k2, v2,
                            torch.tensor([base + len(path) - 1], dtype=torch.int32, device=cuda),
                            torch.ones(1, dtype=torch.int32, device=cuda), None, tail=16, **kw)
        assert torch.equal(one[:, 0], tree[:, node]), node


def test_head_dim_256_plain_decode_and_splits(cuda):
    """One-token decode over a long cache (many key splits) and a short one (one split), D = 256."""
    B, T, H, Hkv, S, D = 3, 1, 8, 4, 4096, 256
    q, k, v, _ = _inputs(B, T, H, Hkv, S, D, cuda, 5)
    kv_len = torch.tensor([4000, 3, 1200], dtype=torch.int32, device=cuda)
    n_new = torch.ones(B, dtype=torch.int32, device=cuda)
    out = ops.attention(q, k, v, kv_len, n_new, None)
    want = ref.attention(q.float(), k.float(), v.float(), kv_len, n_new, None)
    torch.testing.assert_close(out.float(), want.float(), atol=3e-2, rtol=3e-2)


def test_window_refused_below_tree_depth(cuda):
    B, T, H, Hkv, S, D = 1, 8, 4, 2, 256, 128
    q, k, v, _ = _inputs(B, T, H, Hkv, S, D, cuda, 1)
    mask = torch.tensor([_tree_bits(T, torch.Generator().manual_seed(0))[0]], device=cuda)
    one = torch.ones(1, dtype=torch.int32, device=cuda)
    with pytest.raises(RuntimeError, match="window"):
        ops.attention(q, k, v, one * 100, one * T, mask, window=32)


def test_gelu_tanh_mul(cuda):
    g = torch.Generator(device=cuda).manual_seed(0)
    gu = (3 * torch.randn(37, 2 * 688, device=cuda, generator=g)).bfloat16()
    out = ops.gelu_tanh_mul(gu)
    want = ref.gelu_tanh_mul(gu)  # the same bf16 rounding steps in torch
    torch.testing.assert_close(out.float(), want.float(), atol=2e-2, rtol=1e-2)
    exact = ref.gelu_tanh_mul(gu.float())
    torch.testing.assert_close(out.float(), exact, atol=6e-2, rtol=2e-2)
