"""Exact-tail attention: a tree verification pass computes every node bit for bit as a one-token pass at the same
position does, which is what makes greedy speculative decoding reproduce plain greedy decoding exactly."""

import pytest
import torch

from economize_b200 import ops
from economize_b200.ops import reference as ref

pytestmark = pytest.mark.gpu


def _tree(T, g):
    """A random topological tree: parents[t] < t, bits = ancestors + self."""
    parents, bits = [-1], [1]
    for t in range(1, T):
        p = int(torch.randint(0, t, (1,), generator=g))
        parents.append(p)
        bits.append(bits[p] | (1 << t))
    return parents, bits


def _as_i64(bits):
    return [b if b < 2**63 else b - 2**64 for b in bits]


def _caches(fp8, B, Hkv, S, D, dev, g):
    k = torch.randn(B, Hkv, S, D, device=dev, generator=g)
    v = torch.randn(B, Hkv, S, D, device=dev, generator=g)
    if not fp8:
        return k.bfloat16(), v.bfloat16(), None, None
    ks = torch.rand(Hkv, device=dev, generator=g) * 0.02 + 0.01
    vs = torch.rand(Hkv, device=dev, generator=g) * 0.02 + 0.01
    kq = (k / ks[None, :, None, None]).to(torch.float8_e4m3fn)
    vq = (v / vs[None, :, None, None]).to(torch.float8_e4m3fn)
    return kq, vq, ks, vs


@pytest.mark.parametrize("fp8,D", [(False, 128), (True, 128), (False, 64)])
@pytest.mark.parametrize("base", [5, 250, 700])
def test_tree_pass_equals_one_token_passes(cuda, fp8, D, base):
    g = torch.Generator(device=cuda).manual_seed(base)
    gc = torch.Generator().manual_seed(base)
    B, T, H, Hkv, S = 1, 61, 32, 8, 1024
    k, v, ks, vs = _caches(fp8, B, Hkv, S, D, cuda, g)
    q = torch.randn(B, T, H, D, device=cuda, generator=g).bfloat16()
    parents, bits = _tree(T, gc)
    mask = torch.tensor([_as_i64(bits)], device=cuda)
    kv_len = torch.tensor([base], dtype=torch.int32, device=cuda)
    n_new = torch.tensor([T], dtype=torch.int32, device=cuda)
    tree_out = ops.attention(q, k, v, kv_len, n_new, mask, k_scale=ks, v_scale=vs, tail=16)
    want = ref.attention(q.float(), (k.float() * ks[None, :, None, None]) if fp8 else k.float(),
                         (v.float() * vs[None, :, None, None]) if fp8 else v.float(), kv_len, n_new, mask)
    torch.testing.assert_close(tree_out.float(), want.float(), atol=3e-2, rtol=3e-2)
    for node in range(T):
        path = []
        n = node
        while n >= 0:
            path.append(n)
            n = parents[n]
        path.reverse()  # root .. node, one per depth
        d = len(path) - 1
        k2, v2 = k.clone(), v.clone()
        for depth, n in enumerate(path):  # the accepted path at consecutive slots, as plain decoding writes it
            k2[:, :, base + depth] = k[:, :, base + n]
            v2[:, :, base + depth] = v[:, :, base + n]
        one = ops.attention(q[:, node:node + 1].contiguous(), k2, v2,
                            torch.tensor([base + d], dtype=torch.int32, device=cuda),
                            torch.ones(1, dtype=torch.int32, device=cuda), None, k_scale=ks, v_scale=vs, tail=16)
        assert torch.equal(one[:, 0], tree_out[:, node]), (node, d)


def test_tail_with_lse_and_causal(cuda):
    g = torch.Generator(device=cuda).manual_seed(3)
    B, T, H, Hkv, S, D = 2, 5, 8, 2, 512, 128
    k = torch.randn(B, Hkv, S, D, device=cuda, generator=g).bfloat16()
    v = torch.randn(B, Hkv, S, D, device=cuda, generator=g).bfloat16()
    q = torch.randn(B, T, H, D, device=cuda, generator=g).bfloat16()
    kv_len = torch.tensor([130, 9], dtype=torch.int32, device=cuda)
    n_new = torch.tensor([T, T], dtype=torch.int32, device=cuda)
    lse = torch.empty(B, T, H, device=cuda)
    lse_ref = torch.empty(B, T, H, device=cuda)
    out = ops.attention(q, k, v, kv_len, n_new, None, tail=16, lse_out=lse)
    want = ops.attention(q, k, v, kv_len, n_new, None, lse_out=lse_ref)
    torch.testing.assert_close(out.float(), want.float(), atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(lse, lse_ref, atol=1e-3, rtol=1e-4)
    assert ops.require().status(0) == 0


@pytest.mark.parametrize("T,lens", [(1, [300, 17]), (40, [129, 0]), (61, [700, 64])])
def test_head_dim_64_attention(cuda, T, lens):
    g = torch.Generator(device=cuda).manual_seed(T)
    gc = torch.Generator().manual_seed(T)
    B, H, Hkv, S, D = 2, 8, 2, 1024, 64
    k = torch.randn(B, Hkv, S, D, device=cuda, generator=g).bfloat16()
    v = torch.randn(B, Hkv, S, D, device=cuda, generator=g).bfloat16()
    q = torch.randn(B, T, H, D, device=cuda, generator=g).bfloat16()
    kv_len = torch.tensor(lens, dtype=torch.int32, device=cuda)
    n_new = torch.full((B,), T, dtype=torch.int32, device=cuda)
    mask = torch.tensor([_as_i64(_tree(T, gc)[1]) for _ in range(B)], device=cuda) if T > 1 else None
    for tail in (0, 16):
        out = ops.attention(q, k, v, kv_len, n_new, mask, tail=tail)
        want = ref.attention(q.float(), k.float(), v.float(), kv_len, n_new, mask)
        torch.testing.assert_close(out.float(), want.float(), atol=3e-2, rtol=3e-2)


def test_head_dim_64_model_tree_equals_plain(cuda):
    """A model with 64-dimensional heads (the Llama-3.2-1B / Qwen2.5-0.5B shape) through the engine."""
    import economize_b200 as eco
    from economize_b200.models.config import tiny_llama
    from economize_b200.models.llama import CausalLM, init_weights
    from economize_b200.techniques.eagle3 import Eagle3Config

    cfg = tiny_llama(hidden_size=512, num_heads=8, num_kv_heads=2, head_dim=64, num_layers=3)
    em = eco.apply(init_weights(CausalLM(cfg, torch.bfloat16, cuda), seed=0), Eagle3Config())
    ps = [torch.randint(0, cfg.vocab_size, (n,), generator=torch.Generator().manual_seed(n)).to(cuda)
          for n in (17, 140)]
    plain = em.decode_batch(ps, 24, decoding=eco.DecodeConfig(cycle_length=1))
    tree = em.decode_batch(ps, 24, decoding=eco.DecodeConfig(
        cycle_length=7, draft_policy="dynamic_tree", draft_policy_options={"depth": 6, "topk": 10, "total_tokens": 60},
        cuda_graphs=True))
    for a, b in zip(plain, tree):
        assert torch.equal(a.tokens, b.tokens)
    assert ops.require().status(0) == 0
