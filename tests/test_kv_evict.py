"""KV eviction: keep masks hide exactly the evicted slots, every policy keeps its budget, decoding stays lossless
for the evicted model, and the tensor-core scores match the PyTorch reference."""

import pytest
import torch

import economize_b200 as eco
from economize_b200 import ops
from economize_b200.ops import reference as ref
from economize_b200.techniques.eagle3 import Eagle3Config
from economize_b200.techniques.kv_evict import KVEvictConfig, keep_words

from .helpers import gpu_tiny_model, prompts, reference_greedy, tiny_model


def test_keep_words_roundtrip():
    keep = torch.rand(2, 3, 64) > 0.5
    w = keep_words(keep)
    bits = ((w.long()[..., None] >> torch.arange(32)) & 1).bool().reshape(2, 3, 64)
    assert torch.equal(bits, keep)


def test_keep_mask_equals_attention_over_kept_keys():
    g = torch.Generator().manual_seed(0)
    B, T, H, Hkv, D, S = 1, 3, 4, 2, 16, 64
    q = torch.randn(B, T, H, D, generator=g)
    k = torch.randn(B, Hkv, S, D, generator=g)
    v = torch.randn(B, Hkv, S, D, generator=g)
    kv_len, n_new = torch.tensor([20], dtype=torch.int32), torch.tensor([T], dtype=torch.int32)
    keep = torch.ones(B, Hkv, S, dtype=torch.bool)
    keep[:, :, 5:12] = False
    out = ref.attention(q, k, v, kv_len, n_new, None, keep=keep_words(keep))
    sel = torch.tensor([i for i in range(S) if not 5 <= i < 12])
    out2 = ref.attention(q, k[:, :, sel], v[:, :, sel], kv_len - 7, n_new, None)
    torch.testing.assert_close(out, out2)


def test_reference_scores_sum_to_query_count():
    g = torch.Generator().manual_seed(1)
    B, T, H, Hkv, D, S = 1, 4, 4, 2, 16, 32
    q = torch.randn(B, T, H, D, generator=g)
    k = torch.randn(B, Hkv, S, D, generator=g)
    kv_len, n_new = torch.zeros(1, dtype=torch.int32), torch.tensor([10], dtype=torch.int32)
    lse = torch.empty(B, T, H)
    ref.attention(q, k, k, kv_len, n_new, None, lse_out=lse, q_offset=6)
    scores = torch.zeros(B, Hkv, S)
    ref.attention_scores(q, k, kv_len, n_new, None, lse, scores, D ** -0.5, q_offset=6)
    # every query row distributes probability 1 over its visible keys; a KV head serves T x G rows
    torch.testing.assert_close(scores.sum(-1), torch.full((1, 2), float(T * H // Hkv)))


@pytest.mark.parametrize("method", ["streaming", "h2o", "snapkv", "pyramidkv"])
def test_eviction_policies(method):
    model = tiny_model()
    eff = eco.apply(model, KVEvictConfig(method=method, budget=16, window=4), Eagle3Config(),
                    decoding=eco.DecodeConfig(cycle_length=4))
    p = prompts((40,))[0]
    out = eff.decode(p, 8)
    tech = eff.techniques["kv_evict"]
    frac = tech.kept_fraction(torch.tensor([40]))
    if method == "pyramidkv":
        assert 0.2 < frac < 0.6
    else:
        assert abs(frac - 16 / 40) < 0.03
    # lossless with respect to the evicted model: speculative output equals its own plain decoding
    plain = eff.decode(p, 8, decoding=eco.DecodeConfig(cycle_length=1))
    assert torch.equal(out.tokens, plain.tokens)


@pytest.mark.gpu
def test_scores_kernel_matches_reference(cuda):
    g = torch.Generator(device=cuda).manual_seed(0)
    B, T, H, Hkv, D, S = 2, 32, 8, 2, 128, 512
    q = torch.randn(B, T, H, D, device=cuda, generator=g).bfloat16()
    k = torch.randn(B, Hkv, S, D, device=cuda, generator=g).bfloat16()
    kv_len = torch.zeros(B, dtype=torch.int32, device=cuda)
    n_new = torch.tensor([300, 400], dtype=torch.int32, device=cuda)
    lse = torch.empty(B, T, H, device=cuda)
    ops.attention(q, k, k, kv_len, n_new, None, lse_out=lse, q_offset=268)
    lse_ref = torch.empty_like(lse)
    ref.attention(q.float(), k.float(), k.float(), kv_len, n_new, None, lse_out=lse_ref, q_offset=268)
    torch.testing.assert_close(lse, lse_ref, atol=2e-2, rtol=1e-3)
    s1 = torch.zeros(B, Hkv, S, device=cuda)
    ops.attention_scores(q, k, kv_len, n_new, None, lse, s1, q_offset=268)
    s2 = torch.zeros_like(s1)
    ref.attention_scores(q.float(), k.float(), kv_len, n_new, None, lse_ref, s2, D ** -0.5, q_offset=268)
    torch.testing.assert_close(s1, s2, atol=2e-3, rtol=3e-2)


@pytest.mark.gpu
def test_eviction_on_gpu_is_lossless(cuda):
    model = gpu_tiny_model(cuda)
    eff = eco.apply(model, KVEvictConfig(method="snapkv", budget=64, window=16), Eagle3Config(),
                    decoding=eco.DecodeConfig(cycle_length=4))
    p = prompts((200,))[0].to(cuda)
    plain = eff.decode(p, 12, decoding=eco.DecodeConfig(cycle_length=1)).tokens
    assert torch.equal(eff.decode(p, 12).tokens.cpu(), plain.cpu())
