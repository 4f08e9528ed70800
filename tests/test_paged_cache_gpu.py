"""Paged KV caches on the CUDA kernels: attention (tree, causal prefill, exact tail, fp8 codes), the rotary store,
KV compaction and KIVI coding read and write through per-layer page tables and give the contiguous cache's bits;
ring caches of sliding-window layers decode exactly as the contiguous cache does, with tree == plain decoding."""

import pytest
import torch

import economize_b200 as eco
from economize_b200 import ops
from economize_b200.models.config import tiny_llama
from economize_b200.models.llama import CausalLM, init_weights
from economize_b200.ops import reference as ref
from economize_b200.runtime.cache import PagedKVCache
from economize_b200.techniques.eagle3 import Eagle3Config
from economize_b200.techniques.kv_quant import KIVIConfig

pytestmark = pytest.mark.gpu


def _tree_bits(T, gc):
    bits = [1]
    for t in range(1, T):
        p = int(torch.randint(0, t, (1,), generator=gc))
        bits.append(bits[p] | (1 << t))
    return [b if b < 2**63 else b - 2**64 for b in bits]


def _paged_copy(flat_k, flat_v, dev, fp8=False):
    """A one-layer paged cache holding the same keys as ``flat [B, Hkv, S, D]``, pages in shuffled order."""
    B, Hkv, S, D = flat_k.shape
    cache = PagedKVCache(1, B, Hkv, S, D, flat_k.dtype, dev)
    perm = torch.randperm(cache.num_pages, generator=torch.Generator().manual_seed(3)).to(torch.int32).to(dev)
    cache.tables[0] = perm.reshape(B, -1)
    k, v = cache.layer(0)
    for b in range(B):
        for c in range(S // 128):
            page = int(cache.tables[0, b, c])
            k[page] = flat_k[b, :, c * 128:(c + 1) * 128]
            v[page] = flat_v[b, :, c * 128:(c + 1) * 128]
    return cache


@pytest.mark.parametrize("D", [64, 128, 256])
@pytest.mark.parametrize("tail", [0, 16])
def test_paged_attention_equals_contiguous(cuda, D, tail):
    g = torch.Generator(device=cuda).manual_seed(D)
    B, T, H, Hkv, S = 2, 61, 8, 2, 1024
    k = torch.randn(B, Hkv, S, D, device=cuda, generator=g).bfloat16()
    v = torch.randn(B, Hkv, S, D, device=cuda, generator=g).bfloat16()
    q = torch.randn(B, T, H, D, device=cuda, generator=g).bfloat16()
    mask = torch.tensor([_tree_bits(T, torch.Generator().manual_seed(b)) for b in range(B)], device=cuda)
    kv_len = torch.tensor([700, 90], dtype=torch.int32, device=cuda)
    n_new = torch.full((B,), T, dtype=torch.int32, device=cuda)
    cache = _paged_copy(k, v, cuda)
    pk, pv = cache.layer(0)
    for window in (0, 100):
        want = ops.attention(q, k, v, kv_len, n_new, mask, tail=tail, window=window)
        got = ops.attention(q, pk, pv, kv_len, n_new, mask, tail=tail, window=window, pages=cache.pages(0))
        assert torch.equal(got, want), window
    # causal prefill over the pages
    kv0 = torch.zeros(B, dtype=torch.int32, device=cuda)
    n = torch.tensor([300, 41], dtype=torch.int32, device=cuda)
    qp = torch.randn(B, 300, H, D, device=cuda, generator=g).bfloat16()
    assert torch.equal(ops.attention(qp, pk, pv, kv0, n, None, pages=cache.pages(0)),
                       ops.attention(qp, k, v, kv0, n, None))
    assert ops.require().status(0) == 0


def test_paged_rope_store_and_compaction(cuda):
    g = torch.Generator(device=cuda).manual_seed(1)
    B, T, H, Hkv, S, D = 2, 9, 8, 2, 512, 128
    flat = torch.zeros(1, 2, B, Hkv, S, D, device=cuda, dtype=torch.bfloat16)
    cache = _paged_copy(flat[0, 0], flat[0, 1], cuda)
    qkv = torch.randn(B, T, (H + 2 * Hkv) * D, device=cuda, generator=g).bfloat16()
    kv_len = torch.tensor([250, 120], dtype=torch.int32, device=cuda)  # writes cross a page boundary
    n_new = torch.full((B,), T, dtype=torch.int32, device=cuda)
    pos = (kv_len[:, None] + torch.arange(T, device=cuda)).int().contiguous()
    cos = torch.randn(1024, D // 2, device=cuda, generator=g)
    sin = torch.randn(1024, D // 2, device=cuda, generator=g)
    k, v = cache.layer(0)
    q1 = ops.rope_store(qkv, pos, cos, sin, H, Hkv, D, flat[0, 0], flat[0, 1], kv_len, n_new)
    q2 = ops.rope_store(qkv, pos, cos, sin, H, Hkv, D, k, v, kv_len, n_new, pages=cache.pages(0))
    assert torch.equal(q1, q2)
    assert torch.equal(ref.paged_logical(k, cache.pages(0)), flat[0, 0])
    assert torch.equal(ref.paged_logical(v, cache.pages(0)), flat[0, 1])
    path = torch.tensor([[0, 3, 5, 8] + [8] * 5, [0, 1, 2, 4] + [4] * 5], dtype=torch.int32, device=cuda)
    n_acc = torch.tensor([3, 3], dtype=torch.int32, device=cuda)
    ops.kv_compact(flat, kv_len, path, n_acc)
    ops.kv_compact(cache.data, kv_len, path, n_acc, cache.tables)
    assert torch.equal(ref.paged_logical(k, cache.pages(0)), flat[0, 0])


def _windowed(dev, head_dim=128):
    cfg = tiny_llama(hidden_size=512, num_heads=4, num_kv_heads=2, head_dim=head_dim, num_layers=3,
                     intermediate_size=1024, layer_types=("sliding_attention", "full_attention", "sliding_attention"),
                     sliding_window=200)
    return init_weights(CausalLM(cfg, torch.bfloat16, dev), seed=0)


def test_ring_cache_decoding_equals_contiguous(cuda):
    em = eco.apply(_windowed(cuda), Eagle3Config())
    prompts = [torch.randint(0, 1024, (n,), generator=torch.Generator().manual_seed(n)).to(cuda) for n in (900, 40)]
    tree = dict(cycle_length=7, draft_policy="dynamic_tree", cuda_graphs=True,
                draft_policy_options={"depth": 6, "topk": 10, "total_tokens": 60})
    # a chunked prefill rounds differently from a whole one on the GPU, so each paged run is compared with the
    # contiguous run of the same options; tree decoding must also equal plain decoding
    chunked = em.decode_batch(prompts, 24, decoding=eco.DecodeConfig(cycle_length=1, prefill_chunk=256))
    whole = em.decode_batch(prompts, 24, decoding=eco.DecodeConfig(cycle_length=1))
    for dc, base in ((eco.DecodeConfig(cycle_length=1, window_cache=True, prefill_chunk=256), chunked),
                     (eco.DecodeConfig(**tree, window_cache=True, prefill_chunk=256), chunked),
                     (eco.DecodeConfig(**tree, kv_pages=True), whole)):
        out = em.decode_batch(prompts, 24, decoding=dc)
        for a, b in zip(base, out):
            assert torch.equal(a.tokens, b.tokens), dc
    assert ops.require().status(0) == 0


def test_paged_kivi_decoding_equals_contiguous(cuda):
    em = eco.apply(_windowed(cuda), KIVIConfig(bits=2, residual=128))
    prompts = [torch.randint(0, 1024, (700,), generator=torch.Generator().manual_seed(7)).to(cuda)]
    base = em.decode_batch(prompts, 16, decoding=eco.DecodeConfig(cycle_length=1))
    out = em.decode_batch(prompts, 16, decoding=eco.DecodeConfig(cycle_length=1, kv_pages=True))
    assert torch.equal(base[0].tokens, out[0].tokens)
