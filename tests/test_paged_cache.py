"""Paged KV caches: a pool of 128-slot pages with one page table per layer, and ring tables for sliding-window
layers (``DecodeConfig(window_cache=True)``). Generation through a paged or ring cache equals generation through the
contiguous cache, the ring's memory follows the window, and the reference ops read and write through the tables."""

import pytest
import torch

import economize_b200 as eco
from economize_b200.errors import ConfigError
from economize_b200.models.config import tiny_llama
from economize_b200.models.llama import CausalLM, init_weights
from economize_b200.ops import reference as ref
from economize_b200.runtime.cache import PagedKVCache, ring_pages
from economize_b200.techniques.eagle3 import Eagle3Config
from economize_b200.techniques.kv_evict import KVEvictConfig

TREE = dict(cycle_length=7, draft_policy="dynamic_tree", draft_policy_options={"depth": 6, "topk": 10,
                                                                               "total_tokens": 60})


def _windowed():
    cfg = tiny_llama(num_layers=3, layer_types=("sliding_attention", "full_attention", "sliding_attention"),
                     sliding_window=100)
    return init_weights(CausalLM(cfg, torch.float32, "cpu"), seed=0)


def test_ring_tables_and_memory():
    c = PagedKVCache(3, 2, 2, 1024, 64, torch.float32, "cpu", windows=[100, 0, 100], reserve=128)
    assert c.rings == [ring_pages(100, 128)] * 1 + [0] + [ring_pages(100, 128)] and c.rings[0] == 3
    assert c.num_pages == 2 * (3 + 8 + 3)  # two rings of 3 pages and one full layer of 8 pages per row
    t = c.tables
    assert torch.equal(t[0, 0], torch.tensor([0, 1, 2, 0, 1, 2, 0, 1], dtype=torch.int32))
    assert len(set(t[1].flatten().tolist())) == 16  # a full layer's pages are its own


@pytest.mark.parametrize("decoding", [dict(cycle_length=1), TREE])
def test_paged_and_ring_generation_equal_contiguous(decoding):
    em = eco.apply(_windowed(), Eagle3Config())
    prompts = [torch.randint(0, 1024, (n,), generator=torch.Generator().manual_seed(n)) for n in (600, 17)]
    base = em.decode_batch(prompts, 16, decoding=eco.DecodeConfig(cycle_length=1))
    for extra in (dict(kv_pages=True), dict(window_cache=True, prefill_chunk=128)):
        out = em.decode_batch(prompts, 16, decoding=eco.DecodeConfig(**decoding, **extra))
        for a, b in zip(base, out):
            assert torch.equal(a.tokens, b.tokens), extra


def test_reference_ops_through_page_tables():
    g = torch.Generator().manual_seed(0)
    B, Hkv, H, D, S = 2, 2, 4, 16, 384
    cache = PagedKVCache(1, B, Hkv, S, D, torch.float32, "cpu")
    cache.tables[0] = cache.tables[0].flip(1)  # any page order
    k, v = cache.layer(0)
    pages = cache.pages(0)
    qkv = torch.randn(B, 5, (H + 2 * Hkv) * D, generator=g)
    kv_len = torch.tensor([200, 7], dtype=torch.int32)
    n_new = torch.tensor([5, 5], dtype=torch.int32)
    pos = (kv_len[:, None] + torch.arange(5)).int()
    cos, sin = torch.randn(512, D // 2, generator=g), torch.randn(512, D // 2, generator=g)
    flat_k, flat_v = torch.zeros(B, Hkv, S, D), torch.zeros(B, Hkv, S, D)
    body = torch.randn(B, Hkv, S, D, generator=g)
    flat_k += body
    flat_v += body * 0.5
    for b in range(B):  # fill the pool with the same committed keys
        for c in range(S // 128):
            page = int(pages[b, c])
            k[page] = flat_k[b, :, c * 128:(c + 1) * 128]
            v[page] = flat_v[b, :, c * 128:(c + 1) * 128]
    q1 = ref.rope_store(qkv, pos, cos, sin, H, Hkv, D, flat_k, flat_v, kv_len, n_new)
    q2 = ref.rope_store(qkv, pos, cos, sin, H, Hkv, D, k, v, kv_len, n_new, pages=pages)
    torch.testing.assert_close(q1, q2)
    torch.testing.assert_close(ref.paged_logical(k, pages), flat_k)
    o1 = ref.attention(q1, flat_k, flat_v, kv_len, n_new, None, window=50)
    o2 = ref.attention(q2, k, v, kv_len, n_new, None, window=50, pages=pages)
    torch.testing.assert_close(o1, o2)
    path = torch.tensor([[0, 2, 4, 4, 4], [0, 1, 3, 3, 3]])
    n_acc = torch.tensor([2, 2], dtype=torch.int32)
    whole = torch.stack([flat_k, flat_v])[None]  # [1, 2, B, Hkv, S, D]
    ref.kv_compact(whole, kv_len, path, n_acc)
    ref.kv_compact(cache.data, kv_len, path, n_acc, cache.tables)
    torch.testing.assert_close(ref.paged_logical(k, pages), whole[0, 0])


def test_paged_cache_refuses_keep_bitmap_techniques():
    em = eco.apply(_windowed(), KVEvictConfig(method="streaming", budget=64, window=16))
    with pytest.raises(ConfigError, match="paged"):
        em.decode_batch([torch.arange(40)], 4, decoding=eco.DecodeConfig(cycle_length=1, kv_pages=True))
