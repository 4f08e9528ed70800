"""Canary padding: every output buffer a kernel writes through a pointer it was given sits inside a larger buffer
whose guard regions hold a canary value; after the launch the guards must be untouched (an out-of-bounds write
shows up here as a changed canary instead of as silent corruption). Covers the cache writers (rotary store,
compaction, KIVI coding, eviction scores) on contiguous and paged caches, at sizes that end on odd tile
boundaries. The bounds-checked build (``ECZ_CHECK=1``) runs the same tests with index checks in the kernels."""

import pytest
import torch

from economize_b200 import ops
from economize_b200.runtime.cache import PagedKVCache

pytestmark = pytest.mark.gpu

PAD = 1024  # guard elements on each side (keeps the view 16-byte aligned for TMA)


def _guarded(shape, dtype, dev, fill=0.0):
    """A tensor of ``shape`` inside a buffer with ``PAD`` canary elements on both sides: (view, buffer)."""
    n = 1
    for s in shape:
        n *= s
    buf = torch.full((n + 2 * PAD,), -7.25 if dtype.is_floating_point else 77, dtype=dtype, device=dev)
    view = buf[PAD:PAD + n].view(*shape)
    view.fill_(fill)
    return view, buf


def _intact(buf, dtype):
    canary = -7.25 if dtype.is_floating_point else 77
    head, tail = buf[:PAD], buf[-PAD:]
    if buf.dtype == torch.float8_e4m3fn:
        head, tail = head.float(), tail.float()
    return bool((head == canary).all() and (tail == canary).all())


@pytest.mark.parametrize("D", [64, 128, 256])
def test_rope_store_and_compaction_stay_in_bounds(cuda, D):
    g = torch.Generator(device=cuda).manual_seed(D)
    B, T, H, Hkv, S, L = 3, 61, 8, 2, 384, 2
    cache, buf = _guarded((L, 2, B, Hkv, S, D), torch.bfloat16, cuda)
    qkv = torch.randn(B, T, (H + 2 * Hkv) * D, device=cuda, generator=g).bfloat16()
    kv_len = torch.tensor([S - T, 0, 200], dtype=torch.int32, device=cuda)  # the first row fills the cache's end
    n_new = torch.full((B,), T, dtype=torch.int32, device=cuda)
    pos = (kv_len[:, None] + torch.arange(T, device=cuda)).int().contiguous()
    cos = torch.randn(S, D // 2, device=cuda, generator=g)
    sin = torch.randn(S, D // 2, device=cuda, generator=g)
    for layer in range(L):
        ops.rope_store(qkv, pos, cos, sin, H, Hkv, D, cache[layer, 0], cache[layer, 1], kv_len, n_new)
    path = torch.randint(0, T, (B, T), device=cuda, generator=g).int()
    path[:, 0] = 0
    ops.kv_compact(cache, kv_len, path, torch.full((B,), T - 1, dtype=torch.int32, device=cuda))
    torch.cuda.synchronize()
    assert _intact(buf, torch.bfloat16)
    assert ops.require().status(0) == 0


def test_paged_pool_stays_in_bounds(cuda):
    g = torch.Generator(device=cuda).manual_seed(3)
    B, T, H, Hkv, S, D, L = 2, 40, 4, 2, 512, 128, 2
    pool = PagedKVCache(L, B, Hkv, S, D, torch.bfloat16, cuda, windows=[200, 0], reserve=128)
    data, buf = _guarded(tuple(pool.data.shape), torch.bfloat16, cuda)
    pool.data = data
    kv_len = torch.tensor([S - T - 64, 130], dtype=torch.int32, device=cuda)
    n_new = torch.full((B,), T, dtype=torch.int32, device=cuda)
    pos = (kv_len[:, None] + torch.arange(T, device=cuda)).int().contiguous()
    cos = torch.randn(S, D // 2, device=cuda, generator=g)
    sin = torch.randn(S, D // 2, device=cuda, generator=g)
    qkv = torch.randn(B, T, (H + 2 * Hkv) * D, device=cuda, generator=g).bfloat16()
    for layer in range(L):
        k, v = pool.layer(layer)
        ops.rope_store(qkv, pos, cos, sin, H, Hkv, D, k, v, kv_len, n_new, pages=pool.pages(layer))
    path = torch.arange(T, device=cuda).expand(B, T).int().contiguous()
    ops.kv_compact(pool.data, kv_len, path, torch.full((B,), T - 1, dtype=torch.int32, device=cuda), pool.tables)
    torch.cuda.synchronize()
    assert _intact(buf, torch.bfloat16)


def test_kivi_codes_and_scores_stay_in_bounds(cuda):
    g = torch.Generator(device=cuda).manual_seed(4)
    B, Hkv, S, D, L, H, T = 2, 2, 512, 128, 1, 4, 8
    cache = torch.randn(L, 2, B, Hkv, S, D, device=cuda, generator=g).bfloat16()
    chunk = ops.require().kivi_chunk_size(2)
    kivi, kbuf = _guarded((L, B, Hkv, S // 128, chunk), torch.uint8, cuda, fill=0)
    chunks = torch.zeros(B, dtype=torch.int32, device=cuda)
    ops.kivi_quantize(cache, kivi, torch.tensor([S, 300], dtype=torch.int32, device=cuda), chunks, 2, 0, S // 128)
    q = torch.randn(B, T, H, D, device=cuda, generator=g).bfloat16()
    kv_len = torch.tensor([S - T, 100], dtype=torch.int32, device=cuda)
    n_new = torch.full((B,), T, dtype=torch.int32, device=cuda)
    lse = torch.empty(B, T, H, device=cuda)
    ops.attention(q, cache[0, 0], cache[0, 1], kv_len, n_new, None, lse_out=lse)
    scores, sbuf = _guarded((B, Hkv, S), torch.float32, cuda)
    ops.attention_scores(q, cache[0, 0], kv_len, n_new, None, lse, scores)
    torch.cuda.synchronize()
    assert _intact(kbuf, torch.uint8) and _intact(sbuf, torch.float32)
    assert ops.require().status(0) == 0
