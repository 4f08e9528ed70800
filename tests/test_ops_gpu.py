"""Numerics of every CUDA kernel against the plain PyTorch fp32 implementation of the same op
(economize_b200.ops.reference), at small shapes that cover the tile edges (tile-unaligned M, N, K, slots), GQA
packing, tree masks, causal prefill with ragged rows, and split-K / split-key reductions."""

import pytest
import torch

from economize_b200 import ops
from economize_b200.ops import reference as ref

pytestmark = pytest.mark.gpu


def _close(a, b, atol, rtol=2e-2):
    torch.testing.assert_close(a.float(), b.float(), atol=atol, rtol=rtol)


@pytest.mark.parametrize("rows,hidden", [(1, 4096), (61, 4096), (7, 256), (33, 8192)])
@pytest.mark.parametrize("with_resid", [False, True])
def test_rmsnorm(cuda, rows, hidden, with_resid):
    g = torch.Generator(device=cuda).manual_seed(0)
    x = torch.randn(rows, hidden, device=cuda, generator=g).bfloat16()
    r = torch.randn(rows, hidden, device=cuda, generator=g).bfloat16() if with_resid else None
    w = (1 + 0.1 * torch.randn(hidden, device=cuda, generator=g)).bfloat16()
    out, res = ops.rmsnorm(x, w, 1e-5, r)
    e_out, e_res = ref.rmsnorm(x, w, 1e-5, r)  # same bf16 rounding steps, computed by torch
    _close(res, e_res, 0, 0)
    _close(out, e_out, 2e-2)
    exact = ref.rmsnorm(x.float(), w.float(), 1e-5, None if r is None else r.float())[0]
    _close(out, exact, 5e-2)


@pytest.mark.parametrize("M,N,K", [(1, 256, 256), (61, 6144, 4096), (64, 512, 688), (200, 1024, 512),
                                   (300, 384, 1024), (5, 128256 // 16, 4096)])
def test_linear(cuda, M, N, K):
    g = torch.Generator(device=cuda).manual_seed(1)
    x = torch.randn(M, K, device=cuda, generator=g).bfloat16()
    w = (torch.randn(N, K, device=cuda, generator=g) * 0.02).bfloat16()
    y = ops.linear(x, w)
    expect = x.float() @ w.float().T
    _close(y, expect, 2e-2 * expect.abs().max().item() / 4 + 1e-3)
    assert ops.require().status(0) == 0


def test_linear_deterministic_in_rows(cuda):
    """A row's result does not depend on how many other rows the launch has (up to 256 rows)."""
    g = torch.Generator(device=cuda).manual_seed(2)
    x = torch.randn(61, 4096, device=cuda, generator=g).bfloat16()
    w = (torch.randn(4096, 4096, device=cuda, generator=g) * 0.02).bfloat16()
    full = ops.linear(x, w)
    one = ops.linear(x[:1].contiguous(), w)
    assert torch.equal(full[:1], one) or (full[:1] - one).abs().max().item() < 1e-2


def _cache(B, Hkv, S, D, dev, g):
    k = (torch.randn(B, Hkv, S, D, device=dev, generator=g)).bfloat16()
    v = (torch.randn(B, Hkv, S, D, device=dev, generator=g)).bfloat16()
    return k, v


def _tree_mask(B, T, dev, g):
    """Random topological trees: node 0 the root, every node's parent an earlier node; bits = ancestors + self."""
    masks = torch.zeros(B, T, dtype=torch.int64)
    for b in range(B):
        anc = [1]
        for t in range(1, T):
            p = int(torch.randint(0, t, (1,)))
            anc.append(anc[p] | (1 << t))
        masks[b] = torch.tensor([a if a < 2**63 else a - 2**64 for a in anc])
    return masks.to(dev)


@pytest.mark.parametrize("B,T,H,Hkv,S,lens", [
    (1, 61, 32, 8, 832, [512]),      # the benchmark's tree pass
    (2, 61, 8, 2, 300, [120, 37]),   # ragged, slots not a multiple of the key tile
    (3, 1, 32, 8, 700, [600, 1, 129]),  # plain decode
    (2, 10, 4, 4, 200, [0, 64]),     # no GQA
])
def test_tree_attention(cuda, B, T, H, Hkv, S, lens):
    g = torch.Generator(device=cuda).manual_seed(3)
    D = 128
    k, v = _cache(B, Hkv, S, D, cuda, g)
    q = torch.randn(B, T, H, D, device=cuda, generator=g).bfloat16()
    kv_len = torch.tensor(lens, dtype=torch.int32, device=cuda)
    n_new = torch.full((B,), T, dtype=torch.int32, device=cuda)
    mask = _tree_mask(B, T, cuda, g)
    out = ops.attention(q, k, v, kv_len, n_new, mask)
    expect = ref.attention(q.float(), k.float(), v.float(), kv_len, n_new, mask)
    _close(out, expect, 2e-2)
    assert ops.require().status(0) == 0


@pytest.mark.parametrize("B,T,H,Hkv,lens", [(1, 512, 32, 8, [512]), (3, 200, 8, 2, [200, 17, 150]),
                                            (2, 40, 4, 2, [40, 39])])
def test_causal_prefill_attention(cuda, B, T, H, Hkv, lens):
    g = torch.Generator(device=cuda).manual_seed(4)
    D, S = 128, T + 64
    k, v = _cache(B, Hkv, S, D, cuda, g)
    q = torch.randn(B, T, H, D, device=cuda, generator=g).bfloat16()
    kv_len = torch.zeros(B, dtype=torch.int32, device=cuda)
    n_new = torch.tensor(lens, dtype=torch.int32, device=cuda)
    out = ops.attention(q, k, v, kv_len, n_new, None)
    expect = ref.attention(q.float(), k.float(), v.float(), kv_len, n_new, None)
    for b, n in enumerate(lens):
        _close(out[b, :n], expect[b, :n], 2e-2)


def test_attention_q_offset(cuda):
    """A drafter's tree step: queries are the last W nodes of a forwarded region, visible by ancestor bits."""
    g = torch.Generator(device=cuda).manual_seed(5)
    B, W, H, Hkv, S, D = 2, 10, 8, 2, 256, 128
    k, v = _cache(B, Hkv, S, D, cuda, g)
    q = torch.randn(B, W, H, D, device=cuda, generator=g).bfloat16()
    kv_len = torch.tensor([100, 7], dtype=torch.int32, device=cuda)
    n_new = torch.full((B,), 30, dtype=torch.int32, device=cuda)
    full = _tree_mask(B, 30, cuda, g)
    mask = full[:, 20:].contiguous()
    out = ops.attention(q, k, v, kv_len, n_new, mask, q_offset=20)
    expect = ref.attention(q.float(), k.float(), v.float(), kv_len, n_new, mask, q_offset=20)
    _close(out, expect, 2e-2)


@pytest.mark.parametrize("qk_norm", [False, True])
@pytest.mark.parametrize("D", [64, 128, 256])
def test_rope_store(cuda, qk_norm, D):
    g = torch.Generator(device=cuda).manual_seed(6)
    B, T, H, Hkv, S = 2, 7, 8, 2, 64
    qkv = torch.randn(B, T, (H + 2 * Hkv) * D, device=cuda, generator=g).bfloat16()
    pos = torch.randint(0, 40, (B, T), device=cuda, generator=g, dtype=torch.int32)
    inv = 1.0 / (10000 ** (torch.arange(0, D, 2, device=cuda).float() / D))
    ang = torch.arange(64, device=cuda).float()[:, None] * inv[None]
    cos, sin = ang.cos().contiguous(), ang.sin().contiguous()
    kv_len = torch.tensor([3, 20], dtype=torch.int32, device=cuda)
    n_new = torch.tensor([7, 5], dtype=torch.int32, device=cuda)
    qn = (1 + 0.1 * torch.randn(D, device=cuda, generator=g)).bfloat16() if qk_norm else None
    kn = (1 + 0.1 * torch.randn(D, device=cuda, generator=g)).bfloat16() if qk_norm else None
    kc, vc = torch.zeros(B, Hkv, S, D, device=cuda).bfloat16(), torch.zeros(B, Hkv, S, D, device=cuda).bfloat16()
    kr, vr = kc.clone(), vc.clone()
    q = ops.rope_store(qkv, pos, cos, sin, H, Hkv, D, kc, vc, kv_len, n_new, qn, kn, 1e-6)
    qe = ref.rope_store(qkv, pos, cos, sin, H, Hkv, D, kr, vr, kv_len, n_new, qn, kn, 1e-6)
    _close(q, qe, 2e-2)
    _close(kc, kr, 2e-2)
    _close(vc, vr, 0, 0)


def test_silu_mul(cuda):
    g = torch.Generator(device=cuda).manual_seed(7)
    x = torch.randn(61, 2 * 14336, device=cuda, generator=g).bfloat16()
    _close(ops.silu_mul(x), ref.silu_mul(x.float()), 3e-2)


def test_argmax(cuda):
    g = torch.Generator(device=cuda).manual_seed(8)
    x = torch.randn(61, 128256, device=cuda, generator=g).bfloat16()
    x[3, 17] = 100.0
    x[4, :] = 0
    got = ops.argmax(x)
    assert torch.equal(got, x.float().argmax(-1))
    assert got[4].item() == 0


def test_greedy_accept_and_compact(cuda):
    g = torch.Generator().manual_seed(9)
    B, T = 4, 61
    parents = torch.zeros(B, T, dtype=torch.int64)
    for b in range(B):
        for t in range(1, T):
            parents[b, t] = int(torch.randint(0, t, (1,), generator=g))
    tokens = torch.randint(0, 5, (B, T), generator=g)
    pred = torch.randint(0, 5, (B, T), generator=g)
    e_n, e_path, e_out = ref.greedy_accept(tokens, parents, pred)
    n, path, out = ops.greedy_accept(tokens.to(cuda), parents.to(cuda), pred.to(cuda))
    assert torch.equal(n.cpu(), e_n)
    for b in range(B):
        k = int(e_n[b])
        assert torch.equal(path[b, : k + 1].cpu(), e_path[b, : k + 1])
        assert torch.equal(out[b, : k + 1].cpu(), e_out[b, : k + 1])
    cache = torch.randn(3, 2, B, 2, 128, 128, generator=g).bfloat16()
    kv_len = torch.tensor([0, 5, 50, 60], dtype=torch.int32)
    exp = cache.clone()
    ref.kv_compact(exp, kv_len, e_path, e_n)
    got = cache.to(cuda)
    ops.kv_compact(got, kv_len.to(cuda), path, n)
    assert torch.equal(got.cpu(), exp)


def test_sample_kernel_matches_reference(cuda):
    g = torch.Generator(device=cuda).manual_seed(10)
    probs = torch.softmax(torch.randn(33, 128256, device=cuda, generator=g) * 3, -1)
    u = torch.rand(33, device=cuda, generator=g)
    got = ops.sample(probs, u)
    want = ref.sample(probs.double().cpu(), u.cpu())
    # inverse CDF in fp32 vs fp64: equal, or adjacent in the support at a CDF boundary
    diff = (got.cpu() != want).sum().item()
    assert diff <= 1


def test_rejection_kernel_matches_reference(cuda):
    g = torch.Generator().manual_seed(11)
    B, k, V = 16, 4, 4096
    p = torch.softmax(torch.randn(B, k + 1, V, generator=g), -1)
    q = torch.softmax(torch.randn(B, k, V, generator=g) * 2, -1)
    drafts = torch.multinomial(q.reshape(-1, V), 1, generator=g).reshape(B, k)
    # make some drafts near-certain accepts
    p[:, :k].scatter_(2, drafts[..., None], 0.5)
    p = p / p.sum(-1, keepdim=True)
    u_acc, u_draw = torch.rand(B, k, generator=g), torch.rand(B, generator=g)
    n_ref, out_ref = ref.rejection(p.double(), q.double(), drafts, u_acc.double(), u_draw.double())
    n_got, out_got = ops.rejection(p.to(cuda), q.to(cuda), drafts.to(cuda), u_acc.to(cuda), u_draw.to(cuda))
    assert torch.equal(n_got.cpu(), n_ref)
    for b in range(B):
        j = int(n_ref[b])
        assert torch.equal(out_got[b, :j].cpu(), out_ref[b, :j])
        assert abs(int(out_got[b, j]) - int(out_ref[b, j])) <= 1 or out_got[b, j] == out_ref[b, j]


@pytest.mark.parametrize("M,N,K", [(1, 6144, 4096), (61, 4096, 4096), (61, 1024, 14336), (40, 28672, 4096),
                                   (7, 264, 512)])
def test_linear_parts_matches_fp32(cuda, M, N, K):
    g = torch.Generator(device=cuda).manual_seed(0)
    x = torch.randn(M, K, device=cuda, generator=g).bfloat16()
    w = (torch.randn(N, K, device=cuda, generator=g) * 0.02).bfloat16()
    y = ops.linear_parts(x, w)
    dense = y.sum() if isinstance(y, ops.Partials) else y
    _close(dense, x.float() @ w.float().t(), 2e-2)


def test_consumers_reduce_partials_exactly(cuda):
    g = torch.Generator(device=cuda).manual_seed(1)
    B, T, H, Hkv, D, S, hidden = 1, 61, 8, 2, 128, 256, 4096
    x = torch.randn(B * T, hidden, device=cuda, generator=g).bfloat16()
    # rmsnorm of a projection output
    w = (torch.randn(hidden, hidden, device=cuda, generator=g) * 0.02).bfloat16()
    p = ops.linear_parts(x, w)
    assert isinstance(p, ops.Partials) and p.data.shape[0] > 1
    nw = (1 + 0.1 * torch.randn(hidden, device=cuda, generator=g)).bfloat16()
    r = torch.randn(B * T, hidden, device=cuda, generator=g).bfloat16()
    a, ra = ops.rmsnorm(p, nw, 1e-5, r)
    b, rb = ops.rmsnorm(p.sum(), nw, 1e-5, r)
    assert torch.equal(a, b) and torch.equal(ra, rb)
    # silu_mul of a gate/up projection
    wgu = (torch.randn(2 * 1024, hidden, device=cuda, generator=g) * 0.02).bfloat16()
    pg = ops.linear_parts(x, wgu)
    assert torch.equal(ops.silu_mul(pg), ops.silu_mul(pg.sum()))
    # rope_store of a qkv projection
    wqkv = (torch.randn((H + 2 * Hkv) * D, hidden, device=cuda, generator=g) * 0.02).bfloat16()
    pq = ops.linear_parts(x, wqkv)
    pq = ops.Partials(pq.data.reshape(pq.data.shape[0], B, T, -1)) if isinstance(pq, ops.Partials) else pq
    dense = pq.sum() if isinstance(pq, ops.Partials) else pq
    inv = 1.0 / (10000 ** (torch.arange(0, D, 2, device=cuda).float() / D))
    ang = torch.arange(512, device=cuda).float()[:, None] * inv[None]
    cos, sin = ang.cos().contiguous(), ang.sin().contiguous()
    pos = torch.arange(T, device=cuda, dtype=torch.int32)[None].contiguous()
    kv_len = torch.zeros(B, dtype=torch.int32, device=cuda)
    n_new = torch.full((B,), T, dtype=torch.int32, device=cuda)
    outs = []
    for qkv in (pq, dense):
        kc = torch.zeros(B, Hkv, S, D, dtype=torch.bfloat16, device=cuda)
        vc = torch.zeros_like(kc)
        q = ops.rope_store(qkv, pos, cos, sin, H, Hkv, D, kc, vc, kv_len, n_new)
        outs.append((q, kc, vc))
    for u, v in zip(*outs):
        assert torch.equal(u, v)


def test_partials_index_like_the_dense_tensor(cuda):
    g = torch.Generator(device=cuda).manual_seed(2)
    x = torch.randn(2, 9, 4096, device=cuda, generator=g).bfloat16()
    w = (torch.randn(4096, 4096, device=cuda, generator=g) * 0.02).bfloat16()
    p = ops.linear_parts(x, w)
    assert isinstance(p, ops.Partials)
    rows, cols = torch.tensor([0, 1], device=cuda), torch.tensor([3, 8], device=cuda)
    assert torch.equal(p[rows, cols].sum(), p.sum()[rows, cols])


@pytest.mark.parametrize("rows,V,k", [(1, 32000, 10), (10, 32000, 10), (61, 1024, 16), (3, 128256, 4),
                                      (200, 32000, 8)])
def test_topk_logp_matches_torch(cuda, rows, V, k):
    g = torch.Generator(device=cuda).manual_seed(0)
    logits = torch.randn(rows, V, device=cuda, generator=g) * 3
    d2t = torch.randint(0, 5, (V,), device=cuda, generator=g)
    vals, ids = ops.topk_logp(logits, k, -1e4, d2t)
    ref = torch.log_softmax(logits, -1).topk(k, -1)
    _close(vals, ref.values, 1e-4, 1e-5)
    assert torch.equal(ids, ref.indices + d2t[ref.indices])


def test_topk_logp_split_repeats_and_masked_chunks(cuda):
    """Rows split over several CTAs: the per-row arrival counters reset themselves, so back-to-back calls agree, and
    chunks that hold only -inf logits merge correctly."""
    g = torch.Generator(device=cuda).manual_seed(3)
    logits = torch.randn(7, 32000, device=cuda, generator=g)
    logits[:, 4000:30000] = float("-inf")
    first = ops.topk_logp(logits, 16, -1e4, None)
    for _ in range(3):
        again = ops.topk_logp(logits, 16, -1e4, None)
        assert torch.equal(first[0], again[0]) and torch.equal(first[1], again[1])
    ref = torch.log_softmax(logits, -1).topk(16, -1)
    _close(first[0], ref.values, 1e-4, 1e-5)
    assert torch.equal(first[1], ref.indices)


@pytest.mark.gpu
def test_host_index_tensors_are_refused_before_launch(cuda):
    """Index tensors on the host would be dereferenced as device pointers: the bindings refuse them."""
    from economize_b200 import ops

    q = torch.randn(1, 1, 4, 128, device=cuda).bfloat16()
    k = torch.zeros(1, 2, 128, 128, device=cuda).bfloat16()
    with pytest.raises(RuntimeError, match="must be on the device"):
        ops.attention(q, k, k.clone(), torch.tensor([5], dtype=torch.int32), torch.tensor([1], dtype=torch.int32))


@pytest.mark.gpu
def test_chunked_prefill_matches_whole_prefill(cuda):
    import economize_b200 as eco

    from .helpers import gpu_tiny_model, prompts

    model = gpu_tiny_model(cuda)
    p = [x.to(cuda) for x in prompts((300, 517))]
    em = eco.apply(model)
    whole = em.decode_batch(p, 12, decoding=eco.DecodeConfig(cycle_length=1))
    chunked = em.decode_batch(p, 12, decoding=eco.DecodeConfig(cycle_length=1, prefill_chunk=128))
    # a 5-token last chunk runs the projections through the skinny-GEMM kernel, whose K split differs from the one
    # a 517-token pass takes, so the two caches agree to rounding, not bit for bit: the first token agrees and every
    # token of the chunked run is greedy under a causal recompute of its own sequence
    for prompt, a, b in zip(p, whole, chunked):
        assert int(a.tokens[0]) == int(b.tokens[0])
        seq = torch.cat([prompt, b.tokens.to(cuda)])
        logits = em(seq[None])[0].float()
        for i, tok in enumerate(b.tokens.tolist()):
            row = logits[prompt.numel() - 1 + i]
            assert (row.max() - row[tok]).item() <= 0.08 * max(1.0, row.abs().max().item())


@pytest.mark.gpu
@pytest.mark.parametrize("k,depth,total", [(10, 6, 60), (4, 3, 16), (8, 4, 40)])
def test_fused_tree_kernels_match_the_reference(cuda, k, depth, total):
    """tree_expand + tree_select against the tensor operations of the engine's reference tree drafting."""
    from economize_b200.decoding.tree import select_candidates
    from economize_b200.ops._ext import require

    C = require()
    g = torch.Generator(device=cuda).manual_seed(k)
    B = 3
    n_cand = k + (depth - 1) * k * k
    f_scores = -torch.rand(B, k, device=cuda, generator=g)
    f_tokens = torch.randint(0, 1000, (B, k), device=cuda, generator=g)
    cand_t = torch.empty(B, n_cand, dtype=torch.int64, device=cuda)
    cand_s = torch.empty(B, n_cand, device=cuda)
    cand_p = torch.empty(B, n_cand, dtype=torch.int64, device=cuda)
    cand_t[:, :k], cand_s[:, :k], cand_p[:, :k] = f_tokens, f_scores, -1
    ref_t, ref_s, ref_p, ref_d = [f_tokens.clone()], [f_scores.clone()], [torch.full((B, k), -1, device=cuda)], \
        [torch.zeros(k, device=cuda)]
    f_cand = torch.arange(k, device=cuda).expand(B, k).contiguous()
    rf_cand, rf_scores = f_cand.clone(), f_scores.clone()
    parent_fwd = torch.full((B, k), -1, dtype=torch.int64, device=cuda)
    fwd_bits = torch.zeros(B, (depth - 1) * k, dtype=torch.int64, device=cuda)
    fwd_bits[:, :k] = 1 << torch.arange(k, device=cuda)
    origin = torch.zeros(B, k, dtype=torch.int64, device=cuda)
    for d in range(1, depth):
        c_vals = -torch.rand(B, k, k, device=cuda, generator=g) * 3
        c_ids = torch.randint(0, 1000, (B, k, k), device=cuda, generator=g)
        nb = torch.empty(B, k, dtype=torch.int64, device=cuda)
        C.tree_expand(c_vals, c_ids, f_scores, f_cand, f_tokens, parent_fwd, fwd_bits, origin, nb, cand_t, cand_s,
                      cand_p, d, d < depth - 1)
        child_scores = (rf_scores[:, :, None] + c_vals).reshape(B, k * k)
        ref_t.append(c_ids.reshape(B, k * k))
        ref_s.append(child_scores)
        ref_p.append(rf_cand[:, :, None].expand(B, k, k).reshape(B, k * k))
        ref_d.append(torch.full((k * k,), float(d), device=cuda))
        if d < depth - 1:
            pick = child_scores.topk(k, -1).indices
            rf_scores = child_scores.gather(1, pick)
            rf_cand = k + (d - 1) * k * k + pick
            assert torch.equal(f_cand, rf_cand) and torch.allclose(f_scores, rf_scores)
            assert torch.equal(origin, pick // k)
            assert torch.equal(nb, (1 << (d * k + torch.arange(k, device=cuda)))[None] |
                               fwd_bits.gather(1, (d - 1) * k + pick // k))
    assert torch.equal(cand_t, torch.cat(ref_t, 1)) and torch.equal(cand_p, torch.cat(ref_p, 1))
    torch.testing.assert_close(cand_s, torch.cat(ref_s, 1))
    tok, par = C.tree_select(cand_t, cand_s, cand_p, k, total)
    rtok, rpar = select_candidates(torch.cat(ref_t, 1), torch.cat(ref_s, 1), torch.cat(ref_p, 1), torch.cat(ref_d),
                                   total)
    assert torch.equal(tok, rtok) and torch.equal(par, rpar)


def test_tree_layout_matches_pointer_doubling(cuda):
    from economize_b200.decoding.tree import ancestor_bits, popcount64

    g = torch.Generator().manual_seed(4)
    for T in (1, 7, 61, 64):
        parents = torch.zeros(3, T, dtype=torch.int64)
        for i in range(1, T):
            parents[:, i] = torch.randint(0, i, (3,), generator=g)
        kv_len = torch.tensor([5, 0, 700], dtype=torch.int32)
        bits, pos = ops.tree_layout(parents.to(cuda), kv_len.to(cuda), 63)
        ref = ancestor_bits(parents, 63)
        assert torch.equal(bits.cpu(), ref)
        assert torch.equal(pos.cpu(), (kv_len[:, None] + popcount64(ref) - 1).int())


def test_rope_store_reports_positions_and_slots_out_of_range(cuda):
    """A position past the rotary tables or a slot past the cache is reported in the status word and never read or
    written (the tables of a model cover its cache's capacity, so the engine never hits this)."""
    g = torch.Generator(device=cuda).manual_seed(9)
    B, T, H, Hkv, S, D = 1, 4, 4, 2, 128, 128
    qkv = torch.randn(B, T, (H + 2 * Hkv) * D, device=cuda, generator=g).bfloat16()
    cos = torch.randn(64, D // 2, device=cuda, generator=g)
    sin = torch.randn(64, D // 2, device=cuda, generator=g)
    k = torch.zeros(B, Hkv, S, D, device=cuda, dtype=torch.bfloat16)
    v = torch.zeros_like(k)
    ops.require().status(0)  # start clean
    pos = torch.tensor([[10, 63, 64, 500]], dtype=torch.int32, device=cuda)
    q = ops.rope_store(qkv, pos, cos, sin, H, Hkv, D, k, v, torch.tensor([0], dtype=torch.int32, device=cuda),
                       torch.tensor([T], dtype=torch.int32, device=cuda))
    torch.cuda.synchronize()
    assert ops.require().status(0) & 32 and torch.isfinite(q.float()).all()
    kv_len = torch.tensor([S - 2], dtype=torch.int32, device=cuda)  # the last two tokens fall past the cache
    ops.rope_store(qkv, pos.clamp(max=63), cos, sin, H, Hkv, D, k, v, kv_len,
                   torch.tensor([T], dtype=torch.int32, device=cuda))
    torch.cuda.synchronize()
    assert ops.require().status(0) & 32
    assert k[0, :, S - 2:].abs().sum() > 0  # the two slots inside the cache were written
