"""fp8 KV cache (kv_fp8): calibrated per-head scales, e4m3 writes, attention over codes, lossless decoding of the
fp8 model, and the kernel paths against the PyTorch reference."""

import pytest
import torch

import economize_b200 as eco
from economize_b200 import ops
from economize_b200.ops import reference as ref
from economize_b200.techniques.eagle3 import Eagle3Config
from economize_b200.techniques.kv_quant import KVFp8Config, calibrate_kv_scales

from .helpers import gpu_tiny_model, prompts, reference_greedy, tiny_model


def test_calibrated_scales_cover_the_range():
    model = tiny_model()
    k, v = calibrate_kv_scales(model, [torch.randint(0, 1024, (2, 24))])
    assert k.shape == (4, 2) and v.shape == (4, 2) and (k > 0).all()
    eff = eco.apply(model, KVFp8Config(), calibration=torch.randint(0, 1024, (2, 24)))
    cache = eff.model.new_cache(1, 128)
    assert cache.data.dtype == torch.float8_e4m3fn and cache.scales[0].shape == (4, 2)


def test_fp8_model_decodes_losslessly():
    model = tiny_model()
    eff = eco.apply(model, KVFp8Config(), Eagle3Config(), calibration=torch.randint(0, 1024, (1, 32)),
                    decoding=eco.DecodeConfig(cycle_length=4))
    p = prompts((21,))[0]
    out = eff.decode(p, 10).tokens
    assert torch.equal(out, reference_greedy(eff.model, p, 10))
    # the fp8 cache changes the logits only slightly
    base = eco.EfficientModel(tiny_model(), [], eco.DecodeConfig())
    rel = (eff(p[None]) - base(p[None])).norm() / base(p[None]).norm()
    assert rel < 0.1


def test_unit_scales_need_no_calibration():
    eff = eco.apply(tiny_model(), KVFp8Config(scale="none"))
    assert eff.model.kv_dtype == torch.float8_e4m3fn
    with pytest.raises(eco.ConfigError):
        eco.apply(tiny_model(), KVFp8Config())  # per-head scales need calibration tokens


def test_reference_fp8_roundtrip():
    g = torch.Generator().manual_seed(0)
    B, T, H, Hkv, D, S = 1, 5, 4, 2, 128, 128
    qkv = torch.randn(B, T, (H + 2 * Hkv) * D, generator=g)
    cos, sin = torch.ones(16, D // 2), torch.zeros(16, D // 2)
    pos = torch.arange(T, dtype=torch.int32)[None]
    kc = torch.zeros(B, Hkv, S, D, dtype=torch.float8_e4m3fn)
    vc = torch.zeros_like(kc)
    ks, vs = torch.tensor([0.01, 0.02]), torch.tensor([0.015, 0.005])
    kv_len, n_new = torch.zeros(1, dtype=torch.int32), torch.full((1,), T, dtype=torch.int32)
    ref.rope_store(qkv, pos, cos, sin, H, Hkv, D, kc, vc, kv_len, n_new, k_scale=ks, v_scale=vs)
    k = qkv[..., H * D:(H + Hkv) * D].reshape(B, T, Hkv, D).transpose(1, 2)
    back = kc[:, :, :T].float() * ks[None, :, None, None]
    assert ((back - k).abs() <= k.abs() * 0.07 + 1e-3).all()


# ---- GPU ------------------------------------------------------------------------------------------------------
def _fp8_case(cuda, B, T, Hkv, S, ctx, seed=0):
    g = torch.Generator(device=cuda).manual_seed(seed)
    H, D = 4 * Hkv, 128
    kc = (torch.randn(B, Hkv, S, D, device=cuda, generator=g) * 40).clamp(-440, 440).to(torch.float8_e4m3fn)
    vc = (torch.randn(B, Hkv, S, D, device=cuda, generator=g) * 40).clamp(-440, 440).to(torch.float8_e4m3fn)
    ks = torch.rand(Hkv, device=cuda, generator=g) * 0.02 + 0.005
    vs = torch.rand(Hkv, device=cuda, generator=g) * 0.02 + 0.005
    q = torch.randn(B, T, H, D, device=cuda, generator=g).bfloat16()
    kv_len = torch.full((B,), ctx, dtype=torch.int32, device=cuda)
    n_new = torch.full((B,), T, dtype=torch.int32, device=cuda)
    return q, kc, vc, ks, vs, kv_len, n_new


@pytest.mark.gpu
@pytest.mark.parametrize("B,T,Hkv,S,ctx", [(1, 1, 8, 1024, 700), (2, 61, 8, 1024, 500), (1, 16, 2, 4096, 3000),
                                           (4, 7, 4, 256, 100)])
def test_fp8_attention_matches_reference(cuda, B, T, Hkv, S, ctx):
    from economize_b200.decoding.tree import ancestor_bits

    q, kc, vc, ks, vs, kv_len, n_new = _fp8_case(cuda, B, T, Hkv, S, ctx)
    parents = torch.randint(0, 1, (B, T), device=cuda)
    for t in range(1, T):
        parents[:, t] = torch.randint(0, t, (B,), device=cuda)
    parents[:, 0] = -1
    mask = ancestor_bits(parents, T) if T > 1 else None
    out = ops.attention(q, kc, vc, kv_len, n_new, mask, k_scale=ks, v_scale=vs)
    exp = ref.attention(q.float(), kc, vc, kv_len, n_new, mask, k_scale=ks, v_scale=vs)
    torch.testing.assert_close(out.float(), exp.float(), atol=2e-2, rtol=2e-2)


@pytest.mark.gpu
def test_fp8_rope_store_codes_match_reference(cuda):
    g = torch.Generator(device=cuda).manual_seed(3)
    B, T, H, Hkv, D, S = 2, 9, 8, 2, 128, 256
    qkv = torch.randn(B, T, (H + 2 * Hkv) * D, device=cuda, generator=g).bfloat16()
    inv = 1.0 / (10000 ** (torch.arange(0, D, 2, device=cuda).float() / D))
    ang = torch.arange(64, device=cuda).float()[:, None] * inv[None]
    cos, sin = ang.cos().contiguous(), ang.sin().contiguous()
    pos = (torch.arange(T, device=cuda, dtype=torch.int32)[None] + 5).expand(B, T).contiguous()
    ks = torch.tensor([0.011, 0.017], device=cuda)
    vs = torch.tensor([0.013, 0.007], device=cuda)
    kv_len = torch.tensor([5, 5], dtype=torch.int32, device=cuda)
    n_new = torch.tensor([T, 4], dtype=torch.int32, device=cuda)
    outs = []
    for fn in (ops.rope_store, ref.rope_store):
        kc = torch.zeros(B, Hkv, S, D, dtype=torch.float8_e4m3fn, device=cuda)
        vc = torch.zeros_like(kc)
        fn(qkv, pos, cos, sin, H, Hkv, D, kc, vc, kv_len, n_new, k_scale=ks, v_scale=vs)
        outs.append((kc.view(torch.uint8), vc.view(torch.uint8)))
    assert torch.equal(outs[0][1], outs[1][1])  # values: exact
    assert (outs[0][0].int() - outs[1][0].int()).abs().max() <= 1  # keys: rotary rounding may differ by one code


@pytest.mark.gpu
def test_fp8_engine_decodes_on_gpu(cuda):
    model = gpu_tiny_model(cuda)
    eff = eco.apply(model, KVFp8Config(), Eagle3Config(), calibration=torch.randint(0, 1024, (1, 64)),
                    decoding=eco.DecodeConfig(cycle_length=4))
    p = prompts((30,))[0].to(cuda)
    plain = eff.decode(p, 16, decoding=eco.DecodeConfig(cycle_length=1)).tokens
    spec = eff.decode(p, 16).tokens
    assert torch.equal(spec.cpu(), plain.cpu())


# ---- KIVI -----------------------------------------------------------------------------------------------------
def test_kivi_pack_roundtrip_error():
    from economize_b200.ops.kivi import dequant_chunks, pack_chunks

    g = torch.Generator().manual_seed(0)
    k = torch.randn(1, 2, 128, 128, generator=g).bfloat16()
    v = torch.randn(1, 2, 128, 128, generator=g).bfloat16()
    kk, vv = dequant_chunks(pack_chunks(k, v, 4), 4)
    assert (kk - k.float()).norm() / k.float().norm() < 0.12
    assert (vv - v.float()).norm() / v.float().norm() < 0.1


def test_kivi_model_decodes_losslessly():
    from economize_b200.techniques.kv_quant import KIVIConfig

    model = tiny_model()
    eff = eco.apply(model, KIVIConfig(bits=4, residual=16), Eagle3Config(), decoding=eco.DecodeConfig(cycle_length=4))
    p = prompts((300,))[0]
    spec = eff.decode(p, 8).tokens
    plain = eff.decode(p, 8, decoding=eco.DecodeConfig(cycle_length=1)).tokens
    assert torch.equal(spec, plain)
    tech = eff.techniques["kivi"]
    data, chunks = next(iter(tech._store.values()))
    assert int(chunks[0]) == (300 + 8 - 16) // 128  # the prompt's old chunks (and any that aged since) are coded


@pytest.mark.gpu
@pytest.mark.parametrize("bits", [2, 4])
def test_kivi_kernels_match_reference(cuda, bits):
    from economize_b200.ops.kivi import chunk_bytes

    g = torch.Generator(device=cuda).manual_seed(0)
    L, B, Hkv, S, D, H, T = 2, 2, 2, 512, 128, 8, 7
    cache = torch.randn(L, 2, B, Hkv, S, D, device=cuda, generator=g).bfloat16()
    kv_len = torch.tensor([400, 300], dtype=torch.int32, device=cuda)
    outs = {}
    for name, fn in (("kernel", ops.kivi_quantize), ("ref", ref.kivi_quantize)):
        kivi = torch.zeros(L, B, Hkv, S // 128, chunk_bytes(bits), dtype=torch.uint8, device=cuda)
        chunks = torch.zeros(B, dtype=torch.int32, device=cuda)
        fn(cache, kivi, kv_len, chunks, bits, 64, 8)
        outs[name] = (kivi, chunks)
    assert outs["kernel"][1].tolist() == [2, 1] == outs["ref"][1].tolist()
    assert torch.equal(outs["kernel"][0], outs["ref"][0])
    kivi, chunks = outs["kernel"]
    q = torch.randn(B, T, H, D, device=cuda, generator=g).bfloat16()
    n_new = torch.full((B,), T, dtype=torch.int32, device=cuda)
    for layer in range(L):
        k, v = cache[layer, 0], cache[layer, 1]
        got = ops.attention(q, k, v, kv_len, n_new, None, kivi=kivi[layer], kivi_chunks=chunks, kivi_bits=bits)
        exp = ref.attention(q.float(), k, v, kv_len, n_new, None, kivi=kivi[layer], kivi_chunks=chunks,
                            kivi_bits=bits)
        torch.testing.assert_close(got.float(), exp.float(), atol=2e-2, rtol=2e-2)
