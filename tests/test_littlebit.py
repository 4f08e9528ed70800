"""LittleBit: sign packing round trip, the bit budget, Dual-SVID with residual compensation beating one path, a
decoding model under the technique, its saved factors, and the CUDA sign products against fp32."""

import pytest
import torch

import economize_b200 as eco
from economize_b200.ops.littlebit import LittleBitWeight, pack_signs, unpack_signs
from economize_b200.techniques.littlebit import LittleBitConfig, littlebit_factors, rank_for_bpw

from .helpers import prompts, tiny_model


def test_pack_roundtrip():
    x = torch.randn(5, 70)
    assert torch.equal(unpack_signs(pack_signs(x), 70), torch.where(x < 0, -1.0, 1.0))


def test_bit_budget():
    assert rank_for_bpw(4096, 4096, 0.55, paths=2) == 546  # the paper's rank at this budget
    assert rank_for_bpw(64, 64, 0.1) == 0


def test_residual_path_helps():
    g = torch.Generator().manual_seed(0)
    w = torch.randn(128, 96, generator=g) @ torch.randn(96, 96, generator=g) / 10
    one = LittleBitWeight(*littlebit_factors(w, 32, False), torch.float32).dequantize(torch.float32)
    two = LittleBitWeight(*littlebit_factors(w, 32, True), torch.float32).dequantize(torch.float32)
    assert (w - two).norm() < (w - one).norm() < w.norm()


def test_littlebit_model_decodes_and_reloads(tmp_path):
    m = tiny_model()
    em = eco.apply(m, LittleBitConfig(bpw=1.0, rank_multiple=8))
    tech = em.techniques["littlebit"]
    assert tech.bits_per_weight() <= 1.0 + 1e-6
    out = em.decode(prompts((12,))[0], 6).tokens
    assert out.numel() == 6
    em.save_pretrained(tmp_path)
    again = eco.load(tiny_model(), tmp_path)
    x = torch.randn(3, 256)
    a = em.model.layers[0].wqkv.linear(x)
    b = again.model.layers[0].wqkv.linear(x)
    torch.testing.assert_close(a, b)


@pytest.mark.gpu
@pytest.mark.parametrize("M", [1, 3, 16])
def test_sign_products_match_dense(cuda, M):
    g = torch.Generator().manual_seed(M)
    w = torch.randn(512, 384, generator=g)
    lw = LittleBitWeight(*littlebit_factors(w, 64, True), torch.bfloat16).to(cuda)
    x = torch.randn(M, 384, device=cuda).bfloat16()
    ref = x.float() @ lw.dequantize(torch.float32).t()
    torch.testing.assert_close(lw.linear(x).float(), ref, atol=0.05 * float(ref.abs().max()), rtol=0.02)


def test_smooth_sign_gradient_and_qat_lowers_output_error():
    from economize_b200.techniques.littlebit import LittleBitConfig
    from economize_b200.techniques.littlebit.qat import smooth_sign

    x = torch.tensor([-0.5, -0.001, 0.0, 0.001, 0.5], requires_grad=True)
    y = smooth_sign(x, 100.0)
    assert y.tolist() == [-1.0, -1.0, 1.0, 1.0, 1.0]
    y.sum().backward()
    expect = 100.0 * (1 - torch.tanh(100.0 * x.detach()) ** 2)
    assert torch.allclose(x.grad, expect)
    cal = torch.randint(0, 1024, (2, 48), generator=torch.Generator().manual_seed(2))
    cfg = LittleBitConfig(bpw=1.0, layers=(1,), targets=("w_down",), rank_multiple=8, qat_steps=25, qat_lr=1e-3,
                          calibration_tokens=96)
    em = eco.apply(tiny_model(), cfg, calibration=cal)
    report = em.techniques["littlebit"].qat_report
    assert list(report) == ["0:w_down"]
    before, after = report["0:w_down"]
    assert after < before
    p = prompts((17,))[0]
    assert em.decode(p, 6, decoding=eco.DecodeConfig(cycle_length=1)).tokens.numel() == 6
