"""Weight transforms: low-rank factorization, Hadamard rotation (exact invariance), FLAP width pruning, vendor MTP
heads and the distillation objectives."""

import pytest
import torch

import economize_b200 as eco
from economize_b200.techniques.eagle3 import Eagle3Config
from economize_b200.techniques.lowrank import LowRankConfig, LowRankWeight
from economize_b200.techniques.quant import QuantConfig
from economize_b200.techniques.rotate import RotateConfig, random_hadamard
from economize_b200.techniques.vendor_mtp import VendorMTPConfig
from economize_b200.techniques.width_prune import WidthPruneConfig
from economize_b200.train import fit

from .helpers import prompts, reference_greedy, tiny_model

CAL = torch.randint(0, 1024, (2, 32), generator=torch.Generator().manual_seed(6))


def _logits(model, p):
    return eco.EfficientModel(model, [], eco.DecodeConfig())(p[None])


def test_hadamard_is_orthogonal():
    for n in (256, 96):
        q = random_hadamard(n)
        torch.testing.assert_close(q @ q.t(), torch.eye(n), atol=1e-5, rtol=0)


def test_rotation_preserves_the_function():
    p = prompts((13,))[0]
    ref = _logits(tiny_model(), p)
    eff = eco.apply(tiny_model(), RotateConfig(seed=3))
    torch.testing.assert_close(eff(p[None]), ref, atol=2e-4, rtol=1e-4)


def test_rotation_then_quantization():
    p = prompts((13,))[0]
    ref = _logits(tiny_model(), p)
    eff = eco.apply(tiny_model(), RotateConfig(), QuantConfig(format="int4"))
    assert (eff(p[None]) - ref).norm() / ref.norm() < 0.5


@pytest.mark.parametrize("method", ["svd", "svd_llm"])
def test_lowrank(method):
    eff = eco.apply(tiny_model(), LowRankConfig(method=method, ratio=0.6), calibration=CAL)
    assert isinstance(eff.model.layers[0].wqkv, LowRankWeight)
    p = prompts((11,))[0]
    assert torch.equal(eff.decode(p, 6).tokens, reference_greedy(eff.model, p, 6))


def test_width_prune_shrinks_the_mlp():
    eff = eco.apply(tiny_model(), WidthPruneConfig(ratio=0.3), calibration=CAL)
    f = eff.model.layers[0].w_down.shape[1]
    assert f % 64 == 0 and f < 688 and eff.model.layers[0].w_gate_up.shape[0] == 2 * f
    p = prompts((11,))[0]
    assert torch.equal(eff.decode(p, 6).tokens, reference_greedy(eff.model, p, 6))


def test_vendor_mtp_drafts_losslessly_and_trains():
    model = tiny_model()
    eff = eco.apply(model, VendorMTPConfig())
    p = prompts((19,))[0]
    assert torch.equal(eff.decode(p, 10).tokens, reference_greedy(model, p, 10))
    fit(eff, torch.randint(0, 1024, (4, 24)), steps=2, batch_size=2)


@pytest.mark.parametrize("objective", ["distill_kl", "hass"])
def test_distillation_objectives(objective):
    eff = eco.apply(tiny_model(), Eagle3Config(train_steps=2))
    before = eff.techniques["eagle3"].fc.detach().clone()
    fit(eff, torch.randint(0, 1024, (4, 24)), objective=objective, steps=2, batch_size=2)
    assert not torch.equal(before, eff.techniques["eagle3"].fc)
