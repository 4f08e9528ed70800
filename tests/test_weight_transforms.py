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


def test_block_hadamard_reference_is_the_sylvester_transform():
    from economize_b200.ops import reference

    h = torch.ones(1, 1)
    while h.shape[0] < 32:
        h = torch.cat([torch.cat([h, h], 1), torch.cat([h, -h], 1)], 0)
    x = torch.randn(5, 96, dtype=torch.float64)
    want = (x.view(5, 3, 32) @ (h.double() / 32 ** 0.5)).view(5, 96)
    torch.testing.assert_close(reference.hadamard(x, 32).double(), want, atol=1e-5, rtol=1e-5)
    with pytest.raises(ValueError):
        reference.hadamard(x, 64)


@pytest.mark.parametrize("kw", [dict(), dict(residual=False), dict(residual=False, values=False),
                                dict(online=(), residual=False), dict(seed=None, block=8, layers=(1, 3))])
def test_each_rotation_preserves_the_function(kw):
    p = prompts((13,))[0]
    ref = _logits(tiny_model(), p)
    eff = eco.apply(tiny_model(), RotateConfig(**kw))
    cfg = eff.techniques["rotate"].config
    want = [0] * 4 if not cfg.online else [(min(cfg.block or 16, 16) if not cfg.layers or i + 1 in cfg.layers else 0)
                                           for i in range(4)]
    assert [layer.down_hadamard for layer in eff.model.layers] == want
    torch.testing.assert_close(eff(p[None]), ref, atol=2e-4, rtol=1e-4)
    assert torch.equal(eff.decode(p, 6).tokens, reference_greedy(eff.model, p, 6))


def test_rotate_config_checks():
    for kw, why in ((dict(online=("mlp.up_proj",)), "online rotations"), (dict(block=12), "power of two"),
                    (dict(online=(), values=False, residual=False), "rotates nothing"), (dict(layers=(0,)), "1-indexed"),
                    (dict(seed=True), "seed")):
        with pytest.raises(eco.ConfigError, match=why):
            RotateConfig(**kw)
    from economize_b200.techniques.rotate import online_block

    assert (online_block(14336), online_block(14336, 512), online_block(28672 * 4), online_block(688)) == \
        (2048, 512, 8192, 16)


def test_online_rotation_exports_an_unrotated_down_projection():
    from economize_b200.models.hf import export_hf_state as to_hf_state

    p = prompts((13,))[0]
    eff = eco.apply(tiny_model(), RotateConfig(residual=False, values=False))
    base = tiny_model()
    got = to_hf_state(eff.model)
    want = to_hf_state(base)
    torch.testing.assert_close(got["model.layers.0.mlp.down_proj.weight"], want["model.layers.0.mlp.down_proj.weight"],
                               atol=1e-6, rtol=1e-5)
    del p


def test_online_rotation_refuses_activation_sparse_mlps():
    from economize_b200.techniques.mlp_sparsity import CatsConfig as CATSConfig

    for configs in ((RotateConfig(), CATSConfig()), (CATSConfig(), RotateConfig())):  # weights attach first
        with pytest.raises(eco.ConfigError, match="online-rotated"):
            eco.apply(tiny_model(), *configs, calibration=CAL)
    eco.apply(tiny_model(), RotateConfig(online=()), CATSConfig(backend="dense"), calibration=CAL)
