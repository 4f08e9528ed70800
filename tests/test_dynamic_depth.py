"""Dynamic depth: each policy at its identity setting reproduces the model, skips when configured to (counted by
the device meter), its objective trains, and the drafting-cycle methods (FREE, DMTD, Hidden Transfer) decode."""

import pytest
import torch

import economize_b200 as eco
from economize_b200.techniques.dynamic_depth import (CalmConfig, DmtdConfig, FlexiDepthConfig, FreeConfig,
                                                     GateSkipConfig, HiddenTransferConfig, LoRADropConfig, MoDConfig,
                                                     SkipDecodeConfig)
from economize_b200.train.objective import OBJECTIVES

from .helpers import prompts, tiny_model

CAL = torch.randint(0, 1024, (2, 24), generator=torch.Generator().manual_seed(3))


@pytest.fixture(scope="module")
def plain():
    return eco.apply(tiny_model()).decode_batch(prompts(), 12, decoding=eco.DecodeConfig(cycle_length=1))


@pytest.mark.parametrize("cfg", [
    GateSkipConfig(gate_bias=100.0), MoDConfig(), SkipDecodeConfig(), CalmConfig(threshold=1.0),
    LoRADropConfig(period=1, layers=(2, 3)), FlexiDepthConfig(router_bias=100.0),
    CalmConfig(threshold=1.0, confidence="state"),
])
def test_identity_settings_reproduce_the_model(plain, cfg):
    em = eco.apply(tiny_model(), cfg)
    out = em.decode_batch(prompts(), 12, decoding=eco.DecodeConfig(cycle_length=1))
    for a, b in zip(plain, out):
        assert torch.equal(a.tokens, b.tokens), cfg.technique
    stats = em.techniques[cfg.technique].depth_stats()
    assert stats["layer_tokens_entered"] > 0


@pytest.mark.parametrize("cfg,expect", [
    (GateSkipConfig(gate_bias=0.0, threshold=0.9), 0.0),  # every gate is 0.5 < 0.9: every gated layer skipped
    (SkipDecodeConfig(max_layers=4, min_layers=1, warmup=0, decay=1), 10 / 28),  # 4 layers at t = 0, then 1
    (CalmConfig(confidence="state", threshold=1e-3, min_layer=1), 0.25),
])
def test_skipping_is_counted(cfg, expect):
    em = eco.apply(tiny_model(), cfg)
    em.decode_batch(prompts(), 8, decoding=eco.DecodeConfig(cycle_length=1))
    stats = em.techniques[cfg.technique].depth_stats()
    assert stats["run_fraction"] == pytest.approx(expect, abs=0.05), stats


@pytest.mark.parametrize("cfg", [GateSkipConfig(gate_bias=2.0), MoDConfig(), FlexiDepthConfig(router_bias=2.0),
                                 LoRADropConfig(layers=(2, 3))])
def test_depth_objectives_train(cfg):
    em = eco.apply(tiny_model(), cfg)
    obj = OBJECTIVES.get(cfg.technique)(em)
    params = obj.parameters()
    assert params
    opt = torch.optim.Adam(params, lr=2e-3)
    losses = []
    for _ in range(8):
        loss, _ = obj.loss(CAL)
        opt.zero_grad()
        loss.backward()
        opt.step()
        losses.append(float(loss.detach()))
    assert min(losses[1:]) < losses[0] or losses[-1] < losses[1], losses


def test_calm_classifier_objective():
    em = eco.apply(tiny_model(), CalmConfig(confidence="classifier", threshold=0.9))
    obj = OBJECTIVES.get("calm")(em)
    opt = torch.optim.Adam(obj.parameters(), lr=1e-2)
    first = None
    for _ in range(10):
        loss, _ = obj.loss(CAL)
        opt.zero_grad()
        loss.backward()
        opt.step()
        first = first if first is not None else float(loss.detach())
    assert float(loss.detach()) < first


def test_hidden_transfer_is_lossless_and_trains(plain):
    model = tiny_model()
    em = eco.apply(model, HiddenTransferConfig(transfer_layers=(1, 2, 3)))
    out = em.decode_batch(prompts(), 12)
    for a, b in zip(plain, out):
        assert torch.equal(a.tokens, b.tokens)
    obj = OBJECTIVES.get("hidden_transfer_kl")(em)
    opt = torch.optim.Adam(obj.parameters(), lr=1e-3)
    losses = []
    for _ in range(4):
        loss, _ = obj.loss(CAL)
        opt.zero_grad()
        loss.backward()
        opt.step()
        losses.append(float(loss.detach()))
    assert losses[-1] < losses[0]


@pytest.mark.parametrize("cfg", [FreeConfig(exit_layer=2, threshold=1e-6), DmtdConfig(decoding_layers=2)])
def test_drafting_depth_methods_decode(cfg):
    em = eco.apply(tiny_model(), cfg)
    out = em.decode_batch(prompts(), 12)
    assert all(r.tokens.numel() == 12 for r in out)
    assert sum(r.accepted for r in out) > 0  # drafts are kept (lossy methods)


def test_depth_configs_validate():
    with pytest.raises(eco.ConfigError):
        MoDConfig(kv="routed")
    with pytest.raises(eco.ConfigError):
        eco.apply(tiny_model(), CalmConfig(min_layer=4))
    with pytest.raises(eco.IncompatibleTechniquesError):
        eco.apply(tiny_model(), GateSkipConfig(), MoDConfig())


@pytest.mark.gpu
@pytest.mark.parametrize("cfg", [CalmConfig(confidence="state", threshold=0.5), GateSkipConfig(gate_bias=0.5),
                                 SkipDecodeConfig(max_layers=2, min_layers=1, decay=4),
                                 LoRADropConfig(layers=(1,), period=2), HiddenTransferConfig(transfer_layers=(1,))])
def test_depth_methods_run_in_cuda_graphs(cuda, cfg):
    from .helpers import gpu_tiny_model

    model = gpu_tiny_model(cuda)
    ps = [p.to(cuda) for p in prompts((17, 30))]
    base = eco.apply(gpu_tiny_model(cuda)).decode_batch(ps, 10, decoding=eco.DecodeConfig(cycle_length=1))
    em = eco.apply(model, cfg)
    out = em.decode_batch(ps, 10, decoding=eco.DecodeConfig(cycle_length=1 if cfg.technique != "hidden_transfer"
                                                            else 2, cuda_graphs=True))
    assert all(r.tokens.numel() == 10 for r in out)
    if cfg.technique == "hidden_transfer":  # verified drafts: the model's own tokens
        assert all(torch.equal(a.tokens.cpu(), b.tokens.cpu()) for a, b in zip(base, out))
    else:
        assert em.techniques[cfg.technique].depth_stats()["layer_tokens_entered"] > 0


def test_hoeffding_bentkus_and_fixed_sequence_testing():
    from economize_b200.techniques.dynamic_depth import hoeffding_bentkus_pvalue, ltt_threshold, token_mismatch

    assert hoeffding_bentkus_pvalue(0.0, 200, 0.1) < 1e-6  # no loss on many examples: risk > 0.1 is implausible
    assert hoeffding_bentkus_pvalue(0.2, 200, 0.1) == 1.0  # mean above epsilon: cannot reject
    ps = [hoeffding_bentkus_pvalue(m, 100, 0.2) for m in (0.0, 0.05, 0.1, 0.15)]
    assert ps == sorted(ps)  # a larger mean loss gives a larger p-value
    cands = [0.2, 0.4, 0.6, 0.8]
    losses = [[0.5] * 100, [0.0] * 100, [0.0] * 100, [0.0] * 100]  # 0.2 fails; 0.4 and above pass
    assert ltt_threshold(cands, losses, delta=0.05, epsilon=0.1) == 0.4
    gap = [[0.0] * 100, [0.5] * 100, [0.0] * 100, [0.0] * 100]  # the walk stops at the first failure (0.4)
    assert ltt_threshold(cands, gap, delta=0.05, epsilon=0.1) == 0.6
    assert ltt_threshold(cands, [[0.5] * 10] * 4, delta=0.05, epsilon=0.1) == 1.0
    assert token_mismatch(torch.tensor([1, 2, 3]), torch.tensor([1, 5, 3, 4])) == 0.5


def test_calm_calibration_restores_config_and_certifies():
    from economize_b200.techniques.dynamic_depth import calibrate_threshold

    em = eco.apply(tiny_model(), CalmConfig(confidence="state", threshold=0.3))
    lam = calibrate_threshold(em, prompts(), 8, delta=0.2, epsilon=0.5, candidates=(0.5, 0.9, 0.999))
    assert lam in (0.5, 0.9, 0.999, 1.0)
    assert em.techniques["calm"].config.threshold == 0.3


def test_free_beta_mixture_threshold():
    from economize_b200.techniques.dynamic_depth import beta_moments, bmm_threshold, free_calibration_pairs

    g = torch.Generator().manual_seed(0)
    a, b = beta_moments(torch.distributions.Beta(torch.tensor(8.0), torch.tensor(2.0)).sample((20000,)))
    assert abs(a - 8.0) < 0.5 and abs(b - 2.0) < 0.2
    conf = torch.cat([torch.rand(500, generator=g) * 0.5, 0.5 + torch.rand(500, generator=g) * 0.5])
    agree = torch.arange(1000) >= 500  # confident tokens agree, unsure ones do not
    lam = bmm_threshold(conf, agree, posterior=0.5)
    assert 0.35 <= lam <= 0.65
    assert bmm_threshold(conf, torch.ones(1000, dtype=torch.bool)) == 0.9  # one class only: the default
    em = eco.apply(tiny_model(), FreeConfig(exit_layer=2))
    c, ok = free_calibration_pairs(em, prompts()[0][None])
    assert c.shape == ok.shape == (17,) and bool(((c >= 0) & (c <= 1)).all())
