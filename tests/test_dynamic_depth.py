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
