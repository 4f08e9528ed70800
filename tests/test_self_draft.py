"""Self-drafting sub-network drafters (layer_skip, early_exit, kangaroo, knapspec): views share the target's
weights, searches pick sensible layers, and decoding stays lossless."""

import pytest
import torch

import economize_b200 as eco
from economize_b200.techniques._self_draft import block_influence, layer_view
from economize_b200.techniques.early_exit import EarlyExitConfig
from economize_b200.techniques.kangaroo import KangarooConfig
from economize_b200.techniques.knapspec import KnapSpecConfig, knapsack_keep
from economize_b200.techniques.layer_skip import LayerSkipConfig

from .helpers import prompts, reference_greedy, tiny_model

CAL = torch.randint(0, 1024, (2, 24), generator=torch.Generator().manual_seed(5))


def test_full_view_equals_target():
    model = tiny_model()
    view = layer_view(model, range(4))
    p = prompts((13,))[0]
    a = eco.EfficientModel(model, [], eco.DecodeConfig())(p[None])
    b = eco.EfficientModel(view, [], eco.DecodeConfig())(p[None])
    assert torch.equal(a, b)
    assert view.layers[0].wqkv is model.layers[0].wqkv  # shared, not copied


def test_skipping_both_sublayers_is_dropping_the_layer():
    model = tiny_model()
    p = prompts((9,))[0][None]
    a = eco.EfficientModel(layer_view(model, [0, (1, True, True), 2, 3]), [], eco.DecodeConfig())(p)
    b = eco.EfficientModel(layer_view(model, [0, 2, 3]), [], eco.DecodeConfig())(p)
    torch.testing.assert_close(a, b)


def test_block_influence_shape():
    bi = block_influence(tiny_model(), [CAL])
    assert bi.shape == (4,) and (bi >= 0).all()


@pytest.mark.parametrize("config", [LayerSkipConfig(skip=(2,)), LayerSkipConfig(search="influence", ratio=0.3),
                                    LayerSkipConfig(search="greedy", ratio=0.3),
                                    LayerSkipConfig(search="interleave", ratio=0.3), EarlyExitConfig(exit_layer=2),
                                    KangarooConfig(exit_layer=1), KnapSpecConfig(budget=0.6)])
def test_self_drafters_are_lossless(config):
    model = tiny_model()
    eff = eco.apply(model, config, calibration=CAL, decoding=eco.DecodeConfig(cycle_length=4))
    p = prompts((19,))[0]
    out = eff.decode(p, 12)
    assert torch.equal(out.tokens, reference_greedy(model, p, 12))


def test_layer_skip_search_respects_edges():
    eff = eco.apply(tiny_model(), LayerSkipConfig(search="influence", ratio=0.5), calibration=CAL)
    tech = eff.techniques["layer_skip"]
    _ = tech.view
    assert tech.skipped and 0 not in tech.skipped and 3 not in tech.skipped


def test_knapsack():
    keep = knapsack_keep([5.0, 4.0, 3.0], [4.0, 3.0, 2.0], 5.0, 100)
    assert keep == [False, True, True]


def test_kangaroo_adapter_trains():
    from economize_b200.train import fit

    model = tiny_model()
    eff = eco.apply(model, KangarooConfig(exit_layer=1))
    before = [p.detach().clone() for p in eff.techniques["kangaroo"].adapter.parameters()]
    data = torch.randint(0, 1024, (8, 32), generator=torch.Generator().manual_seed(1))
    fit(eff, data, steps=3, batch_size=4)
    after = list(eff.techniques["kangaroo"].adapter.parameters())
    assert any(not torch.equal(a, b) for a, b in zip(before, after))
    assert model.layers[1].wqkv is not eff.techniques["kangaroo"].adapter[0].wqkv


@pytest.mark.parametrize("adaptation", ["lora", "full"])
def test_early_exit_readout_adaptation_trains_and_stays_lossless(adaptation):
    from economize_b200.techniques.early_exit import EarlyExitConfig
    from economize_b200.train.objective import OBJECTIVES

    model = tiny_model()
    plain = eco.apply(model).decode_batch(prompts(), 16, decoding=eco.DecodeConfig(cycle_length=1))
    em = eco.apply(model, EarlyExitConfig(exit_layer=2, adaptation=adaptation))
    obj = OBJECTIVES.get("layerskip")(em)
    cal = torch.randint(0, 1024, (2, 32), generator=torch.Generator().manual_seed(0))
    opt = torch.optim.Adam(obj.parameters(), lr=3e-3)
    losses = []
    for _ in range(6):
        loss, _ = obj.loss(cal)
        opt.zero_grad()
        loss.backward()
        opt.step()
        losses.append(float(loss.detach()))
    assert losses[-1] < losses[0]
    out = em.decode_batch(prompts(), 16, decoding=eco.DecodeConfig(cycle_length=4))
    for a, b in zip(plain, out):
        assert torch.equal(a.tokens, b.tokens)
