"""EAGLE-1/2 (eagle) drafting and training, and FR-Spec head restriction around EAGLE-3."""

import torch

import economize_b200 as eco
from economize_b200.techniques.eagle import EagleConfig
from economize_b200.techniques.eagle3 import Eagle3Config
from economize_b200.techniques.frspec import FRSpecConfig, frequent_tokens
from economize_b200.train import fit

from .helpers import prompts, reference_greedy, tiny_model


def test_eagle_chain_and_tree_are_lossless():
    model = tiny_model()
    eff = eco.apply(model, EagleConfig())
    p = prompts((23,))[0]
    ref = reference_greedy(model, p, 12)
    assert torch.equal(eff.decode(p, 12).tokens, ref)
    tree = eco.DecodeConfig(cycle_length=5, draft_policy="dynamic_tree",
                            draft_policy_options={"depth": 3, "topk": 3, "total_tokens": 8})
    assert torch.equal(eff.decode(p, 12, decoding=tree).tokens, ref)


def test_eagle_identity_init_drafts_the_previous_feature():
    model = tiny_model()
    eff = eco.apply(model, EagleConfig())
    eff.techniques["eagle"].reset_parameters(identity=True)
    out = eff.decode(prompts((15,))[0], 8)
    assert out.tokens.numel() == 8


def test_eagle_feature_objective_trains():
    model = tiny_model()
    eff = eco.apply(model, EagleConfig())
    data = torch.randint(0, 1024, (8, 24), generator=torch.Generator().manual_seed(2))
    hist = fit(eff, data, steps=4, batch_size=4)
    assert hist is not None


def test_frspec_restricts_eagle3_head():
    model = tiny_model()
    cal = torch.randint(0, 200, (4, 64), generator=torch.Generator().manual_seed(0))
    eff = eco.apply(model, Eagle3Config(), FRSpecConfig(vocab_size=256), calibration=cal)
    tech = eff.techniques["eagle3"]
    assert tech.lm_head.shape[0] == 256 and int(tech.t2d.sum()) == 256
    ids = torch.arange(256) + tech.d2t.cpu()
    assert set(ids.tolist()) == set(frequent_tokens(cal, 1024, 256).tolist())
    p = prompts((18,))[0]
    assert torch.equal(eff.decode(p, 10).tokens, reference_greedy(model, p, 10))
