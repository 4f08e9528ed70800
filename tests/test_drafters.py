"""Every drafting technique is lossless under greedy verification (CPU fp32 oracle) and actually drafts."""

import pytest
import torch

import economize_b200 as eco
from economize_b200 import ops
from economize_b200.ops import reference
from economize_b200.techniques.draft_model import DraftModelConfig
from economize_b200.techniques.lookup import LookupConfig
from economize_b200.techniques.medusa import MEDUSA_TREES, MedusaConfig

from .helpers import prompts, tiny_model

TREE = {"depth": 6, "topk": 10, "total_tokens": 60}


@pytest.fixture(scope="module")
def model():
    return tiny_model()


@pytest.fixture(scope="module")
def plain(model):
    return eco.apply(model).decode_batch(prompts(), 32, decoding=eco.DecodeConfig(cycle_length=1))


@pytest.mark.parametrize("make,decoding", [
    (lambda m: LookupConfig(), eco.DecodeConfig(cycle_length=5)),
    (lambda m: LookupConfig(match="latest", max_ngram=2), eco.DecodeConfig(cycle_length=3)),
    (lambda m: MedusaConfig(num_heads=4, tree="mc_sim_7b_63"), None),
    (lambda m: MedusaConfig(num_heads=3), None),
    (lambda m: DraftModelConfig(model=tiny_model(num_layers=2)), eco.DecodeConfig(cycle_length=5)),
    (lambda m: DraftModelConfig(model=m), eco.DecodeConfig(cycle_length=7, draft_policy="dynamic_tree",
                                                             draft_policy_options=TREE)),
])
def test_lossless(model, plain, make, decoding):
    em = eco.apply(model, make(model))
    out = em.decode_batch(prompts(), 32, decoding=decoding)
    for a, b in zip(plain, out):
        assert torch.equal(a.tokens, b.tokens)
    assert max(r.mean_accepted_length for r in out) > 1.0


def test_self_draft_accepts(model, plain):
    """The target drafting for itself agrees with itself on every chain draft."""
    em = eco.apply(model, DraftModelConfig(model=model))
    out = em.decode_batch(prompts(), 32, decoding=eco.DecodeConfig(cycle_length=4))
    assert all(r.mean_accepted_length == pytest.approx(4.0, abs=0.2) for r in out)


def test_medusa_tree_table():
    paths = MEDUSA_TREES.get("mc_sim_7b_63")
    assert len(paths) == 63 and max(len(p) for p in paths) == 4
    with pytest.raises(eco.ConfigError):
        MedusaConfig(num_heads=2, tree="mc_sim_7b_63")
    with pytest.raises(eco.ConfigError):
        MedusaConfig(tree=((0, 1),))


def test_medusa_state_names(model):
    em = eco.apply(model, MedusaConfig(num_heads=2))
    names = set(em.techniques["medusa"].export_state())
    assert {"heads.0.blocks.0.linear.weight", "heads.0.blocks.0.linear.bias", "heads.1.proj.weight"} <= names


def test_ngram_reference():
    hist = torch.tensor([[5, 1, 2, 3, 9, 9, 1, 2, 3, 0], [1, 2, 3, 4, 5, 6, 7, 8, 0, 0]])
    length = torch.tensor([9, 8])
    out = reference.ngram(hist, length, 3, 1, 3)
    assert out[0].tolist() == [9, 9, 1]  # "1 2 3" first seen at 1, followed by 9 9 1
    assert out[1].tolist() == [-1, -1, -1]  # 8 never occurred before


def test_medusa_training_objective(model):
    from economize_b200.train import fit

    em = eco.apply(model, MedusaConfig(num_heads=2))
    data = torch.stack([torch.cat([p[:17], r]) for p, r in zip(prompts((17, 17)), [torch.arange(16)] * 2)])
    res = fit(em, data, steps=3, batch_size=2, seed=0, log_every=1)
    assert res.steps == 3 and "loss" in res.final
