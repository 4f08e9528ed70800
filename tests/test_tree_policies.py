"""Sequoia static trees and SpecExec search (economize ``tests/test_sequoia.py`` and ``tests/test_specexec.py``):
the best-first tree search against exhaustive search, the options' checks, acceptance recording, and lossless decoding on
the CPU fp32 path (both policies must reproduce plain greedy decoding)."""

import itertools

import pytest
import torch

import economize_b200 as eco
from economize_b200.decoding.policies import SequoiaPolicy
from economize_b200.decoding.sequoia import (AcceptanceProfile, StaticTree, expected_tokens, measure_acceptance,
                                             probe_paths, sequoia_tree)
from economize_b200.decoding.specexec import SearchOptions
from economize_b200.errors import ConfigError
from economize_b200.techniques.eagle3 import Eagle3Config

from .helpers import prompts, tiny_model

RATES = (0.6, 0.15, 0.06, 0.03)


def _all_trees(nodes: int, depth: int, ranks: int):
    """Every rank tree (closed under parents) of at most ``nodes`` nodes and depth ``depth`` (small cases only)."""
    universe = [p for L in range(1, depth + 1) for p in itertools.product(range(ranks), repeat=L)]
    for n in range(1, nodes + 1):
        for combo in itertools.combinations(universe, n):
            have = set(combo)
            if all(len(p) == 1 or p[:-1] in have for p in combo):
                yield combo


@pytest.mark.parametrize("nodes,depth", [(3, 2), (5, 3), (6, 2)])
def test_best_first_matches_exhaustive_search(nodes, depth):
    rates = (0.5, 0.2, 0.1)
    best = max(expected_tokens(t, rates) for t in _all_trees(nodes, depth, 3))
    tree = sequoia_tree(rates, nodes, depth)
    assert tree.size <= nodes and tree.depth <= depth
    assert tree.expected == pytest.approx(best)
    assert expected_tokens(tree, rates) == pytest.approx(best)


def test_best_first_per_depth_rates_and_gaps():
    per_depth = ((0.9, 0.05), (0.2, 0.3))  # after the root: confident; below: the 2nd rank is the likelier one
    best = max(expected_tokens(t, per_depth) for t in _all_trees(4, 3, 2))
    assert sequoia_tree(per_depth, 4, 3).expected == pytest.approx(best)
    skip = sequoia_tree((0.0, 0.5), 2, 2)  # rank 0 never matches: the tree leaves it out
    assert all(0 not in p for p in skip.paths)


def test_latency_aware_choice_prefers_smaller_trees_when_passes_are_costly():
    flat = sequoia_tree(RATES, 32, 6)
    steep = sequoia_tree(RATES, 32, 6, verify_latency=[1.0 + 0.2 * i for i in range(33)], draft_latency=0.05)
    assert steep.size < flat.size
    assert flat.expected > expected_tokens(StaticTree.from_paths([(0,) * d for d in range(1, 7)]), RATES)


def test_static_tree_and_profile():
    tree = StaticTree.from_paths([(1,), (0,), (0, 0)])
    assert tree.paths == ((0,), (1,), (0, 0)) and tree.parents == (-1, -1, 0) and tree.forwarded == 1
    assert probe_paths(2, 3) == ((0,), (1,), (2,), (0, 0), (0, 1), (0, 2))
    prof = AcceptanceProfile()
    prof.add(0, [0, 1, 2], 1)
    prof.add(0, [0, 1], None)
    prof.add(1, [0], 0)
    assert prof.rates() == pytest.approx((1 / 3, 0.5, 0.0))
    assert prof.rates(per_depth=True)[1] == pytest.approx((1.0, 0.0, 0.0))


@pytest.mark.parametrize("options,match", [
    ({}, "needs a tree"),
    ({"acceptance": RATES, "paths": [(0,)]}, "not both"),
    ({"paths": [(0, 1)]}, "not in the tree"),
    ({"paths": [(0,)], "depth": 3}, "explicit"),
    ({"acceptance": (0.7, 0.5)}, "sum to at"),
    ({"acceptance": RATES, "draft_latency": 0.1}, "next to verify_latency"),
    ({"acceptance": RATES, "total_tokens": 80}, "at most 63"),
    ({"acceptance": RATES, "bogus": 1}, "unknown sequoia option"),
])
def test_sequoia_options_are_checked(options, match):
    with pytest.raises(ConfigError, match=match):
        SequoiaPolicy(eco.DecodeConfig(cycle_length=5, draft_policy="sequoia", draft_policy_options=options))


@pytest.mark.parametrize("options,match", [
    ({"width": 9, "topk": 8}, "exceeds topk"),
    ({"decay": 0.0}, "decay"),
    ({"depth": 10, "width": 8}, "64-bit"),
    ({"depth": 2, "width": 1, "topk": 2, "total_tokens": 10}, "exceeds the 4 candidates"),
    ({"topk": 20, "width": 4}, "at most 16"),
])
def test_specexec_options_are_checked(options, match):
    with pytest.raises(ConfigError, match=match):
        SearchOptions.from_options(options, 8)


@pytest.fixture(scope="module")
def em():
    return eco.apply(tiny_model(), Eagle3Config())


@pytest.fixture(scope="module")
def plain(em):
    return em.decode_batch(prompts(), 32, decoding=eco.DecodeConfig(cycle_length=1))


@pytest.mark.parametrize("options", [
    {"acceptance": RATES, "total_tokens": 24, "depth": 5},
    {"acceptance": ((0.5, 0.2), (0.6, 0.1, 0.05)), "total_tokens": 12, "depth": 4},
    {"paths": [(0,), (1,), (0, 0), (0, 1), (1, 0), (0, 0, 0)]},
])
def test_sequoia_is_lossless(em, plain, options):
    cfg = eco.DecodeConfig(cycle_length=6, draft_policy="sequoia", draft_policy_options=options)
    for a, b in zip(plain, em.decode_batch(prompts(), 32, decoding=cfg)):
        assert torch.equal(a.tokens, b.tokens)


@pytest.mark.parametrize("options", [
    {"depth": 5, "width": 4, "topk": 4, "total_tokens": 20},
    {"depth": 8, "width": 8, "topk": 8, "total_tokens": 60, "decay": 0.9},
    {"depth": 2, "width": 1, "topk": 3, "total_tokens": 4, "decay": 1.0},
])
def test_specexec_is_lossless(em, plain, options):
    cfg = eco.DecodeConfig(cycle_length=options["depth"] + 1, draft_policy="specexec", draft_policy_options=options)
    for a, b in zip(plain, em.decode_batch(prompts(), 32, decoding=cfg)):
        assert torch.equal(a.tokens, b.tokens)


def test_measure_acceptance_feeds_sequoia(em, plain):
    rates = measure_acceptance(em, prompts()[:2], 16, depth=3, width=4)
    assert len(rates) == 4 and all(0.0 <= r <= 1.0 for r in rates) and sum(rates) <= 1.0 + 1e-6
    per = measure_acceptance(em, prompts()[:2], 16, depth=3, width=4, per_depth=True)
    assert len(per) >= 1 and all(len(row) == 4 for row in per)
    if sum(rates) > 0:
        cfg = eco.DecodeConfig(cycle_length=5, draft_policy="sequoia",
                               draft_policy_options={"acceptance": rates, "total_tokens": 16, "depth": 4})
        for a, b in zip(plain, em.decode_batch(prompts(), 32, decoding=cfg)):
            assert torch.equal(a.tokens, b.tokens)


def test_oracle_drafter_fills_the_deepest_path():
    """With a drafter that always agrees with the target, every cycle accepts the tree's rank-0 spine."""
    model = tiny_model()
    with torch.no_grad():
        for layer in model.layers:
            layer.wo.zero_()
            layer.w_down.zero_()
        model.lm_head.copy_(model.embed * 30)
    em = eco.apply(model, Eagle3Config())
    em.techniques["eagle3"].reset_parameters(seed=1, identity=True)
    ps = prompts()
    seq = eco.DecodeConfig(cycle_length=6, draft_policy="sequoia",
                           draft_policy_options={"acceptance": (0.9, 0.05), "total_tokens": 12, "depth": 5})
    spx = eco.DecodeConfig(cycle_length=6, draft_policy="specexec",
                           draft_policy_options={"depth": 5, "width": 2, "topk": 2, "total_tokens": 8})
    for cfg in (seq, spx):
        for p, r in zip(ps, em.decode_batch(ps, 30, decoding=cfg)):
            assert torch.equal(r.tokens, p[-1].repeat(30))
            assert r.mean_accepted_length == pytest.approx(6, abs=0.01)


def test_policies_need_tree_steps():
    from economize_b200.techniques.medusa import MedusaConfig

    med = eco.apply(tiny_model(), MedusaConfig())
    with pytest.raises(ConfigError, match="tree steps"):
        med.decode_batch(prompts()[:1], 4, decoding=eco.DecodeConfig(
            cycle_length=4, draft_policy="specexec", draft_policy_options={"width": 2, "topk": 2, "total_tokens": 8}))
