"""Cost logs of generations (economize ``decoding/cost.py``): the engine turns its per-cycle acceptance history
into one event per model call with positions, and the summary compares layer applications with plain decoding."""

import torch

import economize_b200 as eco
from economize_b200.decoding.cost import CostKind, CostLog, LayerFootprint
from economize_b200.techniques.eagle3 import Eagle3Config

from .helpers import prompts, tiny_model


def test_plain_log_counts_one_call_per_token():
    em = eco.apply(tiny_model())
    ps = prompts()
    for p, r in zip(ps, em.decode_batch(ps, 10, decoding=eco.DecodeConfig(cycle_length=1))):
        log = r.cost
        assert log.count(CostKind.EXACT) == 1 + r.cycles == 10  # the prefill makes the first token
        assert [e.position for e in log.events] == [0] + list(range(p.numel(), p.numel() + 9))
        s = log.summary(4, p.numel(), 10)
        assert s["relative_layer_tokens"] == 1.0 and s["draft_steps"] == 0


def test_tree_log_follows_the_accepted_history():
    em = eco.apply(tiny_model(), Eagle3Config())
    em.techniques["eagle3"].reset_parameters(seed=2)
    ps = prompts()
    cfg = eco.DecodeConfig(cycle_length=5, draft_policy="dynamic_tree",
                           draft_policy_options={"depth": 4, "topk": 4, "total_tokens": 16})
    for p, r in zip(ps, em.decode_batch(ps, 20, decoding=cfg)):
        log = r.cost
        exact = [e for e in log.events if e.kind == CostKind.EXACT]
        assert len(exact) == 1 + r.cycles
        assert all(e.tokens == 17 for e in exact[1:])
        assert log.count(CostKind.DRAFT) == 3 * r.cycles and log.count(CostKind.DRAFT_OBSERVE) == r.cycles
        # each verification starts where the previous cycle's accepted tokens end
        gaps = [b.position - a.position for a, b in zip(exact[1:], exact[2:])]
        obs = [e.tokens - 1 for e in log.events if e.kind == CostKind.DRAFT_OBSERVE]
        assert gaps == obs[:-1]
        assert sum(t - 1 for t in obs) == r.accepted
        s = log.summary(4, p.numel(), r.tokens.numel())
        assert s["exact_calls"] == 1 + r.cycles and "eagle3" in s["module_layer_tokens"]


def test_footprints_and_tuples():
    assert LayerFootprint.of([3, 1, 2]) == LayerFootprint(1, 3)
    assert LayerFootprint.of([1, 3]).layers == (1, 3)
    log = CostLog()
    log.record_footprint(CostKind.DRAFT, 2, 5, LayerFootprint.of([1, 3], module="m"), step=1)
    log.mark_last_wasted()
    assert log.events[0].kind == "draft_wasted" and log.events[0].layer_tokens == 4
    assert log.as_tuples({"draft_wasted": "w"}) == [("w", 2, 5)]
