"""Speculative sampling is lossless: the joint distribution of the first two generated tokens equals the target's
own sampling distribution (exact enumeration over a 16-token vocabulary), for rejection sampling of chains and for
sampled-match verification of trees; the fused accept/resample rule matches its reference on fixed uniforms."""

import pytest
import torch

import economize_b200 as eco
from economize_b200 import ops
from economize_b200.decoding import TopPSampler
from economize_b200.runtime.cache import StepBatch
from economize_b200.techniques.eagle3 import Eagle3Config

from .helpers import micro_model

V = 16
TEMP = 1.0


@torch.no_grad()
def exact_joint(model, prompt):
    """p(x1, x2 | prompt) by enumeration."""
    def next_probs(seq):
        n = seq.numel()
        cache = model.new_cache(1, 128)
        h, _ = model.forward_step(seq[None], StepBatch.prefill(torch.tensor([n], dtype=torch.int32), n), cache)
        return torch.softmax(model.logits(h[0, -1]).float() / TEMP, -1)

    p1 = next_probs(prompt)
    joint = torch.zeros(V, V)
    for a in range(V):
        joint[a] = p1[a] * next_probs(torch.cat([prompt, torch.tensor([a])]))
    return joint


def empirical_joint(em, prompt, cfg, n=3000, seed=0):
    torch.manual_seed(seed)
    out = em.decode_batch([prompt] * n, 2, decoding=cfg, selector=TopPSampler(temperature=TEMP))
    counts = torch.zeros(V, V)
    for r in out:
        counts[int(r.tokens[0]), int(r.tokens[1])] += 1
    return counts / n


@pytest.fixture(scope="module")
def setup():
    model = micro_model(V)
    em = eco.apply(model, Eagle3Config())
    em.techniques["eagle3"].reset_parameters(seed=5, std=0.3)
    prompt = torch.tensor([3, 7, 1, 12, 5])
    return em, prompt, exact_joint(model, prompt)


@pytest.mark.parametrize("cfg", [
    eco.DecodeConfig(cycle_length=3, verifier="rejection"),
    eco.DecodeConfig(cycle_length=3),  # greedy verifier + sampler: sampled-match
    eco.DecodeConfig(cycle_length=3, draft_policy="dynamic_tree", draft_policy_options={"depth": 2, "topk": 3}),
])
def test_lossless_sampling(setup, cfg):
    em, prompt, exact = setup
    emp = empirical_joint(em, prompt, cfg)
    tv = 0.5 * (emp - exact).abs().sum().item()
    assert tv < 0.08, tv


def test_negative_control_detects_a_biased_sampler(setup):
    """The TV test has power: a sampler at another temperature is rejected."""
    em, prompt, exact = setup
    torch.manual_seed(1)
    out = em.decode_batch([prompt] * 3000, 2, decoding=eco.DecodeConfig(cycle_length=1),
                          selector=TopPSampler(temperature=0.5))
    counts = torch.zeros(V, V)
    for r in out:
        counts[int(r.tokens[0]), int(r.tokens[1])] += 1
    assert 0.5 * (counts / 3000 - exact).abs().sum().item() > 0.1


def test_rejection_rule_reference():
    g = torch.Generator().manual_seed(0)
    B, k = 64, 3
    p = torch.softmax(torch.randn(B, k + 1, V, generator=g), -1)
    q = torch.softmax(torch.randn(B, k, V, generator=g), -1)
    drafts = torch.multinomial(q.reshape(-1, V), 1, generator=g).reshape(B, k)
    u_acc, u_draw = torch.rand(B, k, generator=g), torch.rand(B, generator=g)
    n_acc, out = ops.rejection(p, q, drafts, u_acc, u_draw)
    for b in range(B):
        j = int(n_acc[b])
        assert torch.equal(out[b, :j], drafts[b, :j])
        if j < k:
            x = int(drafts[b, j])
            assert u_acc[b, j] * q[b, j, x] >= p[b, j, x]
        else:
            assert p[b, k, int(out[b, k])] > 0
