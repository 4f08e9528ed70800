"""The engine on the CUDA path (bf16, sm_100a kernels).

Greedy speculative decoding (chains and trees) must reproduce plain greedy decoding through the same engine token
for token: the projections split K the same way for one row and for a verification pass, and attention takes the
last positions before every query in position order (the exact tail), so an accepted token's logits are the bits a
one-token pass computes. Plain decoding itself is checked against a full causal recompute up to a rounding-sized
logit gap (a prompt-length pass reduces keys differently from a one-token pass)."""

import pytest
import torch

import economize_b200 as eco
from economize_b200.models.config import tiny_llama
from economize_b200.models.llama import CausalLM, init_weights
from economize_b200.techniques.eagle3 import Eagle3Config

pytestmark = pytest.mark.gpu

TREE = {"depth": 6, "topk": 10, "total_tokens": 60}


@pytest.fixture(scope="module")
def em(cuda):
    cfg = tiny_llama(hidden_size=512, num_heads=4, num_kv_heads=2, head_dim=128, num_layers=4)
    model = init_weights(CausalLM(cfg, torch.bfloat16, cuda), seed=0)
    return eco.apply(model, Eagle3Config())


def _prompts(cuda, lengths=(17, 40, 129)):
    g = torch.Generator().manual_seed(0)
    return [torch.randint(0, 1024, (n,), generator=g).to(cuda) for n in lengths]


def _assert_greedy(em, prompt, tokens, tol=0.08):
    seq = torch.cat([prompt, tokens.to(prompt.device)])
    logits = em(seq[None])[0].float()
    n = prompt.numel()
    for i, tok in enumerate(tokens.tolist()):
        row = logits[n - 1 + i]
        gap = (row.max() - row[tok]).item()
        assert gap <= tol * max(1.0, row.abs().max().item()), (i, tok, int(row.argmax()), gap)


def test_plain_decoding_is_greedy(em, cuda):
    prompts = _prompts(cuda)
    for p, r in zip(prompts, em.decode_batch(prompts, 24, decoding=eco.DecodeConfig(cycle_length=1))):
        assert r.tokens.numel() == 24
        _assert_greedy(em, p, r.tokens)


@pytest.mark.parametrize("graphs", [False, True])
@pytest.mark.parametrize("tree", [False, True])
def test_spec_decoding_is_greedy(em, cuda, graphs, tree):
    prompts = _prompts(cuda)
    cfg = (eco.DecodeConfig(cycle_length=7, draft_policy="dynamic_tree", draft_policy_options=TREE,
                            cuda_graphs=graphs) if tree else eco.DecodeConfig(cycle_length=5, cuda_graphs=graphs))
    spec = em.decode_batch(prompts, 40, decoding=cfg)
    plain = em.decode_batch(prompts, 40, decoding=eco.DecodeConfig(cycle_length=1))
    for p, s, q in zip(prompts, spec, plain):
        assert s.tokens.numel() == 40
        assert torch.equal(s.tokens, q.tokens)
        _assert_greedy(em, p, s.tokens)
    assert eco.ops.require().status(0) == 0


def test_graph_replay_matches_eager(em, cuda):
    """The captured cycle computes what the eager cycle computes (same kernels, same order)."""
    prompts = _prompts(cuda)
    base = dict(cycle_length=7, draft_policy="dynamic_tree", draft_policy_options=TREE)
    eager = em.decode_batch(prompts, 32, decoding=eco.DecodeConfig(**base))
    graphed = em.decode_batch(prompts, 32, decoding=eco.DecodeConfig(**base, cuda_graphs=True))
    for a, b in zip(eager, graphed):
        assert torch.equal(a.tokens, b.tokens)
        assert a.accepted == b.accepted


def test_chain_is_bit_identical_to_plain(em, cuda):
    """A verified chain occupies the same cache slots as plain decoding and every kernel reduces a row the same
    way whatever the number of rows in the pass, so greedy chain speculation reproduces plain decoding exactly."""
    prompts = _prompts(cuda)
    plain = em.decode_batch(prompts, 48, decoding=eco.DecodeConfig(cycle_length=1))
    for graphs in (False, True):
        chain = em.decode_batch(prompts, 48, decoding=eco.DecodeConfig(cycle_length=5, cuda_graphs=graphs))
        for p, c in zip(plain, chain):
            assert torch.equal(p.tokens, c.tokens)


@pytest.mark.parametrize("kind", ["lookup", "medusa", "draft_model"])
def test_other_drafters_on_gpu(em, cuda, kind):
    from economize_b200.techniques.draft_model import DraftModelConfig
    from economize_b200.techniques.lookup import LookupConfig
    from economize_b200.techniques.medusa import MedusaConfig

    model = em.model
    cfg = {"lookup": LookupConfig(), "medusa": MedusaConfig(num_heads=4, tree="mc_sim_7b_63"),
           "draft_model": DraftModelConfig(model=model)}[kind]
    e2 = eco.apply(model, cfg)
    prompts = _prompts(cuda)
    for graphs in (False, True):
        dc = eco.DecodeConfig(cycle_length=5, cuda_graphs=graphs)
        out = e2.decode_batch(prompts, 32, decoding=dc)
        for p, r in zip(prompts, out):
            assert r.tokens.numel() == 32
            _assert_greedy(e2, p, r.tokens)
    assert eco.ops.require().status(0) == 0


def test_ngram_kernel(cuda):
    from economize_b200.ops import reference

    g = torch.Generator().manual_seed(3)
    hist = torch.randint(0, 6, (8, 300), generator=g)
    length = torch.randint(5, 300, (8,), generator=g).to(torch.int32)
    for earliest in (True, False):
        want = reference.ngram(hist, length, 5, 1, 3, earliest)
        got = eco.ops.ngram(hist.to(cuda), length.to(cuda), 5, 1, 3, earliest)
        assert torch.equal(got.cpu(), want)


@pytest.mark.parametrize("policy,options", [
    ("sequoia", {"acceptance": (0.6, 0.15, 0.06, 0.03), "total_tokens": 32, "depth": 6}),
    ("specexec", {"depth": 6, "width": 8, "topk": 8, "total_tokens": 48}),
])
def test_tree_policies_are_greedy_and_graph_stable(em, cuda, policy, options):
    """Sequoia static trees and SpecExec search on the CUDA path: greedy up to rounding, and the captured cycle
    reproduces the eager one."""
    prompts = _prompts(cuda)
    base = dict(cycle_length=7, draft_policy=policy, draft_policy_options=options)
    eager = em.decode_batch(prompts, 40, decoding=eco.DecodeConfig(**base))
    graphed = em.decode_batch(prompts, 40, decoding=eco.DecodeConfig(**base, cuda_graphs=True))
    for p, a, b in zip(prompts, eager, graphed):
        assert a.tokens.numel() == 40
        _assert_greedy(em, p, a.tokens)
        assert torch.equal(a.tokens, b.tokens)
    assert eco.ops.require().status(0) == 0
