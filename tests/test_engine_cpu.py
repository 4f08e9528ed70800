"""Lossless decoding on the CPU fp32 oracle path: speculative chains and dynamic trees equal
plain greedy decoding, which equals full recompute and Hugging Face's greedy generate."""

import pytest
import torch

import economize_b200 as eco
from economize_b200.techniques.eagle3 import Eagle3Config

from .helpers import prompts, reference_greedy, tiny_model

TREE = {"depth": 6, "topk": 10, "total_tokens": 60}


@pytest.fixture(scope="module")
def em():
    return eco.apply(tiny_model(), Eagle3Config())


@pytest.fixture(scope="module")
def plain(em):
    return em.decode_batch(prompts(), 32, decoding=eco.DecodeConfig(cycle_length=1))


def test_plain_equals_recompute(em, plain):
    for p, r in zip(prompts(), plain):
        assert torch.equal(r.tokens, reference_greedy(em.model, p, 32))


def test_plain_equals_hf_generate(em, plain):
    transformers = pytest.importorskip("transformers")
    hf = transformers.LlamaForCausalLM(em.model.config.to_hf()).eval()
    hf.load_state_dict(em.model.hf_state_dict())
    for p, r in zip(prompts(), plain):
        out = hf.generate(p[None], max_new_tokens=32, do_sample=False, pad_token_id=0)
        assert torch.equal(out[0, p.numel():], r.tokens)


def test_config1_chain_of_4(em, plain):
    chain = em.decode_batch(prompts(), 32, decoding=eco.DecodeConfig(cycle_length=5))
    for a, b in zip(plain, chain):
        assert torch.equal(a.tokens, b.tokens)


@pytest.mark.parametrize("opts", [TREE, {"depth": 3, "topk": 4, "total_tokens": 10}, {"depth": 1, "topk": 3}])
def test_dynamic_tree(em, plain, opts):
    cfg = eco.DecodeConfig(cycle_length=opts["depth"] + 1, draft_policy="dynamic_tree", draft_policy_options=opts)
    tree = em.decode_batch(prompts(), 32, decoding=cfg)
    for a, b in zip(plain, tree):
        assert torch.equal(a.tokens, b.tokens)


def test_oracle_drafter_accepts_everything():
    """A target that repeats its input token with certainty (residual outputs zero, head = 30 x the embedding) and
    an identity-initialised EAGLE-3 head (which drafts the token whose features it reads) agree on every draft:
    each cycle must accept all of them, in chains and in dynamic trees (whose best path is then the deepest)."""
    model = tiny_model()
    with torch.no_grad():
        for layer in model.layers:
            layer.wo.zero_()
            layer.w_down.zero_()
        model.lm_head.copy_(model.embed * 30)
    em = eco.apply(model, Eagle3Config())
    em.techniques["eagle3"].reset_parameters(seed=1, identity=True)
    ps = prompts()
    base = em.decode_batch(ps, 30, decoding=eco.DecodeConfig(cycle_length=1))
    assert all(torch.equal(r.tokens, p[-1].repeat(30)) for p, r in zip(ps, base))
    for cfg, tau in ((eco.DecodeConfig(cycle_length=7, draft_policy="dynamic_tree", draft_policy_options=TREE), 7),
                     (eco.DecodeConfig(cycle_length=4), 4)):
        out = em.decode_batch(ps, 30, decoding=cfg)
        for a, b in zip(base, out):
            assert torch.equal(a.tokens, b.tokens)
            assert b.mean_accepted_length == pytest.approx(tau, abs=0.01)


def test_accept_all_is_lossy_but_runs(em):
    out = em.decode_batch(prompts(), 12, decoding=eco.DecodeConfig(cycle_length=4, lossless=False))
    assert all(r.tokens.numel() == 12 for r in out)
    assert all(r.mean_accepted_length == 4.0 for r in out)


def test_confidence_policy_is_lossless(em, plain):
    out = em.decode_batch(prompts(), 32, decoding=eco.DecodeConfig(cycle_length=5, min_confidence=0.5))
    for a, b in zip(plain, out):
        assert torch.equal(a.tokens, b.tokens)


def test_typical_verifier_runs(em):
    cfg = eco.DecodeConfig(cycle_length=4, verifier="typical", verifier_options={"threshold": 0.09, "alpha": 0.3})
    out = em.decode_batch(prompts(), 10, decoding=cfg)
    assert all(r.tokens.numel() == 10 for r in out)


def test_stop_token(em, plain):
    stop = int(plain[0].tokens[5])
    out = em.decode_batch(prompts()[:1], 32, decoding=eco.DecodeConfig(cycle_length=5), stop=stop)[0]
    assert out.tokens[-1].item() == stop and out.tokens.numel() <= 6


def test_generate_hf_style(em):
    ids = torch.stack([prompts((12,))[0]])
    out = em.generate(ids, max_new_tokens=8, decoding=eco.DecodeConfig(cycle_length=3))
    assert out.shape == (1, 20) and torch.equal(out[0, :12], ids[0])


def test_finished_rows_stop_advancing(em):
    """A row that reached its token budget keeps its KV position while the other rows decode on (its cache never
    runs past the capacity reserved for it)."""
    cfg = eco.DecodeConfig(cycle_length=7, draft_policy="dynamic_tree", draft_policy_options=TREE)
    ps = prompts()
    out = em.decode_batch(ps, [2, 30], decoding=cfg)
    assert [r.tokens.numel() for r in out] == [2, 30]
    engine = em.decoder(cfg)
    state = next(s for (b, _, out_cap), s in engine._states.items() if b == 2 and out_cap == 30 + engine.depth + 2)
    assert int(state.kv_len[0]) <= ps[0].numel() + 1 + 7  # prefill token + at most one cycle's commit
