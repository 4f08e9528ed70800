"""Hydra, ReDrafter, PARD and cross-layer jump drafting: lossless under greedy verification (chains and dynamic
trees), and their objectives train."""

import pytest
import torch

import economize_b200 as eco
from economize_b200.techniques.dflash import DFlashConfig
from economize_b200.techniques.hydra import HydraConfig
from economize_b200.techniques.jump import JumpConfig
from economize_b200.techniques.pard import PardConfig
from economize_b200.techniques.redrafter import RedrafterConfig
from economize_b200.train.objective import OBJECTIVES

from .helpers import prompts, tiny_model

CAL = torch.randint(0, 1024, (2, 32), generator=torch.Generator().manual_seed(3))
TREE = eco.DecodeConfig(cycle_length=5, draft_policy="dynamic_tree",
                        draft_policy_options={"depth": 4, "topk": 4, "total_tokens": 16})


@pytest.fixture(scope="module")
def model():
    return tiny_model()


@pytest.fixture(scope="module")
def plain(model):
    return eco.apply(model).decode_batch(prompts(), 20, decoding=eco.DecodeConfig(cycle_length=1))


@pytest.mark.parametrize("make,decoding", [
    (lambda: HydraConfig(num_heads=4), None),
    (lambda: HydraConfig(num_heads=4), TREE),
    (lambda: HydraConfig(num_heads=4, prefix_layer=True), None),
    (lambda: HydraConfig(num_heads=4, prefix_layer=True, prefix_intermediate_size=128), TREE),
    (lambda: RedrafterConfig(beam_width=4, beam_length=4), None),
    (lambda: RedrafterConfig(beam_length=4), eco.DecodeConfig(cycle_length=4)),
    (lambda: PardConfig(model=tiny_model(num_layers=2, seed=1), max_drafts=4), None),
    (lambda: JumpConfig(target_layer=1, source_layer=2), None),
    (lambda: JumpConfig(target_layer=1, source_layers=(2, 3), mixer="concat"), None),
    (lambda: JumpConfig(target_layer=1, source_layers=(1, 4), mixer="attention"), TREE),
    (lambda: JumpConfig(target_layer=2, source_layers=(2, 3, 4), mixer="linear"), None),
    (lambda: JumpConfig(target_layer=1, source_layer=3, exit_layer=3), TREE),
    (lambda: DFlashConfig(block_size=5), None),
    (lambda: DFlashConfig(block_size=5), TREE),
])
def test_lossless(model, plain, make, decoding):
    em = eco.apply(model, make())
    out = em.decode_batch(prompts(), 20, decoding=decoding)
    for a, b in zip(plain, out):
        assert torch.equal(a.tokens, b.tokens)


def test_pard_self_draft_accepts(model, plain):
    # the target itself as the PARD model: the first draft of every cycle is the target's own next token
    em = eco.apply(model, PardConfig(model=model, max_drafts=3))
    out = em.decode_batch(prompts(), 20)
    assert sum(r.accepted for r in out) > 0


@pytest.mark.parametrize("cfg,name", [(HydraConfig(num_heads=3), "step_distill"),
                                      (HydraConfig(num_heads=3, prefix_layer=True), "step_distill"),
                                      (RedrafterConfig(beam_length=3), "step_distill"),
                                      (JumpConfig(target_layer=1, source_layer=2), "jump_rollout"),
                                      (JumpConfig(target_layer=1, source_layers=(2, 3), mixer="attention"),
                                       "jump_rollout")])
def test_objectives_train(cfg, name):
    em = eco.apply(tiny_model(), cfg)
    obj = OBJECTIVES.get(name)(em)
    opt = torch.optim.Adam(obj.parameters(), lr=2e-3)
    losses = []
    for _ in range(8):
        loss, _ = obj.loss(CAL)
        opt.zero_grad()
        loss.backward()
        opt.step()
        losses.append(float(loss.detach()))
    assert min(losses[1:]) < losses[0], losses


@pytest.mark.gpu
@pytest.mark.parametrize("make,decoding", [
    (lambda m: HydraConfig(num_heads=3), None),
    (lambda m: HydraConfig(num_heads=3, prefix_layer=True), None),
    (lambda m: RedrafterConfig(beam_width=4, beam_length=3), None),
    (lambda m: JumpConfig(target_layer=1, source_layer=1), None),
    (lambda m: DFlashConfig(block_size=4), None),
    (lambda m: PardConfig(model=m, max_drafts=3), None),
])
def test_lossless_on_gpu_with_graphs(cuda, make, decoding):
    from .helpers import gpu_tiny_model

    model = gpu_tiny_model(cuda)
    ps = [p.to(cuda) for p in prompts((17, 33))]
    plain = eco.apply(model).decode_batch(ps, 16, decoding=eco.DecodeConfig(cycle_length=1))
    em = eco.apply(model, make(model))
    base = decoding or em.decoding
    import dataclasses

    out = em.decode_batch(ps, 16, decoding=dataclasses.replace(base, cuda_graphs=True))
    for a, b in zip(plain, out):
        assert torch.equal(a.tokens.cpu(), b.tokens.cpu())


def test_hydra_prefix_layer_starts_as_identity_and_trains(model):
    """A fresh prefix layer passes the target state through (its output projections are zero): the same heads draft
    the same tokens with and without it. After training, its parameters have moved and decoding stays lossless."""
    plain_heads = eco.apply(model, HydraConfig(num_heads=3))
    with_prefix = eco.apply(model, HydraConfig(num_heads=3, prefix_layer=True))
    with torch.no_grad():
        for a, b in zip(plain_heads.techniques["hydra"].heads.parameters(),
                        with_prefix.techniques["hydra"].heads.parameters()):
            a.normal_(0, 0.02)
            b.copy_(a)
    dc = eco.DecodeConfig(cycle_length=4)
    for x, y in zip(plain_heads.decode_batch(prompts(), 16, decoding=dc),
                    with_prefix.decode_batch(prompts(), 16, decoding=dc)):
        assert torch.equal(x.tokens, y.tokens) and x.accepted == y.accepted
    obj = OBJECTIVES.get("step_distill")(with_prefix)
    opt = torch.optim.Adam(obj.parameters(), lr=2e-3)
    for _ in range(3):
        loss, _ = obj.loss(CAL)
        opt.zero_grad()
        loss.backward()
        opt.step()
    assert with_prefix.techniques["hydra"].prefix.wo.abs().sum() > 0
    ref = eco.apply(model).decode_batch(prompts(), 16, decoding=eco.DecodeConfig(cycle_length=1))
    for a, b in zip(ref, with_prefix.decode_batch(prompts(), 16, decoding=dc)):
        assert torch.equal(a.tokens, b.tokens)


def test_dflash_block_objective_trains():
    em = eco.apply(tiny_model(), DFlashConfig(block_size=4))
    obj = OBJECTIVES.get("dflash_block")(em, anchors=8)
    opt = torch.optim.Adam(obj.parameters(), lr=3e-3)
    data = torch.randint(0, 1024, (2, 24), generator=torch.Generator().manual_seed(5))
    losses = []
    for _ in range(8):
        loss, metrics = obj.loss(data)
        opt.zero_grad()
        loss.backward()
        opt.step()
        losses.append(float(loss.detach()))
    assert {"root_kl", "block_kl", "block_acc"} <= set(metrics)
    assert min(losses[1:]) < losses[0], losses
    ref = eco.apply(tiny_model()).decode_batch(prompts(), 12, decoding=eco.DecodeConfig(cycle_length=1))
    for a, b in zip(ref, em.decode_batch(prompts(), 12)):
        assert torch.equal(a.tokens, b.tokens)


def test_dflash_block_objective_matches_the_drafter():
    """The objective's root and block logits for an anchor equal what the drafter computes at inference after a
    prefill of the same context (same layer, same masks)."""
    from economize_b200.runtime.cache import StepBatch
    from economize_b200.techniques.dflash.objective import block_logits

    em = eco.apply(tiny_model(), DFlashConfig(block_size=4))
    tech = em.techniques["dflash"]
    tech.reset_parameters(seed=7)
    model = em.model
    prompt = prompts((17,))[0]
    tokens = torch.cat([prompt, torch.tensor([123])])  # the context and the anchor (the root token)
    n = tokens.numel()
    with torch.no_grad():
        _, aux = model.forward_step(tokens[None], StepBatch.prefill(torch.tensor([n], dtype=torch.int32), n),
                                    model.new_cache(1, 128), tech.aux_layers)
        d = tech.drafter()
        d.begin(1, 128)
        fused = d.fuse(aux)[:, :-1]  # the features of the context tokens (the anchor's own are not used)
        sources = torch.cat([torch.zeros_like(fused[:, :1]), fused], 1)
        root_logits, _ = d.observe(tokens[None], sources, torch.zeros(1, dtype=torch.int32),
                                   torch.tensor([n], dtype=torch.int32), torch.tensor([n - 1]))
        root, block = block_logits(tech, aux, tokens[None], torch.tensor([n - 1]), d.mask_id)
    torch.testing.assert_close(root[0, 0], root_logits[0], atol=2e-4, rtol=2e-4)
    torch.testing.assert_close(block[0, 0], d.stash[0], atol=2e-4, rtol=2e-4)


def test_jump_mixers_start_on_the_last_source():
    from economize_b200.techniques.jump import JumpConfig as JC

    model = tiny_model()
    one = eco.apply(model, JC(target_layer=1, source_layer=3))
    for mixer in ("concat", "linear"):
        many = eco.apply(tiny_model(), JC(target_layer=1, source_layers=(2, 3), mixer=mixer))
        many.techniques["jump"].predictor.load_state_dict(one.techniques["jump"].predictor.state_dict())
        dc = eco.DecodeConfig(cycle_length=4)
        for a, b in zip(one.decode_batch(prompts(), 12, decoding=dc), many.decode_batch(prompts(), 12, decoding=dc)):
            assert torch.equal(a.tokens, b.tokens) and a.accepted == b.accepted
    with pytest.raises(eco.ConfigError, match="source_layers"):
        eco.apply(tiny_model(), JC(target_layer=2, source_layers=(1, 3)))


@pytest.mark.parametrize("cfg", [JumpConfig(target_layer=1, source_layer=2, exit_layer=4),
                                 JumpConfig(target_layer=1, source_layers=(1, 3), mixer="concat", exit_layer=3),
                                 JumpConfig(target_layer=2, source_layers=(2, 4), mixer="attention")])
def test_jump_rollout_matches_the_drafter(cfg):
    """Every step of the training rollout reproduces what the drafter computes at decode time from the same start:
    the same predicted states, the same partial passes against the exact and its own keys, the same logits."""
    from economize_b200.runtime.cache import StepBatch
    from economize_b200.ops import reference
    from economize_b200.techniques.jump.rollout import rollout_steps

    em = eco.apply(tiny_model(), cfg)
    tech = em.techniques["jump"]
    g = torch.Generator().manual_seed(7)
    with torch.no_grad():  # a predictor away from its identity start, so the rollout's own states matter
        for p in tech.predictor.parameters():
            p.add_(torch.randn(p.shape, generator=g) * 0.05)
        for p in tech.mixer.parameters():
            p.add_(torch.randn(p.shape, generator=g) * 0.05)
    model = em.model
    tokens = torch.randint(0, 1024, (1, 24), generator=g)
    m, _, r = tech.layers
    capture = tuple(sorted({*range(m, r + 1), *tech.sources}))
    with torch.no_grad():
        cache = model.new_cache(1, 128)
        _, aux = model.forward_step(tokens, StepBatch.prefill(torch.tensor([24], dtype=torch.int32), 24), cache,
                                    capture=capture)
        starts, steps = rollout_steps(tech, tokens, aux, 3)
    assert starts.tolist() == list(range(21))
    drafter = tech.drafter()
    for start in (0, 9, 20):
        with torch.no_grad():
            exact = model.new_cache(1, 128)
            _, ex = model.forward_step(tokens[:, :start + 1], StepBatch.prefill(
                torch.tensor([start + 1], dtype=torch.int32), start + 1), exact, capture=tech.sources)
            drafter.bind_target_cache(exact)
            source = tech.mix(ex)[:, start:start + 1].to(model.dtype)
            for j in range(1, 4):
                slot = torch.tensor([start + j], dtype=torch.int32)
                logits, source = drafter._run(tokens[:, start + j:start + j + 1], source,
                                              StepBatch(slot, torch.ones(1, dtype=torch.int32), slot[:, None]))
                normed = reference.rmsnorm(steps[j - 1][1][:, start:start + 1], model.norm,
                                           model.config.rms_norm_eps)[0]
                want = model.logits(normed)
                torch.testing.assert_close(logits, want.float(), atol=2e-4, rtol=1e-4)


def test_jump_open_loop_objective_trains():
    em = eco.apply(tiny_model(), JumpConfig(target_layer=1, source_layer=2))
    obj = OBJECTIVES.get("jump_rollout")(em, horizon=3, ce_weight=0.5)
    opt = torch.optim.Adam(obj.parameters(), lr=2e-3)
    losses = []
    for _ in range(8):
        loss, stats = obj.loss(CAL)
        opt.zero_grad()
        loss.backward()
        opt.step()
        losses.append(float(loss))
    assert {"state_1", "state_3", "ce_1", "ce_3", "loss"} <= set(stats)
    assert losses[-1] < losses[0]
    with pytest.raises(eco.ConfigError):
        OBJECTIVES.get("jump_rollout")(em, horizon=0)


def test_jump_rl_pieces():
    """Acceptances lie in [0, 1] and equal sum min(p, q) of the rollout's distributions; hybrid log-probabilities
    take the target's distribution at cycle starts and the drafter's elsewhere, with gradients to the drafter."""
    from economize_b200.techniques.jump.rl import hybrid_log_probs, jump_acceptance

    em = eco.apply(tiny_model(), JumpConfig(target_layer=1, source_layer=2))
    tech = em.techniques["jump"]
    tokens = torch.randint(0, 1024, (2, 20), generator=torch.Generator().manual_seed(4))
    acc = jump_acceptance(tech, tokens, 3)
    assert acc.shape == (2, 17, 3) and bool(((acc >= 0) & (acc <= 1 + 1e-5)).all())
    lp = hybrid_log_probs(tech, tokens, first=8, cycle_length=4)
    assert lp.shape == (2, 12) and bool((lp <= 0).all())
    with torch.no_grad():
        exact = torch.log_softmax(em(tokens).float(), -1)
    for i in (0, 4, 8):  # cycle starts: the target's own log-probabilities
        t = 8 + i
        torch.testing.assert_close(lp[:, i], exact[:, t - 1].gather(-1, tokens[:, t:t + 1])[:, 0], atol=1e-4,
                                   rtol=1e-4)
    lp.sum().backward()
    assert tech.predictor.w2.weight.grad is not None and tech.predictor.w2.weight.grad.abs().sum() > 0
    with pytest.raises(eco.ConfigError):
        hybrid_log_probs(tech, tokens, first=8, cycle_length=1)
