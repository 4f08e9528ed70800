"""Training extras: data sources (token files, sharding, passkey), data-parallel fit over two Gloo ranks (each rank
draws its own batches, parameters stay identical), and the Trainer integration's module and collator."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import economize_b200 as eco
from economize_b200.techniques.medusa import MedusaConfig
from economize_b200.train.data import ShardedSource, TensorSource, TokenFileSource, passkey_prompts
from economize_b200.train.trainer import EffCollator, ObjectiveModule

from .helpers import tiny_model


def test_token_file_source(tmp_path):
    path = tmp_path / "tokens.bin"
    np.arange(5000, dtype=np.uint16).tofile(path)
    src = TokenFileSource(path, batch_size=3, seq_len=16, seed=1)
    b = src.next()
    assert b.shape == (3, 17) and bool(((b[:, 1:] - b[:, :-1]) == 1).all())
    state = src.state()
    nxt = src.next()
    src.restore(state)
    assert torch.equal(src.next(), nxt)


def test_sharded_source_partitions_a_stream():
    data = torch.arange(40).reshape(40, 1)
    a = ShardedSource(TensorSource(data, 1, seed=0), 0, 2)
    b = ShardedSource(TensorSource(data, 1, seed=0), 1, 2)
    ref = TensorSource(data, 1, seed=0)
    stream = [int(ref.next()) for _ in range(6)]
    assert [int(a.next()) for _ in range(3)] == stream[0::2]
    assert [int(b.next()) for _ in range(3)] == stream[1::2]


def test_passkey_prompts():
    p, k = passkey_prompts(3, 64, 1024, key_len=4, seed=0)
    assert p.shape == (3, 64) and k.shape == (3, 4)
    for i in range(3):
        row = p[i].tolist()
        assert any(row[j:j + 4] == k[i].tolist() for j in range(60)) and row[-1] == int(k[i, 0])


def test_objective_module_and_collator():
    em = eco.apply(tiny_model(), MedusaConfig(num_heads=2))
    from economize_b200.train.objective import OBJECTIVES

    mod = ObjectiveModule(OBJECTIVES.get("medusa_ce")(em))
    batch = EffCollator()([{"input_ids": list(range(16))}, {"input_ids": list(range(16, 32))}])
    out = mod(**batch)
    out["loss"].backward()
    assert batch["input_ids"].shape == (2, 16)
    assert any(p.grad is not None for p in mod.parameters())
    assert {id(p) for p in mod.parameters()} <= {id(p) for p in em.techniques["medusa"].parameters()}


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _dp_worker(rank, port, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    import torch.distributed as dist

    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=datetime.timedelta(seconds=60))
    try:
        em = eco.apply(tiny_model(), MedusaConfig(num_heads=2))
        data = torch.randint(0, 1024, (64, 24), generator=torch.Generator().manual_seed(0))
        seen = []
        src = TensorSource(data, 4, seed=1000003 * rank)
        orig = src.next

        def record():
            b = orig()
            seen.append(b.clone())
            return b

        src.next = record
        eco.train.fit(em, src, steps=3, batch_size=4, log_every=100)
        flat = torch.cat([p.detach().flatten().float() for p in em.techniques["medusa"].parameters()])
        other = flat.clone()
        dist.broadcast(other, src=0)
        queue.put((rank, bool(torch.equal(flat, other)), seen[0].sum().item()))
    except Exception as err:
        queue.put((rank, f"{type(err).__name__}: {err}", None))
    finally:
        dist.destroy_process_group()


def test_data_parallel_fit_keeps_ranks_in_sync():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_dp_worker, args=(r, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = dict((r, (same, s)) for r, same, s in (queue.get(timeout=180) for _ in procs))
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert res[0][0] is True and res[1][0] is True, res
    assert res[0][1] != res[1][1]  # the ranks drew different batches


def test_offloaded_adamw_matches_adamw():
    import torch

    from economize_b200.train.offload import OffloadedAdamW

    g = torch.Generator().manual_seed(0)
    w0 = torch.randn(8, 5, generator=g)
    a, b = torch.nn.Parameter(w0.clone()), torch.nn.Parameter(w0.clone())
    ref = torch.optim.AdamW([a], lr=1e-2, weight_decay=0.1)
    off = OffloadedAdamW([b], lr=1e-2, weight_decay=0.1)
    for step in range(5):
        x = torch.randn(3, 8, generator=g)
        for p, opt in ((a, ref), (b, off)):
            opt.zero_grad()
            (x @ p).pow(2).sum().backward()
            opt.step()
    assert torch.allclose(a, b, atol=1e-6)
    state = off.state_dict()
    again = OffloadedAdamW([torch.nn.Parameter(b.detach().clone())], lr=1e-2, weight_decay=0.1)
    again.load_state_dict(state)
    assert torch.equal(again._host[0], off._host[0])


def test_fit_with_offloaded_optimizer_trains():
    import torch

    import economize_b200 as eco
    from economize_b200.techniques.eagle3 import Eagle3Config
    from economize_b200.train import fit

    from .helpers import tiny_model

    em = eco.apply(tiny_model(), Eagle3Config())
    data = torch.randint(0, 1024, (4, 32), generator=torch.Generator().manual_seed(1))
    res = fit(em, data, steps=4, batch_size=2, offload_optimizer=True, autocast=None, log_every=1)
    assert res.steps == 4


def test_rl_building_blocks():
    import torch

    from economize_b200.train.rl import acceptance, expected_tokens, token_log_probs

    g = torch.Generator().manual_seed(0)
    head = torch.randn(7, 5, generator=g, requires_grad=True)
    h = torch.randn(2, 9, 5, generator=g)
    tok = torch.randint(0, 7, (2, 9), generator=g)
    lp, ent = token_log_probs(h, tok, lambda x: x @ head.t(), chunk=4)
    full = torch.log_softmax(h @ head.t(), -1)
    assert torch.allclose(lp, full.gather(-1, tok[..., None])[..., 0], atol=1e-6)
    assert torch.allclose(ent, -(full.exp() * full).sum(-1), atol=1e-6)
    lp.sum().backward()
    assert head.grad is not None and head.grad.abs().sum() > 0
    p = torch.tensor([0.5, 0.3, 0.2])
    assert float(acceptance(p, p)) == 1.0
    assert abs(float(acceptance(p, torch.tensor([0.0, 0.0, 1.0]))) - 0.2) < 1e-7
    a = torch.full((4,), 0.6)
    assert abs(float(expected_tokens(a)) - (1 - 0.6 ** 5) / (1 - 0.6)) < 1e-5


def test_distill_from_a_larger_teacher():
    """distill_kl with a larger teacher: the distributions are the teacher's (same tokenizer), the drafter's inputs
    the target's, and the loss goes down."""
    from economize_b200.models.config import tiny_llama
    from economize_b200.models.llama import CausalLM, init_weights
    from economize_b200.techniques.eagle3 import Eagle3Config
    from economize_b200.train import larger_teacher
    from economize_b200.train.objective import OBJECTIVES, _teacher_draft_probs

    from .helpers import tiny_model

    big = init_weights(CausalLM(tiny_llama(num_layers=6, hidden_size=384, num_heads=6, num_kv_heads=2,
                                           intermediate_size=1024), torch.float32, "cpu"), seed=5)
    em = eco.apply(tiny_model(), Eagle3Config(draft_vocab=512))
    tokens = torch.randint(0, 1024, (2, 24), generator=torch.Generator().manual_seed(2))
    obj = OBJECTIVES.get("distill_kl")(em, teacher=big)
    _, probs = _teacher_draft_probs(em, obj.tech, tokens, None, obj.teacher)
    ids = torch.arange(obj.tech.d2t.numel()) + obj.tech.d2t
    want = torch.softmax(larger_teacher(big)(tokens)[..., ids], -1)
    torch.testing.assert_close(probs, want)
    _, own = _teacher_draft_probs(em, obj.tech, tokens, None)
    assert (own - probs).abs().max() > 1e-3  # not the target's distributions
    opt = torch.optim.Adam(obj.parameters(), lr=2e-3)
    losses = []
    for _ in range(6):
        loss, _ = obj.loss(tokens)
        opt.zero_grad()
        loss.backward()
        opt.step()
        losses.append(float(loss))
    assert losses[-1] < losses[0]
    with pytest.raises(eco.ConfigError, match="smaller"):
        larger_teacher(big, vocab_size=4096)(tokens)
