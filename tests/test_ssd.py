"""Speculative speculative decoding over two ranks (Gloo on the CPU): the target's output equals its own greedy
decoding, and with a drafter identical to the target every round after the first is a speculation hit."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from economize_b200.parallel.ssd import SSDConfig


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, port, same, mode, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist

    from economize_b200.parallel.ssd import AsyncSpeculativeDecoder

    from .helpers import prompts, reference_greedy, tiny_model

    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=__import__("datetime").timedelta(seconds=60))
    try:
        model = tiny_model() if rank == 0 or same else tiny_model(num_layers=2, seed=1)
        prompt = prompts((19,))[0]
        res = AsyncSpeculativeDecoder(model, SSDConfig(draft_length=3, fanout=2, mode=mode)).generate(prompt, 14)
        if rank == 0:
            ref = reference_greedy(model, prompt, 14)
            queue.put(("ok", bool(torch.equal(res.tokens, ref)), res.hits, res.rounds, res.acceptance_length))
    except Exception as err:  # report instead of hanging the other rank
        queue.put(("error", f"{type(err).__name__}: {err}"))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("same,mode", [(False, "async"), (True, "async"), (False, "sync")])
def test_ssd_matches_greedy(same, mode):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, port, same, mode, queue)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = queue.get(timeout=180)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert res[0] == "ok", res
    assert res[1], res
    if same and mode == "async":
        assert res[2] == res[3] - 1 and res[4] == 4.0, res  # every round a hit, every draft accepted


def test_ssd_config_bounds():
    with pytest.raises(Exception):
        SSDConfig(draft_length=6, fanout=3)
    with pytest.raises(Exception):
        SSDConfig(temperature=-0.5)
    assert SSDConfig(temperature=0.7).sampling


def _sampling_worker(rank, port, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist

    from economize_b200.parallel.ssd import AsyncSpeculativeDecoder, _probs

    from .helpers import prompts, reference_greedy, tiny_model

    dist.init_process_group("gloo", rank=rank, world_size=2, timeout=__import__("datetime").timedelta(seconds=60))
    try:
        model = tiny_model() if rank == 0 else tiny_model(num_layers=2, seed=1)
        prompt = prompts((19,))[0]
        results = []
        for cfg in (SSDConfig(draft_length=3, fanout=2, temperature=0.8, top_p=1e-6, seed=1),  # nucleus of one token
                    SSDConfig(draft_length=3, fanout=2, temperature=1.0, top_p=0.9, seed=5),
                    SSDConfig(draft_length=3, fanout=2, temperature=1.0, top_p=0.9, seed=5)):
            results.append(AsyncSpeculativeDecoder(model, cfg).generate(prompt, 14))
        if rank == 0:
            greedy = torch.equal(results[0].tokens, reference_greedy(model, prompt, 14))
            same_seed = torch.equal(results[1].tokens, results[2].tokens)
            # every sampled token lies in the target's nucleus after its prefix
            seq = torch.cat([prompt, results[1].tokens])
            import economize_b200 as eco

            logits = eco.apply(model)(seq[None])[0]
            probs = _probs(logits, SSDConfig(temperature=1.0, top_p=0.9))
            n = prompt.numel()
            valid = all(float(probs[n - 1 + i, int(t)]) > 0 for i, t in enumerate(results[1].tokens))
            queue.put(("ok", greedy, same_seed, valid))
    except Exception as err:  # report instead of hanging the other rank
        queue.put(("error", f"{type(err).__name__}: {err}"))
    finally:
        dist.destroy_process_group()


def test_ssd_speculative_sampling():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_sampling_worker, args=(r, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = queue.get(timeout=240)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert res == ("ok", True, True, True), res
