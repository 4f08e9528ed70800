"""Tensor parallelism on 2 CPU ranks (Gloo): the sharded model decodes exactly like the unsharded one (plain
greedy, EAGLE-3 chains and trees) and the distributed argmax equals the single-device argmax."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.slow


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import torch.distributed as dist

    import economize_b200 as eco
    from economize_b200.distributed import init_distributed, tensor_parallel
    from economize_b200.techniques.eagle3 import Eagle3Config
    from tests.helpers import prompts, tiny_model

    torch.set_num_threads(2)
    init_distributed("gloo", timeout_s=60)
    try:
        ps = prompts()
        ref = eco.apply(tiny_model(), Eagle3Config())
        ref.techniques["eagle3"].reset_parameters(seed=2)
        want = {}
        cfgs = {"plain": eco.DecodeConfig(cycle_length=1), "chain": eco.DecodeConfig(cycle_length=4),
                "tree": eco.DecodeConfig(cycle_length=5, draft_policy="dynamic_tree",
                                         draft_policy_options={"depth": 4, "topk": 4, "total_tokens": 16})}
        for k, c in cfgs.items():
            want[k] = [r.tokens for r in ref.decode_batch(ps, 20, decoding=c)]
        em = eco.apply(tiny_model(), Eagle3Config())
        em.techniques["eagle3"].reset_parameters(seed=2)
        tensor_parallel(em)
        ok = {}
        for k, c in cfgs.items():
            got = [r.tokens for r in em.decode_batch(ps, 20, decoding=c)]
            ok[k] = all(torch.equal(a, b) for a, b in zip(got, want[k]))
        x = torch.randn(5, 1024, generator=torch.Generator().manual_seed(0))  # same on both ranks
        from economize_b200.parallel.tp import tp_argmax

        local = x[:, rank * 512:(rank + 1) * 512]  # every rank joins the collective
        ok["argmax"] = torch.equal(tp_argmax(local, em.model.tp, rank * 512), x.argmax(-1))
        queue.put((rank, ok))
    finally:
        dist.barrier()
        dist.destroy_process_group()


def test_tp2_gloo_matches_single_device():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(queue.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    for rank, ok in results.items():
        assert all(ok.values()), (rank, ok)
