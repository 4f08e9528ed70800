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


class GlooSequenceParallel:
    """The interface of :class:`economize_b200.parallel.sp.SequenceParallel` on Gloo collectives, so the host logic
    of a sequence-parallel pass (token shards, captures, the order of reduce-scatter and all-gather rounds) runs on
    CPU ranks."""

    def __init__(self, tp, hidden: int, max_rows: int = 4096, captures: int = 4) -> None:
        self.tp, self.hidden, self.max_rows, self.n_cap = tp, hidden, max_rows, captures
        self.pending = self.rows = None
        self.caps: dict[int, torch.Tensor] = {}
        self.passes = 0

    def fits(self, rows):
        return 1 <= rows <= self.max_rows

    def shard(self, rows):
        per = -(-rows // self.tp.size)
        lo = min(rows, self.tp.rank * per)
        return lo, min(rows, lo + per) - lo

    def _gather(self, part, rows):
        import torch.distributed as dist

        per = -(-rows // self.tp.size)
        padded = torch.zeros(per, self.hidden, dtype=part.dtype)
        padded[:part.shape[0]] = part
        every = [torch.empty_like(padded) for _ in range(self.tp.size)]
        dist.all_gather(every, padded)
        return torch.cat(every)[:rows]

    def rs_linear(self, x, w):
        from economize_b200 import ops

        self.pending = ops.linear(x.reshape(-1, x.shape[-1]), w)

    def reduce_norm(self, resid, weight, eps, rows, partials=True, capture=-1):
        import torch.distributed as dist

        from economize_b200 import ops

        lo, n = self.shard(rows)
        own = None
        if partials:
            full = self.pending.clone()
            dist.all_reduce(full)
            own = full[lo:lo + n]
        normed, new = ops.rmsnorm(own if own is not None else resid, weight, eps, resid if own is not None else None)
        self.rows = self._gather(normed, rows)
        if capture >= 0:
            self.caps[capture] = self._gather(new, rows)
        return new

    def ag_linear(self, w, rows):
        from economize_b200 import ops

        return ops.linear(self.rows[:rows], w)

    def ag_linear_parts(self, w, rows, lead):
        return self.ag_linear(w, rows).reshape(*lead, -1)

    def fetch(self, rows, like):
        self.passes += 1
        return self.rows[:rows].clone()

    def captured(self, slot, rows, like):
        return self.caps[slot][:rows].clone()

    def check(self):
        pass

    def close(self):
        pass


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
        # the sequence-parallel pass (token shards + reduce-scatter / all-gather rounds) on Gloo collectives
        em.model.tp.sp = GlooSequenceParallel(em.model.tp, em.model.config.hidden_size)
        em.refresh()
        for k, c in cfgs.items():
            got = [r.tokens for r in em.decode_batch(ps, 20, decoding=c)]
            ok[f"sp_{k}"] = all(torch.equal(a, b) for a, b in zip(got, want[k]))
        ok["sp_ran"] = em.model.tp.sp.passes > 0
        em.model.tp.sp = None
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
