"""Decode-cycle benchmark: ``python -m economize_b200.bench.cycle [--tree/--chain/--plain] [--batch B]``.

Builds the random-init Llama-3.1-8B architecture and an (untrained, early-exit-initialised) EAGLE-3 head, then
times whole ``generate`` calls (CUDA events) for the chosen drafting mode and reports milliseconds per cycle and
per generated token. The drafter is untrained, so the accepted length is close to one token per cycle; the number
to read is the cycle time, which bounds tokens per second for any acceptance rate. ``--cycles-only`` stops after
the warm-up generation (the case a launch-list capture profiles). ``--breakdown`` records one more generation with
the PyTorch profiler (CUPTI kernel records, graph replays included) and prints device microseconds and launches per
cycle for every kernel name; run it with ``ECZ_PDL=0`` so that no kernel's record includes the time it waits for its
predecessor (with programmatic dependent launch a kernel starts before the previous one ends).

Under ``torchrun --nproc-per-node N`` (``WORLD_SIZE`` > 1) the target is sharded over the N ranks with tensor
parallelism (the fused NVLink collectives; ``--nccl-tp`` for NCCL), every rank decodes the same prompts, the times
are the maximum over the ranks and rank 0 prints (the breakdown is rank 0's kernels).
"""

from __future__ import annotations

import argparse
import datetime
import json
import os

import torch

__all__ = ["main"]


def main(argv: list[str] | None = None) -> None:
    import economize_b200 as eco
    from economize_b200.models.config import llama31_8b
    from economize_b200.models.llama import CausalLM, init_weights
    from economize_b200.techniques.eagle3 import Eagle3Config

    p = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    p.add_argument("--mode", choices=["tree", "chain", "plain", "sequoia", "specexec"], default="tree")
    p.add_argument("--batch", type=int, default=1)
    p.add_argument("--prompt-len", type=int, default=512)
    p.add_argument("--new-tokens", type=int, default=64)
    p.add_argument("--iters", type=int, default=3)
    p.add_argument("--layers", type=int, default=32)
    p.add_argument("--cycles-only", action="store_true")
    p.add_argument("--breakdown", type=int, default=0, metavar="N",
                   help="print the N kernels with the most device time per cycle (PyTorch profiler)")
    p.add_argument("--nccl-tp", action="store_true", help="tensor parallelism over NCCL instead of the fused kernels")
    a = p.parse_args(argv)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if world > 1:
        import torch.distributed as dist

        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", torch.cuda.current_device()))
    cfg = llama31_8b()
    cfg.num_layers = a.layers
    target = init_weights(CausalLM(cfg, torch.bfloat16, "cuda"), seed=0)
    eff = eco.apply(target, Eagle3Config(draft_vocab=32000))
    eff.techniques["eagle3"].reset_parameters(seed=0, identity=True)
    if world > 1:
        from economize_b200.distributed import TPGroup, tensor_parallel

        tensor_parallel(eff.model, TPGroup(rank, world), fused=not a.nccl_tp)
    if a.mode == "tree":
        dc = eco.DecodeConfig(cycle_length=7, draft_policy="dynamic_tree", cuda_graphs=True,
                              draft_policy_options={"depth": 6, "topk": 10, "total_tokens": 60})
    elif a.mode == "sequoia":  # a static tree of 60 nodes shaped for typical EAGLE acceptance rates
        dc = eco.DecodeConfig(cycle_length=7, draft_policy="sequoia", cuda_graphs=True,
                              draft_policy_options={"acceptance": (0.6, 0.15, 0.06, 0.03), "total_tokens": 60,
                                                    "depth": 6})
    elif a.mode == "specexec":
        dc = eco.DecodeConfig(cycle_length=7, draft_policy="specexec", cuda_graphs=True,
                              draft_policy_options={"depth": 6, "width": 10, "topk": 10, "total_tokens": 60})
    elif a.mode == "chain":
        dc = eco.DecodeConfig(cycle_length=7, cuda_graphs=True)
    else:
        dc = eco.DecodeConfig(cycle_length=1, cuda_graphs=True)
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, cfg.vocab_size, (a.prompt_len,), generator=g).cuda() for _ in range(a.batch)]
    res = eff.decode_batch(prompts, a.new_tokens, decoding=dc)  # warm-up: graphs captured here
    torch.cuda.synchronize()
    if a.cycles_only:
        return
    times, cycles = [], 0
    for _ in range(a.iters):
        if world > 1:
            dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        res = eff.decode_batch(prompts, a.new_tokens, decoding=dc)
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    cycles = max(int(r.cycles) for r in res)
    # the prompt pass alone: a generate of one token is the prefill (its pass yields the first token), timed the
    # same way, so the per-cycle figure leaves the prefill out
    eff.decode_batch(prompts, 1, decoding=dc)
    torch.cuda.synchronize()
    pre = []
    for _ in range(a.iters):
        if world > 1:
            dist.barrier()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        eff.decode_batch(prompts, 1, decoding=dc)
        e.record()
        torch.cuda.synchronize()
        pre.append(s.elapsed_time(e))
    ms, ms_pre = min(times), min(pre)
    if world > 1:
        t = torch.tensor([ms, ms_pre], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, ms_pre = (float(v) for v in t.tolist())
    tokens = sum(int(r.tokens.numel()) for r in res)
    if a.breakdown:
        _breakdown(eff, prompts, a.new_tokens, dc, a.breakdown, verbose=rank == 0)
    if rank == 0:
        print(json.dumps({"mode": a.mode, "batch": a.batch, "prompt_len": a.prompt_len,
                          "new_tokens": a.new_tokens, "layers": a.layers, "tp": world,
                          "ms_per_generate": round(ms, 2), "cycles": cycles,
                          "ms_prefill": round(ms_pre, 2),
                          "ms_per_cycle_incl_prefill": round(ms / max(cycles, 1), 3),
                          "ms_per_cycle": round((ms - ms_pre) / max(cycles, 1), 3),
                          "tokens_per_s": round(tokens / ms * 1e3, 1),
                          "mean_accepted": round(sum(r.mean_accepted for r in res) / len(res), 3)}))
    if world > 1:  # release the captured graphs and the NVLink buffers before the group goes away
        eff.refresh()
        tpg = eff.model.tp
        for runtime in (getattr(tpg, "comm", None), getattr(tpg, "sp", None)):
            if runtime is not None:
                runtime.close()
        del eff, res
        import gc

        gc.collect()
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()


def _breakdown(eff, prompts, new_tokens: int, dc, top: int, verbose: bool = True) -> None:
    from torch.profiler import ProfilerActivity, profile

    engine = eff.decoder(dc)
    before = engine.stats.cycles
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        eff.decode_batch(prompts, new_tokens, decoding=dc)
        torch.cuda.synchronize()
    cycles = max(1, engine.stats.cycles - before)
    rows = []
    for e in prof.key_averages():
        t = getattr(e, "self_device_time_total", 0) or getattr(e, "self_cuda_time_total", 0)
        if t > 0:
            rows.append((t, e.count, e.key))
    rows.sort(reverse=True)
    total = sum(r[0] for r in rows)
    if not verbose:
        return
    print(json.dumps({"cycles": cycles, "kernel_us_per_cycle": round(total / cycles, 1),
                      "launches_per_cycle": round(sum(r[1] for r in rows) / cycles, 1)}))
    for t, n, name in rows[:top]:
        print(json.dumps({"kernel": name[:120], "us_per_cycle": round(t / cycles, 1),
                          "launches_per_cycle": round(n / cycles, 2), "share": round(t / total, 4)}))


if __name__ == "__main__":
    main()
