"""Headline benchmark: decode tokens/s + mean accepted length, Llama-3.1-8B + EAGLE-3 dynamic tree on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl ours|reference]

One *step* generates ``--new-tokens`` (256) tokens after uniform-random prompts of ``--prompt-len`` (512) tokens for
``--batch`` rows per GPU through the public API (``EfficientModel.decode_batch``), prefill included. The target is a
random-init Llama-3.1-8B architecture (bf16, seed 0) and the drafter an EAGLE-3 head (draft vocabulary 32000)
trained briefly on the target's own greedy continuations of synthetic prompts (``--train-steps``; 0 keeps the
random head). Decoding: dynamic tree, depth 6, top-k 10, 60 nodes, CUDA graphs.

With N > 1 GPUs (launched by torchrun) every rank serves its own batch (data-parallel replicas; ``scaling``
"weak"); the step time is the max over ranks of the CUDA-event time. ``value`` is the whole job's generated tokens
per second. The model weights (16 GB) exceed L2, so every step streams them from HBM (no flush needed).

``--impl reference`` runs the same metric through the unmodified reference (``baseline/_ref``: economize on
Hugging Face transformers) with the same target and drafter weights.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

HERE = os.path.dirname(os.path.abspath(__file__))
METRIC = "decode tok/s + mean accepted len, Llama-3.1-8B EAGLE-3 tree, 1/2/4/8 B200"
BASELINE_TOKS = None  # BASELINE.md publishes no B200 number for this config
TREE = {"depth": 6, "topk": 10, "total_tokens": 60}


def parse() -> argparse.Namespace:
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--batch", type=int, default=1)
    p.add_argument("--prompt-len", type=int, default=512)
    p.add_argument("--new-tokens", type=int, default=256)
    p.add_argument("--train-steps", type=int, default=150)
    p.add_argument("--train-rounds", type=int, default=3)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--model", choices=("llama31_8b", "tiny"), default="llama31_8b")
    p.add_argument("--no-graphs", action="store_true")
    p.add_argument("--parallel", choices=("dp", "tp"), default="dp",
                   help="dp: one replica per GPU; tp: one model sharded over all GPUs (fused NVLink collectives)")
    p.add_argument("--nccl-tp", action="store_true", help="with --parallel tp: NCCL all-reduces instead of the fused "
                   "GEMM->push / reduce+RMSNorm kernels")
    return p.parse_args()


class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int) -> None:
        self.index = device_index
        self.samples: list[list[str]] = []
        self._stop = threading.Event()
        self._thread: threading.Thread | None = None

    def _run(self) -> None:
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=5)
                for line in out.stdout.strip().splitlines():
                    self.samples.append([x.strip() for x in line.split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self) -> ClockSampler:
        self._thread = threading.Thread(target=self._run, daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=10)

    def summary(self) -> dict:
        sm = [float(s[1]) for s in self.samples if len(s) > 8 and s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if len(s) > 8 and s[2].replace(".", "").isdigit()]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({n for s in self.samples if len(s) > 8 for n, v in zip(names, s[5:9]) if v == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(sm)}


def setup_dist(args: argparse.Namespace):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=1800),
                                device_id=torch.device("cuda", local))
    return world, rank, local


def reduce_max(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def reduce_sum(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist

    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t)
    return float(t.item())


def barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def build_target(args):
    from economize_b200.models.config import llama31_8b, tiny_llama
    from economize_b200.models.llama import CausalLM, init_weights

    cfg = llama31_8b() if args.model == "llama31_8b" else tiny_llama(head_dim=128, num_heads=2, num_kv_heads=1)
    return init_weights(CausalLM(cfg, torch.bfloat16, "cuda"), seed=0)


CACHE_DIR = os.environ.get("ECZ_BENCH_CACHE", "/tmp/economize_b200_bench")


def _cache_path(args, rank: int, world: int) -> str:
    key = (f"{args.model}-b{args.batch}-p{args.prompt_len}-n{args.new_tokens}-t{args.train_steps}x{args.train_rounds}"
           f"-r{rank}-w{world}-v4")
    return os.path.join(CACHE_DIR, f"drafter-{key}.pt")


def reference_module():
    """The installed reference package (``baseline/_ref``), or ``None``."""
    ref_dir = os.path.join(HERE, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_dir, "economize")):
        return None
    if ref_dir not in sys.path:
        sys.path.insert(0, ref_dir)
    try:
        import economize

        return economize
    except Exception:
        return None


def hf_twin(target):
    """A ``transformers`` Llama with the target's weights (bf16, on the GPU)."""
    import transformers

    hcfg = target.config.to_hf()
    with torch.device("cuda"):
        hf = transformers.LlamaForCausalLM(hcfg).to(torch.bfloat16).eval()
    hf.load_state_dict(target.hf_state_dict())
    return hf


def plain_continuations_ref(ref, hf, prompts, new_tokens):
    model = ref.apply(hf)
    out = model.decode_batch(list(prompts), new_tokens, decoding=ref.DecodeConfig(cycle_length=1))
    rows = torch.stack([torch.cat([p, r.tokens.to(p.device)]) for p, r in zip(prompts, out)])
    model.detach()
    return rows


def build_drafter(target, args, rank: int, world: int, prompts, hf=None):
    """EAGLE-3 head weights shared by both arms, in the reference's parameter names.

    The random-init target's greedy continuation is chaotic, so a drafter can only be accurate where it has seen
    the continuation: it is trained (``--train-steps``) on the plain greedy continuations of the benchmark prompts
    produced by BOTH implementations (each arm's own bf16 rounding leads to its own trajectory), starting from an
    early-exit initialisation (fc picks the highest feature, the layer passes it through, the head is the target's
    restricted to the 32000 most frequent continuation tokens). The result is cached on the box, so the arm that
    runs second loads exactly the weights the first one trained.
    """
    import economize_b200 as eco
    from economize_b200.techniques.eagle3 import Eagle3Config
    from economize_b200.techniques.eagle3.formats import from_reference_state, to_reference_state

    vocab = min(32000, target.config.vocab_size)
    em = eco.apply(target, Eagle3Config(draft_vocab=vocab))
    tech = em.techniques["eagle3"]
    path = _cache_path(args, rank, world)
    if os.path.exists(path):
        from_reference_state(tech, torch.load(path, map_location="cuda", weights_only=True))
        return em, to_reference_state(tech)
    tech.reset_parameters(seed=1, identity=True)
    if args.train_steps > 0:
        from economize_b200.train import fit

        def with_prompts(results):
            return torch.stack([torch.cat([p, r.tokens.to(p.device)]) for p, r in zip(prompts, results)])

        plain = em.decode_batch(list(prompts), args.new_tokens,
                                decoding=eco.DecodeConfig(cycle_length=1, cuda_graphs=True))
        data = with_prompts(plain)
        ref = reference_module()
        ref_model = None
        own_hf = False
        if ref is not None:
            own_hf = hf is None
            hf = hf if hf is not None else hf_twin(target)
            try:
                from economize.techniques.eagle3 import Eagle3Config as RefEagle3Config

                ref_model = ref.apply(hf, RefEagle3Config(draft_vocab=vocab, param_dtype="model"))
                ref_cfg = ref.DecodeConfig(cycle_length=TREE["depth"] + 1, draft_policy="dynamic_tree",
                                           draft_policy_options=dict(TREE), cuda_graphs=True)
            except Exception as err:
                print(f"[bench] reference drafter unavailable for training rows ({err})", file=sys.stderr)

        def ref_trajectories():
            ref_tech = ref_model.techniques["eagle3"]
            cur = ref_tech.state_dict()
            ref_tech.load_state_dict({k: v.to(cur[k].device, cur[k].dtype)
                                      for k, v in to_reference_state(tech).items()})
            return with_prompts(ref_model.decode_batch(list(prompts), args.new_tokens, decoding=ref_cfg))

        tech.draft_vocab_from(data[:, args.prompt_len:])
        if ref_model is not None:  # the reference's own greedy trajectory (its tree path, untrained drafter)
            data = torch.cat([data, ref_trajectories()])
            tech.extend_draft_vocab(data[:, args.prompt_len:], data[:1, args.prompt_len:])
        # bf16 tree verification rounds differently from one-token passes and the random target is chaotic, so
        # every implementation's speculative trajectory drifts from its plain one; each round adds the
        # trajectories the current drafter produces in both implementations.
        rounds = max(1, args.train_rounds)
        for rnd in range(rounds):
            fit(em, data, steps=max(1, args.train_steps // rounds), batch_size=min(4, data.shape[0]), seed=rnd,
                lr=1e-3, warmup_steps=5, log_every=max(1, args.train_steps))
            if rnd + 1 < rounds:
                seen = data[:, args.prompt_len:]
                new = [with_prompts(em.decode_batch(list(prompts), args.new_tokens, decoding=decode_config(args)))]
                if ref_model is not None:
                    new.append(ref_trajectories())
                data = torch.cat([data, *new])
                tech.extend_draft_vocab(data[:, args.prompt_len:], seen)
        if ref_model is not None:
            ref_model.detach()
        if own_hf:
            del hf
            torch.cuda.empty_cache()
    state = to_reference_state(tech)
    os.makedirs(CACHE_DIR, exist_ok=True)
    tmp = path + f".{os.getpid()}.tmp"
    torch.save({k: v.cpu() for k, v in state.items()}, tmp)
    os.replace(tmp, path)
    return em, state


def prompts_for(args, rank: int, vocab: int, device) -> torch.Tensor:
    g = torch.Generator().manual_seed(1234 + rank)
    return torch.randint(0, vocab, (args.batch, args.prompt_len), generator=g).to(device)


def decode_config(args):
    import economize_b200 as eco

    return eco.DecodeConfig(cycle_length=TREE["depth"] + 1, draft_policy="dynamic_tree",
                            draft_policy_options=dict(TREE), cuda_graphs=not args.no_graphs)


def acceptance(rows) -> tuple[int, int]:
    """(accepted drafts, verified cycles) over the rows of one step, for either implementation's results."""
    accepted = cycles = 0
    for r in rows:
        if hasattr(r, "acceptance"):  # the reference: one (drafted, accepted) pair per cycle
            accepted += sum(a for _, a in r.acceptance)
            cycles += len(r.acceptance)
        else:
            accepted += r.accepted
            cycles += r.cycles
    return accepted, cycles


def count_launches(step) -> int:
    """Kernels of this package launched by one step (CUPTI trace of an extra, untimed step)."""
    from torch.profiler import ProfilerActivity, profile

    names = ("ecz::", "gemm_swapab", "attn_tc", "attn_merge", "rmsnorm_kernel", "rope_store", "silu_mul",
             "argmax_kernel", "greedy_accept", "kv_compact", "splitk_reduce")
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step()
        torch.cuda.synchronize()
    count = 0
    for ev in prof.events():
        if ev.device_type == torch.autograd.DeviceType.CUDA and any(n in ev.name for n in names):
            count += 1
    return count


def run_ours(args, world, rank):
    target = build_target(args)
    vocab = target.config.vocab_size
    if args.parallel == "tp" and world > 1:
        return run_ours_tp(args, world, rank, target)
    prompts = prompts_for(args, rank, vocab, "cuda")
    em, _ = build_drafter(target, args, rank, world, prompts)
    cfg = decode_config(args)
    rows = list(prompts)
    results = {"cfg": cfg}

    def step():
        results["r"] = em.decode_batch(rows, args.new_tokens, decoding=cfg)

    return em, step, results, prompts


def run_ours_tp(args, world, rank, target):
    """One request stream served by all ranks: the target sharded over them, the drafter replicated."""
    import torch.distributed as dist

    from economize_b200.distributed import TPGroup, tensor_parallel

    prompts = prompts_for(args, 0, target.config.vocab_size, "cuda")  # the same stream on every rank
    if rank == 0:
        em, state = build_drafter(target, args, 0, 1, prompts)
    dist.barrier()
    if rank != 0:
        em, state = build_drafter(target, args, 0, 1, prompts)  # loads rank 0's cached weights
    tech = em.techniques["eagle3"]
    # bit-identical drafters on every rank (every rank must draft the same tree)
    for tensor in tech.state_dict().values():
        dist.broadcast(tensor, src=0)
    tensor_parallel(em, TPGroup(rank, world), fused=not args.nccl_tp)
    cfg = decode_config(args)
    rows = list(prompts)
    results = {"cfg": cfg}

    def step():
        results["r"] = em.decode_batch(rows, args.new_tokens, decoding=cfg)

    return em, step, results, prompts


def run_reference(args, world, rank):
    ref = reference_module()
    if ref is None:
        return None, "reference not importable from baseline/_ref"
    if args.parallel == "tp" and world > 1:
        return None, ("the reference's tensor parallelism loads a checkpoint from disk with transformers' "
                      "tp_plan='auto'; this benchmark's random-init weights exist only in memory")
    from economize.techniques.eagle3 import Eagle3Config as RefEagle3Config

    target = build_target(args)
    vocab = target.config.vocab_size
    prompts = prompts_for(args, rank, vocab, "cuda")
    hf = hf_twin(target)
    _, dstate = build_drafter(target, args, rank, world, prompts, hf=hf)
    del target, _
    torch.cuda.empty_cache()
    model = ref.apply(hf, RefEagle3Config(draft_vocab=min(32000, vocab), param_dtype="model"))
    tech = model.techniques["eagle3"]
    current = tech.state_dict()
    tech.load_state_dict({k: v.to(current[k].device, current[k].dtype) for k, v in dstate.items()}, strict=True)
    cfg = ref.DecodeConfig(cycle_length=TREE["depth"] + 1, draft_policy="dynamic_tree",
                           draft_policy_options=dict(TREE), cuda_graphs=not args.no_graphs)
    rows = list(prompts)
    results = {"cfg": cfg}

    def step():
        results["r"] = model.decode_batch(rows, args.new_tokens, decoding=cfg)

    return (model, step, results, prompts), None


def main() -> None:
    args = parse()
    sys.path.insert(0, HERE)
    if not torch.cuda.is_available():
        print(json.dumps({"metric": METRIC, "unavailable": "no CUDA device"}))
        return
    world, rank, local = setup_dist(args)
    if args.impl == "reference":
        built, why = run_reference(args, world, rank)
        if built is None:
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": why}))
            return
        model, step, results, prompts = built
    else:
        model, step, results, prompts = run_ours(args, world, rank)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        torch.cuda.synchronize()
        barrier(world)
        start.record()
        for _ in range(args.steps):
            step()
        end.record()
        torch.cuda.synchronize()
        barrier(world)
    ms = start.elapsed_time(end) / args.steps
    ms_max = reduce_max(ms, world)
    streams = 1 if (args.parallel == "tp" and world > 1) else world
    new_tokens = args.batch * args.new_tokens * streams
    value = new_tokens / (ms_max / 1e3)
    accepted, cycles = acceptance(results["r"])
    tau_local = 1.0 + accepted / cycles if cycles else None

    # ---- end to end through the public API: pinned host prompts in, host tokens out ----
    host_prompts = [p.cpu().pin_memory() for p in prompts]
    e2e_steps = max(1, min(args.steps, 3))
    torch.cuda.synchronize()
    barrier(world)
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        if args.impl == "reference":
            out = model.decode_batch([p.to("cuda", non_blocking=True) for p in host_prompts], args.new_tokens,
                                     decoding=results["cfg"])
        else:
            out = model.decode_batch(host_prompts, args.new_tokens, decoding=results["cfg"])
        toks = [r.tokens.cpu() for r in out]
    torch.cuda.synchronize()
    e2e_ms = reduce_max((time.perf_counter() - t0) * 1e3 / e2e_steps, world)
    launches = None
    if args.impl == "ours":
        try:
            launches = count_launches(step) * args.steps
        except Exception:
            launches = None
    tau = None
    if tau_local is not None:
        tau = reduce_sum(tau_local, world) / world
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_max, 3), "higher_is_better": True,
            "scaling": "strong" if (args.parallel == "tp" and world > 1) else "weak",
            "vs_baseline": (value / BASELINE_TOKS) if BASELINE_TOKS else None, "dtype": "bf16",
            "data": "synthetic (uniform-random prompts, random-init weights)",
            "mean_accepted_len": round(tau, 4) if tau is not None else None,
            "config": {"model": "Llama-3.1-8B arch" if args.model == "llama31_8b" else "tiny",
                       "drafter": "EAGLE-3 (draft vocab 32000), dynamic tree depth 6 topk 10 nodes 60; trained "
                                  f"{args.train_steps} steps in {args.train_rounds} rounds on the greedy and "
                                  "speculative trajectories of both implementations on the benchmark prompts (same "
                                  "weights in both arms)",
                       "global_batch": args.batch * streams, "seq_len": args.prompt_len,
                       "new_tokens": args.new_tokens,
                       "parallelism": (f"tp{world}" + ("-nccl" if args.nccl_tp else "-fused"))
                       if (args.parallel == "tp" and world > 1) else f"dp{world}",
                       "train_steps": args.train_steps, "cuda_graphs": not args.no_graphs,
                       "l2": "weights (16 GB) exceed L2; no flush"},
            "clocks": clocks.summary(),
            "e2e": {"value": round(new_tokens / (e2e_ms / 1e3), 2), "unit": "tok/s",
                    "h2d_bytes_per_step": sum(p.numel() * p.element_size() for p in host_prompts) * streams,
                    "d2h_bytes_per_step": sum(t.numel() * t.element_size() for t in toks) * streams},
            "gpu_launches": launches,
        }
        if args.impl == "reference":
            line["impl"] = "reference"
        print(json.dumps(line))
    # release the captured graphs (they may hold NCCL calls) and the NVLink buffers before the group goes away
    engine_model = getattr(model, "model", None)
    if hasattr(model, "refresh"):
        model.refresh()
    tp = getattr(engine_model, "tp", None)
    if tp is not None and getattr(tp, "comm", None) is not None:
        tp.comm.close()
    results.clear()
    del step, model
    import gc

    gc.collect()
    torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
