"""Headline benchmark: decode tokens/s + mean accepted length, Llama-3.1-8B + EAGLE-3 dynamic tree on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch B] [--impl ours|reference] [--parallel tp|dp]

One *step* generates ``--new-tokens`` (256) tokens after uniform-random prompts of ``--prompt-len`` (512) tokens for
``--batch`` rows through the public API (``decode_batch``), prefill included. The target is a random-init
Llama-3.1-8B architecture (bf16, N(0, 0.02), seed 0) and the drafter an EAGLE-3 head (draft vocabulary 32000).
Decoding: dynamic tree, depth 6, top-k 10, 60 nodes, CUDA graphs.

Both arms build the same target weights and the same drafter initialisation with the plain PyTorch code of this
file, then each trains its drafter with its OWN ``train.fit`` on its OWN target's greedy continuations of the
benchmark prompts (the same recipe: steps, rounds, batch, learning rate), so neither arm runs the other's code.
``--impl reference`` imports only the unmodified reference (``baseline/_ref``) and ``transformers``.

With N > 1 GPUs (launched by torchrun) the default is tensor parallelism: one request stream served by all ranks
(``scaling`` "strong"); ``--parallel dp`` runs one replica per GPU instead ("weak"). The step time is the max over
ranks of the CUDA-event time; ``value`` is the whole job's generated tokens per second. The model weights (16 GB)
exceed L2, so every step streams them from HBM (no flush needed).
"""

from __future__ import annotations

import argparse
import glob
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
DRAFT_VOCAB = 32000


def parse() -> argparse.Namespace:
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--batch", type=int, default=1)
    p.add_argument("--prompt-len", type=int, default=512)
    p.add_argument("--new-tokens", type=int, default=256)
    p.add_argument("--train-steps", type=int, default=600)
    p.add_argument("--train-rounds", type=int, default=3)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--model", choices=("llama31_8b", "tiny"), default="llama31_8b")
    p.add_argument("--no-graphs", action="store_true")
    p.add_argument("--parallel", choices=("dp", "tp"), default=None,
                   help="dp: one replica per GPU; tp: one model sharded over all GPUs (default with N > 1)")
    p.add_argument("--nccl-tp", action="store_true", help="with tp: NCCL all-reduces instead of the fused kernels")
    p.add_argument("--attn", default=None, help="reference arm: attention implementation (default: economize's "
                   "own kernel, falling back to sdpa, then eager, if it cannot run)")
    p.add_argument("--config", type=int, choices=(1, 2, 3, 4, 5), default=2,
                   help="BASELINE.json configuration: 2 (default) is the headline; 1, 3, 4 and 5 run the "
                   "compositions of economize_b200.bench.configs (this package's arm only)")
    p.add_argument("--scale", choices=("full", "tiny"), default="full",
                   help="configs 3-5: the named architecture, or a small one of the same composition")
    args = p.parse_args()
    if args.parallel is None:
        args.parallel = "tp" if int(os.environ.get("WORLD_SIZE", "1")) > 1 else "dp"
    return args


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


# ---- process group ---------------------------------------------------------------------------------------------

def setup_dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=900),
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


# ---- shared by both arms: plain PyTorch + transformers only ------------------------------------------------------

def hf_config(model: str):
    """The ``transformers`` config of the benchmark architecture."""
    import transformers

    if model == "tiny":
        return transformers.LlamaConfig(vocab_size=1024, hidden_size=256, intermediate_size=688, num_hidden_layers=4,
                                        num_attention_heads=2, num_key_value_heads=1, head_dim=128,
                                        rms_norm_eps=1e-5, rope_theta=1e4, max_position_embeddings=4096,
                                        tie_word_embeddings=False)
    return transformers.LlamaConfig(
        vocab_size=128256, hidden_size=4096, intermediate_size=14336, num_hidden_layers=32, num_attention_heads=32,
        num_key_value_heads=8, head_dim=128, rms_norm_eps=1e-5, rope_theta=500000.0,
        rope_scaling={"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                      "original_max_position_embeddings": 8192},
        max_position_embeddings=131072, tie_word_embeddings=False)


@torch.no_grad()
def build_hf_target(model: str, attn: str = "sdpa"):
    """A ``transformers`` Llama on the GPU with the benchmark weights: every matrix N(0, 0.02) drawn in bf16-rounded
    fp32 from one CUDA generator (seed 0) in state-dict name order, norms at one."""
    import transformers

    cfg = hf_config(model)
    cfg._attn_implementation = attn
    with torch.device("meta"):
        hf = transformers.LlamaForCausalLM(cfg)
    hf = hf.to_empty(device="cuda").to(torch.bfloat16)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(0)
    for name, p in sorted(hf.named_parameters()):
        if p.dim() >= 2:
            p.copy_(torch.randn(p.shape, generator=gen, device="cuda", dtype=torch.float32).mul_(0.02))
        else:
            p.fill_(1.0)
    # the rotary inverse frequencies (non-persistent buffers, left empty by the meta construction): recomputed in
    # fp32 exactly as the module's constructor does
    emb = hf.model.rotary_emb
    fresh = type(emb)(emb.config, device="cuda")
    emb.register_buffer("inv_freq", fresh.inv_freq, persistent=False)
    emb.register_buffer("original_inv_freq", fresh.original_inv_freq, persistent=False)
    emb.attention_scaling = fresh.attention_scaling
    return hf.eval()


def prompts_for(args, stream: int, vocab: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(1234 + stream)
    return torch.randint(0, vocab, (args.batch, args.prompt_len), generator=g).to("cuda")


def draft_vocab_ids(tokens: torch.Tensor, vocab: int, k: int) -> torch.Tensor:
    """EAGLE-3's draft vocabulary: the ``k`` most frequent ids of ``tokens`` (ties and unseen ids in id order),
    returned in ascending id order."""
    counts = torch.bincount(tokens.reshape(-1).long().cpu(), minlength=vocab)[:vocab].double()
    order = torch.argsort(-counts * vocab + torch.arange(vocab, dtype=torch.float64), stable=True)
    return order[:k].sort().values


@torch.no_grad()
def eagle3_init_state(shapes: dict[str, tuple], lm_head: torch.Tensor, ids: torch.Tensor) -> dict[str, torch.Tensor]:
    """The drafter's starting weights in economize's EAGLE-3 parameter names: an early exit of the target (``fc``
    selects the highest fused feature, the attention and MLP output maps are zero, the head is the target's head
    restricted to the draft vocabulary), the other matrices N(0, 0.02) from a CUDA generator (seed 1)."""
    gen = torch.Generator(device="cuda")
    gen.manual_seed(1)
    out: dict[str, torch.Tensor] = {}
    for name in sorted(shapes):
        shape = shapes[name]
        if name == "d2t":
            out[name] = (ids.to("cuda") - torch.arange(ids.numel(), device="cuda")).to(torch.int64)
        elif name == "t2d":
            t2d = torch.zeros(shape, dtype=torch.bool, device="cuda")
            t2d[ids.to("cuda")] = True
            out[name] = t2d
        elif name == "fc.weight":
            h = shape[0]
            fc = torch.zeros(shape, dtype=torch.bfloat16, device="cuda")
            fc[:, -h:] = torch.eye(h, dtype=torch.bfloat16, device="cuda")
            out[name] = fc
        elif name == "lm_head.weight":
            out[name] = lm_head[ids.to(lm_head.device)].to(torch.bfloat16).contiguous()
        elif len(shape) >= 2:
            w = torch.randn(shape, generator=gen, device="cuda", dtype=torch.float32).mul_(0.02)
            if name.endswith(("o_proj.weight", "down_proj.weight")):
                w.zero_()
            out[name] = w.to(torch.bfloat16)
        elif name.endswith(".bias"):
            out[name] = torch.zeros(shape, dtype=torch.bfloat16, device="cuda")
        else:
            out[name] = torch.ones(shape, dtype=torch.bfloat16, device="cuda")
    return out


def with_prompts(prompts, results) -> torch.Tensor:
    return torch.stack([torch.cat([p, r.tokens.to(p.device)]) for p, r in zip(prompts, results)])


CACHE_DIR = os.environ.get("ECZ_BENCH_CACHE", "/tmp/economize_b200_bench")


def _cache_path(args, impl: str, stream: int) -> str:
    key = (f"{impl}-{args.model}-b{args.batch}-p{args.prompt_len}-n{args.new_tokens}-t{args.train_steps}"
           f"x{args.train_rounds}-s{stream}-v5")
    return os.path.join(CACHE_DIR, f"drafter-{key}.pt")


def train_drafter(arm, args, prompts, path: str, log) -> None:
    """The drafter recipe, identical for both arms: the draft vocabulary from the arm's own plain greedy
    continuations, the early-exit initialisation, then ``--train-rounds`` rounds of the arm's own ``fit``, each
    round adding the speculative trajectories the current drafter produces (a tree pass may round differently from
    a one-token pass, so a speculative trajectory can leave the plain one). Cached on the box per arm."""
    if os.path.exists(path):
        arm.load_state(torch.load(path, map_location="cuda", weights_only=True))
        log(f"drafter loaded from {path}")
        return
    t0 = time.perf_counter()
    data = with_prompts(prompts, arm.decode(prompts, plain=True))
    ids = draft_vocab_ids(data[:, args.prompt_len:], arm.vocab, min(DRAFT_VOCAB, arm.vocab))
    arm.load_state(eagle3_init_state(arm.state_shapes(), arm.lm_head(), ids))
    rounds = max(1, args.train_rounds)
    for rnd in range(rounds if args.train_steps > 0 else 0):
        arm.fit(data, steps=max(1, args.train_steps // rounds), seed=rnd)
        if rnd + 1 < rounds:
            spec = with_prompts(prompts, arm.decode(prompts, plain=False))
            fresh = [row for row in spec if not any(torch.equal(row, old) for old in data)]
            if fresh:
                data = torch.cat([data, torch.stack(fresh)])
    state = {k: v.detach().cpu() for k, v in arm.state().items()}
    os.makedirs(CACHE_DIR, exist_ok=True)
    tmp = path + f".{os.getpid()}.tmp"
    torch.save(state, tmp)
    os.replace(tmp, path)
    log(f"drafter trained: {args.train_steps} steps, {data.shape[0]} rows, {time.perf_counter() - t0:.1f} s")


# ---- the reference arm: the unmodified reference only -----------------------------------------------------------

def import_reference():
    """``(economize, None)`` from ``baseline/_ref`` (a ``pip --target`` install, a source tree or a site-packages
    layout), else ``(None, why)``."""
    ref_dir = os.path.join(HERE, "baseline", "_ref")
    if not os.path.isdir(ref_dir):
        return None, f"{ref_dir} does not exist (install the reference there)"
    roots = [ref_dir, os.path.join(ref_dir, "src")]
    roots += sorted(glob.glob(os.path.join(ref_dir, "lib", "python*", "site-packages")))
    roots += sorted(glob.glob(os.path.join(ref_dir, "lib64", "python*", "site-packages")))
    found = [r for r in roots if os.path.isfile(os.path.join(r, "economize", "__init__.py"))]
    if not found:
        return None, f"no economize package under {ref_dir} (looked in {', '.join(roots)})"
    sys.path.insert(0, found[0])
    try:
        import economize
    except Exception as err:  # the reason goes into the unavailable line
        return None, f"import economize from {found[0]} failed: {type(err).__name__}: {err}"
    if not os.path.abspath(economize.__file__).startswith(os.path.abspath(ref_dir)):
        return None, f"economize resolved to {economize.__file__}, not the copy in {ref_dir}"
    return economize, None


class RefArm:
    """The reference (economize on ``transformers``) behind the recipe's interface."""

    def __init__(self, ref, hf, args) -> None:
        from economize.techniques.eagle3 import Eagle3Config

        self.ref, self.hf, self.args = ref, hf, args
        self.vocab = hf.config.vocab_size
        self.model = ref.apply(hf, Eagle3Config(draft_vocab=min(DRAFT_VOCAB, self.vocab), param_dtype="model"))
        self.tech = self.model.techniques["eagle3"]
        self.spec_cfg = ref.DecodeConfig(cycle_length=TREE["depth"] + 1, draft_policy="dynamic_tree",
                                         draft_policy_options=dict(TREE), cuda_graphs=not args.no_graphs)
        self.plain_cfg = ref.DecodeConfig(cycle_length=1, cuda_graphs=not args.no_graphs)

    def decode(self, prompts, plain: bool):
        return self.model.decode_batch(list(prompts), self.args.new_tokens,
                                       decoding=self.plain_cfg if plain else self.spec_cfg)

    def state_shapes(self):
        return {k: tuple(v.shape) for k, v in self.tech.state_dict().items()}

    def lm_head(self):
        w = self.hf.lm_head.weight
        return w.full_tensor() if hasattr(w, "full_tensor") else w  # a tp_plan-sharded head is gathered

    def state(self):
        return self.tech.state_dict()

    def load_state(self, state):
        cur = self.tech.state_dict()
        self.tech.load_state_dict({k: v.to(cur[k].device, cur[k].dtype) for k, v in state.items()}, strict=True)

    def fit(self, data, steps: int, seed: int):
        from economize.train import fit

        fit(self.model, data, steps=steps, batch_size=min(4, data.shape[0]), seed=seed, lr=1e-3, warmup_steps=10,
            log_every=max(1, steps))


def run_reference(args, world, rank, log):
    ref, why = import_reference()
    if ref is None:
        return None, why
    if args.parallel == "tp" and world > 1:
        return run_reference_tp(ref, args, world, rank, log)
    import economize.attention

    economize.attention.install()
    prompts = prompts_for(args, rank, hf_config(args.model).vocab_size)
    errors = []
    for attn in ([args.attn] if args.attn else ["economize", "sdpa", "eager"]):
        hf = build_hf_target(args.model, attn)
        arm = RefArm(ref, hf, args)
        try:  # the implementation must serve a tree cycle and a plain step on this box
            arm.decode(prompts[:, :64], plain=False)
            arm.decode(prompts[:, :64], plain=True)
        except Exception as err:
            errors.append(f"{attn}: {type(err).__name__}: {str(err)[:200]}")
            log(f"reference attention {attn!r} cannot run: {err}")
            arm.model.detach()
            del arm, hf
            torch.cuda.empty_cache()
            continue
        arm.attn = attn
        break
    else:
        return None, "reference decoding failed with every attention implementation: " + " | ".join(errors)
    train_drafter(arm, args, prompts, _cache_path(args, "reference", rank), log)
    rows = list(prompts)
    results = {"cfg": arm.spec_cfg, "attn": arm.attn, "streams": world}

    def step():
        results["r"] = arm.model.decode_batch(rows, args.new_tokens, decoding=arm.spec_cfg)

    return (arm.model, step, results, prompts), None


def run_reference_tp(ref, args, world, rank, log):
    """The reference's tensor parallelism: ``transformers``' ``tp_plan="auto"`` through
    ``economize.distributed.tp.load_tensor_parallel`` on a checkpoint of the benchmark weights (written once on the
    box), with the drafter the 1-GPU reference run trained (or trained here)."""
    import torch.distributed as dist

    import economize.attention
    from economize.distributed.tp import load_tensor_parallel

    economize.attention.install()
    ckpt = os.path.join(CACHE_DIR, f"hf-{args.model}")
    if rank == 0 and not os.path.isfile(os.path.join(ckpt, "config.json")):
        hf = build_hf_target(args.model, "sdpa")
        os.makedirs(CACHE_DIR, exist_ok=True)
        hf.save_pretrained(ckpt + f".{os.getpid()}")
        os.replace(ckpt + f".{os.getpid()}", ckpt)
        del hf
        torch.cuda.empty_cache()
    dist.barrier()
    errors = []
    for attn in ([args.attn] if args.attn else ["economize", "sdpa"]):
        try:
            hf = load_tensor_parallel(ckpt, dtype=torch.bfloat16, attn_implementation=attn)
            arm = RefArm(ref, hf, args)
            prompts = prompts_for(args, 0, arm.vocab)
            arm.decode(prompts[:, :64], plain=False)
        except Exception as err:
            errors.append(f"{attn}: {type(err).__name__}: {str(err)[:200]}")
            continue
        arm.attn = attn
        break
    else:
        return None, "reference tensor-parallel decoding failed: " + " | ".join(errors)
    try:  # the recipe on the sharded model, on every rank (the reference's fit joins its collectives on all)
        train_drafter(arm, args, prompts, _cache_path(args, "reference", 0) + f".tp{world}", log)
    except Exception as err:
        return None, f"reference drafter training on a tensor-parallel model failed: {type(err).__name__}: {err}"
    rows = list(prompts)
    results = {"cfg": arm.spec_cfg, "attn": arm.attn, "streams": 1}

    def step():
        results["r"] = arm.model.decode_batch(rows, args.new_tokens, decoding=arm.spec_cfg)

    return (arm.model, step, results, prompts), None


# ---- our arm ------------------------------------------------------------------------------------------------------

class OursArm:
    def __init__(self, target, args) -> None:
        import economize_b200 as eco
        from economize_b200.techniques.eagle3 import Eagle3Config

        self.eco, self.args = eco, args
        self.target = target
        self.full_head = target.head_weight.detach()  # kept whole: sharding replaces the parameter's data
        self.vocab = target.config.vocab_size
        self.model = eco.apply(target, Eagle3Config(draft_vocab=min(DRAFT_VOCAB, self.vocab)))
        self.tech = self.model.techniques["eagle3"]
        self.spec_cfg = eco.DecodeConfig(cycle_length=TREE["depth"] + 1, draft_policy="dynamic_tree",
                                         draft_policy_options=dict(TREE), cuda_graphs=not args.no_graphs)
        self.plain_cfg = eco.DecodeConfig(cycle_length=1, cuda_graphs=not args.no_graphs)

    def decode(self, prompts, plain: bool):
        return self.model.decode_batch(list(prompts), self.args.new_tokens,
                                       decoding=self.plain_cfg if plain else self.spec_cfg)

    def state_shapes(self):
        from economize_b200.techniques.eagle3.formats import to_reference_state

        return {k: tuple(v.shape) for k, v in to_reference_state(self.tech).items()}

    def lm_head(self):
        return self.full_head

    def state(self):
        from economize_b200.techniques.eagle3.formats import to_reference_state

        return to_reference_state(self.tech)

    def load_state(self, state):
        from economize_b200.techniques.eagle3.formats import from_reference_state

        from_reference_state(self.tech, state)

    def fit(self, data, steps: int, seed: int):
        from economize_b200.train import fit

        fit(self.model, data, steps=steps, batch_size=min(4, data.shape[0]), seed=seed, lr=1e-3, warmup_steps=10,
            log_every=max(1, steps))


def build_target(args):
    from economize_b200.models.llama import CausalLM

    hf = build_hf_target(args.model)
    target = CausalLM.from_hf(hf)
    del hf
    torch.cuda.empty_cache()
    return target


def run_ours(args, world, rank, log):
    target = build_target(args)
    tp = args.parallel == "tp" and world > 1
    stream = 0 if tp else rank
    prompts = prompts_for(args, stream, target.config.vocab_size)
    arm = OursArm(target, args)
    if tp:
        import torch.distributed as dist

        from economize_b200.distributed import TPGroup, tensor_parallel

        # the recipe runs on the sharded model: a sharded target sums its partials in another order than one GPU,
        # so its greedy trajectory (what the drafter learns) is its own. Every rank runs the same steps on the same
        # stream (train.fit averages the identical gradients over the ranks, so no rank waits alone in a
        # collective), then rank 0's weights are broadcast
        tensor_parallel(arm.model, TPGroup(rank, world), fused=not args.nccl_tp)
        train_drafter(arm, args, prompts, _cache_path(args, "ours", 0) + f".tp{world}" +
                      ("-nccl" if args.nccl_tp else ""), log)
        dist.barrier()
        for tensor in arm.tech.state_dict().values():  # bit-identical drafters: every rank drafts the same tree
            dist.broadcast(tensor, src=0)
    else:
        train_drafter(arm, args, prompts, _cache_path(args, "ours", stream), log)
    rows = list(prompts)
    results = {"cfg": arm.spec_cfg, "streams": 1 if tp else world, "plain_cfg": arm.plain_cfg}

    def step():
        results["r"] = arm.model.decode_batch(rows, args.new_tokens, decoding=arm.spec_cfg)

    return arm.model, step, results, prompts


CONFIG_METRICS = {
    1: "CPU fp32 plumbing: tiny Llama + EAGLE-3 chain of 4, tokens equal plain greedy",
    3: "decode tok/s + mean accepted len, Llama-3.1-70B arch ShortGPT-8 int4 g128 fp8-KV int8-EAGLE-3, TP=8",
    4: "decode tok/s + mean accepted len, Mixtral-8x7B-style MoE block-fp8 + Medusa-4, EP=8",
    5: "decode tok/s + mean accepted len, 128K context KIVI-2 + StreamingLLM draft view + 1B draft on another GPU",
}


def run_config(args, world, rank, log):
    """Configurations 1, 3, 4 and 5 (economize_b200.bench.configs) through this package's public API."""
    from economize_b200.bench import configs

    kw: dict = {}
    if args.config != 1:
        kw["scale"] = args.scale
        kw["device"] = "cuda"
    if args.config == 3 and world > 1:
        from economize_b200.distributed import TPGroup

        kw["tp"] = TPGroup(rank, world)
    if args.config == 4 and world > 1:
        from economize_b200.parallel.moe import FusedExpertParallel

        kw["ep"] = FusedExpertParallel(rank, world, max_tokens=4096)
    if args.config == 5 and torch.cuda.device_count() > 1:
        kw["draft_device"] = f"cuda:{(torch.cuda.current_device() + 1) % torch.cuda.device_count()}"
    if args.config == 1:
        kw["device"] = "cuda"
    spec = configs.build(args.config, **kw)
    log(f"{spec.name}: {spec.notes}")
    args.batch, args.new_tokens = len(spec.prompts), spec.new_tokens
    args.prompt_len = int(spec.prompts[0].numel())
    import economize_b200 as eco

    results = {"cfg": spec.decoding, "streams": 1 if args.config == 3 else world,
               "plain_cfg": eco.DecodeConfig(cycle_length=1), "spec": spec}

    def step():
        results["r"] = spec.step()

    return spec.model, step, results, spec.prompts


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

    names = ("ecz::", "gemm_", "attn_", "rmsnorm_kernel", "rope_store", "silu_mul", "argmax_kernel",
             "greedy_accept", "kv_compact", "splitk_reduce", "topk_logp", "tree_", "push_", "reduce_rmsnorm")
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        step()
        torch.cuda.synchronize()
    count = 0
    for ev in prof.events():
        if ev.device_type == torch.autograd.DeviceType.CUDA and any(n in ev.name for n in names):
            count += 1
    return count


def main() -> None:
    args = parse()
    sys.path.insert(0, HERE)
    if not torch.cuda.is_available():
        out = {"metric": METRIC, "unavailable": "no CUDA device"}
        if args.impl == "reference":
            out["impl"] = "reference"
        print(json.dumps(out))
        return
    world, rank, local = setup_dist()

    def log(msg: str) -> None:
        print(f"[bench r{rank}] {msg}", file=sys.stderr, flush=True)

    tp = args.parallel == "tp" and world > 1
    if args.config != 2 and args.impl == "reference":
        if rank == 0:
            print(json.dumps({"impl": "reference", "metric": CONFIG_METRICS[args.config],
                              "unavailable": f"configuration {args.config} is a composition this bench drives "
                              "through this package only; the reference publishes no number for it"}))
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return
    if args.config != 2:
        model, step, results, prompts = run_config(args, world, rank, log)
        tp = args.config in (3, 4) and world > 1
    elif args.impl == "reference":
        built, why = run_reference(args, world, rank, log)
        ok = reduce_sum(0.0 if built is None else 1.0, world)
        if ok < world:  # every rank takes the same collective steps: all stop when one cannot run
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": why or "another rank could not build the "
                                  "reference"}))
            if world > 1:
                import torch.distributed as dist

                dist.destroy_process_group()
            return
        model, step, results, prompts = built
    else:
        model, step, results, prompts = run_ours(args, world, rank, log)

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
    streams = results["streams"]
    new_tokens = args.batch * args.new_tokens * streams
    value = new_tokens / (ms_max / 1e3)
    accepted, cycles = acceptance(results["r"])
    tau_local = 1.0 + accepted / cycles if cycles else 0.0
    spec_tokens = [r.tokens.cpu() for r in results["r"]]

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
    equal_plain = None
    if args.impl == "ours":
        try:
            launches = count_launches(step) * args.steps
        except Exception:
            launches = None
        # lossless check: the speculative tokens equal plain greedy decoding through the same engine
        plain = model.decode_batch(list(prompts), args.new_tokens, decoding=results["plain_cfg"])
        equal_plain = all(torch.equal(a, b.tokens.cpu()) for a, b in zip(spec_tokens, plain))
    tau = reduce_sum(tau_local, world) / world
    if rank == 0:
        parallelism = (f"tp{world}" + ("-nccl" if args.nccl_tp and args.impl == "ours" else
                                       "-fused" if args.impl == "ours" else "-hf-auto")) if tp else f"dp{world}"
        if args.config == 4 and world > 1:
            parallelism = f"ep{world}-fused"
        line = {
            "metric": METRIC if args.config == 2 else CONFIG_METRICS[args.config], "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_max, 3), "higher_is_better": True,
            "scaling": "strong" if tp else "weak",
            "vs_baseline": (value / BASELINE_TOKS) if BASELINE_TOKS else None, "dtype": "bf16",
            "data": "synthetic (uniform-random prompts, random-init weights)",
            "mean_accepted_len": round(tau, 4),
            "config": {"model": "Llama-3.1-8B arch" if args.model == "llama31_8b" else "tiny",
                       "drafter": f"EAGLE-3 (draft vocab {DRAFT_VOCAB}), dynamic tree depth 6 topk 10 nodes 60; "
                                  f"trained {args.train_steps} steps in {args.train_rounds} rounds by the arm's own "
                                  "train.fit on its own greedy and speculative trajectories of the benchmark prompts "
                                  "(same initialisation and recipe in both arms)",
                       "global_batch": args.batch * streams, "seq_len": args.prompt_len,
                       "new_tokens": args.new_tokens, "parallelism": parallelism,
                       "train_steps": args.train_steps, "cuda_graphs": not args.no_graphs,
                       "l2": "weights (16 GB) exceed L2; no flush"},
            "clocks": clocks.summary(),
            "e2e": {"value": round(new_tokens / (e2e_ms / 1e3), 2), "unit": "tok/s",
                    "h2d_bytes_per_step": sum(p.numel() * p.element_size() for p in host_prompts) * streams,
                    "d2h_bytes_per_step": sum(t.numel() * t.element_size() for t in toks) * streams},
            "gpu_launches": launches,
        }
        if equal_plain is not None:
            line["tokens_equal_plain_greedy"] = equal_plain
        if args.config != 2:
            spec = results["spec"]
            line["config"] = {"model": spec.name, "scale": args.scale if args.config != 1 else "fixed",
                              "global_batch": args.batch * streams, "seq_len": args.prompt_len,
                              "new_tokens": args.new_tokens, "parallelism": parallelism,
                              "cuda_graphs": bool(getattr(spec.decoding, "cuda_graphs", False)),
                              "l2": "weights exceed L2; no flush" if args.scale == "full" else
                                    "small model: weights fit in L2 (not a roofline number)",
                              **{k: v for k, v in spec.notes.items()}}
        if args.impl == "reference":
            line["impl"] = "reference"
            line["config"]["attn_implementation"] = results.get("attn")
        print(json.dumps(line), flush=True)
    # release the captured graphs (they may hold NCCL calls) and the NVLink buffers before the group goes away
    engine_model = getattr(model, "model", None)
    if hasattr(model, "refresh"):
        model.refresh()
    tpg = getattr(engine_model, "tp", None)
    for runtime in (getattr(tpg, "comm", None), getattr(tpg, "sp", None)):
        if runtime is not None:
            runtime.close()
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
